// Split frame kernel: a C-CTA thread-block cluster (C = 1, 2, 4 or 8) runs all
// 16 positions of a Local AR frame for a tile of up to 8 sessions (16 rows
// with CFG; or 16 sessions, 32 rows, on 2 CTAs), each CTA streaming 1/C of
// every weight matrix, with the GEMMs on
// the fifth-generation tensor cores (tcgen05.mma, accumulators in tensor
// memory).  C is picked per batch so that the tiles x C CTAs fill the device:
// fewer sessions per GPU means more CTAs per session and a shorter frame,
// which is what lets session sharding over more GPUs scale.
//
// Reference ops per position (as in frame_tile.cu: local_ar_wrapper.py:609-751,
// transformer_2501.py:405-442,761-851,1153-1232, sampling
// local_ar_plugins.cu:1211-1370, embedding sum main_decoder_wrapper.py:796-810),
// CTA c of the cluster, nh = 4 / C heads per CTA (C = 8: CTAs 2h and 2h + 1
// both compute head h, each sending 8 of its 16 rows):
//
//   input rows: p = 0 (or every p without the folded tables) the full
//     in-projection in every CTA, x = bf16(bf16(W_in h + b) + pos[p]);
//     p >= 1: x = bf16(emb_proj[p-1][token] + pos[p]) gathered by every CTA
//   LN1 (every CTA, all rows); q|k|v of heads [c nh, +nh); k/v appended to
//     this CTA's TMEM KV cache; attention for those heads;      exchange R1
//       (the heads' outputs to every CTA)
//   o-projection features [256c/C, +256/C) + residual;          exchange R2
//   LN2; FFN1 features [1024c/C, +1024/C) + GELU-tanh; FFN2 partial sums over
//     those features for all 256 outputs, scattered to the owners of the
//     output features (f32);                                     exchange R3
//   own features = the C partial sums in CTA order, + residual;  exchange R4
//   head p vocabulary [2048c/C, +2048/C) for all sessions (bias, CFG combine
//     with the plugin's two roundings, constraints); the other CTAs' sessions'
//     values and non-finite flags go to their owners;           exchange R5
//   one warp, or with C >= 4 a group of C warps, per owned session
//     (sessions [8c/C, +8/C)) samples it
//     (tile_common.cuh: sample_row, sample_group) and send the token to
//     every CTA                                                  exchange R6
//   (with C = 1 there are no exchanges).
//
// GEMMs (swap-AB): D[128 weight rows][R tile rows] = W[128][K] x X[R][K]^T
// on tcgen05.mma kind::f16 M=128 N=R K=16, A = a weight chunk in shared
// memory, B = the activation rows in shared memory, both K-major with the
// 128-byte swizzle; one thread issues, tcgen05.commit signals the weight
// slot free and the accumulator full.  A weight chunk is 128 rows x 128 K
// columns (32 KB) as four 64 x 64 TMA boxes (no multicast); its two 64-row
// halves may come from different places of the same matrix (a head's q and
// k rows, say), and a half that the CTA does not need repeats the first.
// Weights stream through a four-slot ring (three with 32-row tiles) filled
// by a producer warp that runs ahead across GEMMs and positions.  With
// 16-row tiles two accumulator buffers of 16 TMEM columns alternate by
// M-block, so the epilogue of one block overlaps the MMAs of the next; a
// 32-row tile has room for one 32-column buffer only.
//
// Tensor memory (512 columns x 128 lanes): the KV cache of positions 0..14
// of the CTA's heads, lane 32 q + 2 r + half = quadrant q (local head q, or
// with 32-row tiles head q / 2 and rows 16 (q mod 2)..), row r, head dims
// [32 half, +32); K of position j at columns 16 b(j), V at V0 + 16 b(j),
// b(j) = 8 (j mod 2) + j / 2.  Block b(15) is never written (position 15's
// k/v are read from shared memory).  16-row tiles: V0 = 256, so columns
// [240, 256) and [496, 512) are the two accumulator buffers; 32-row tiles:
// V0 = 240 and [480, 512) is the one buffer.
//
// Exchanges push data with st.async into the receivers' shared memory and
// complete on the receiver's round mbarrier, which the receiver arms with
// the bytes it expects (every CTA pushes to every other in every round); two
// barriers alternate by round parity.  Each round's pushes land in buffers
// the receiver does not read or write during the phase that precedes that
// round.  Every wait is
// bounded; a timeout sets invalid bit 4 for the CTA's sessions.
#include <cooperative_groups.h>
#include <cuda.h>

#include <mutex>

#include "frame_common.cuh"
#include "ptx.cuh"
#include "tile_common.cuh"

namespace cg = cooperative_groups;

namespace mtt {
namespace {

constexpr int kSW = 8;                     // consumer warps
constexpr int kSC = kSW * 32;              // consumer threads
constexpr int kSThreads = kSC + 128;       // + the control warpgroup (TMA producer warp, MMA warp)
constexpr int kSProducerRegs = 40;
constexpr int kSConsumerRegs = 232;
static_assert(128 * kSProducerRegs + kSC * kSConsumerRegs <= kSThreads * 168, "register split");
constexpr int kD = 256;
constexpr int kF = 1024;
constexpr int kHeads = 4;
constexpr int kMaxSlots = 4;
constexpr int kChunkRows = 128;
constexpr int kChunkK = 128;
constexpr int kPanelElems = kChunkRows * 64;      // one 128-row x 64-column swizzled panel (16 KB)
constexpr int kChunkElems = 2 * kPanelElems;      // 32 KB
constexpr uint32_t kChunkBytes = kChunkElems * 2;
constexpr int kBoxRows = 64;
constexpr int kLdX = kD + 8;
constexpr int kListBytes = 2 * (kListCap + 16) + 2 * kListCap;  // candidate list + eligible list (u16)

enum Gemm { G_IN = 0, G_QKV, G_O, G_F1, G_F2, G_HEAD };

// Tile geometry per cluster size C and tile rows R (16: 8 sessions, 32: 16
// sessions; R = 32 runs on 2-CTA clusters).
template <int C, int R>
struct Cfg {
  static constexpr int S = R / 2;             // session slots per tile
  static constexpr int nh = C <= kHeads ? kHeads / C : 1;  // heads per CTA (C = 8: a CTA pair shares one)
  static constexpr int att_rows = C <= kHeads ? R : R / 2;  // attention rows each CTA sends (C > 1)
  static constexpr int nq = (3 * nh + 1) / 2;  // qkv M-blocks (pairs of 64-row head groups)
  static constexpr int of = kD / C;          // o-projection / residual features per CTA
  static constexpr int no = of >= 128 ? of / 128 : 1;
  static constexpr int f1 = kF / C;          // FFN1 features per CTA = FFN2 K per CTA
  static constexpr int nf1 = f1 / 128;
  static constexpr int vs = 2048 / C;        // vocabulary slice per CTA (blocks of 128)
  static constexpr int nhb = vs / 128;
  static constexpr int own = S / C;          // sessions sampled per CTA
  static constexpr int ldq = 3 * nh * 64 + 8;
  static constexpr int qkv_elems = R * ldq;
  static constexpr int hid_elems = R * f1;   // FFN hidden as R-row panels
  static constexpr int op_panel = R * 64;    // one R-row x 64-column operand panel
  // The in-projection input (K = 768) is staged in pieces of 256 columns
  // with 32-row tiles (shared memory), whole with 16-row tiles.
  static constexpr int in_pieces = R == 32 ? 3 : 1;
  // Weight ring slots (32 KB each) and accumulator buffers (R TMEM columns
  // each).  The KV cache takes 480 of the 512 TMEM columns; with 16-row
  // tiles K and V keep 16-column gaps at 240 and 496 (two buffers), with
  // 32-row tiles V starts at column 240 and the one buffer is [480, 512).
  static constexpr int slots = R == 32 ? 3 : 4;
  static constexpr int nbuf = R == 32 ? 1 : 2;
  static constexpr uint32_t kv_v = R == 32 ? 240u : 256u;
  static constexpr uint32_t idesc = umma_idesc_bf16(128, R);
  // Warps per owned session in the sampler: a group of >= 4 warps shares one
  // session (sample_group); with 2 or more sessions per 4 warps each warp
  // samples its own (sample_row), which measured faster there.
  static constexpr int sw = kSW / own >= 4 ? kSW / own : 1;
  // FFN2 partial sums received: from every CTA (16-row tiles) or only from
  // the peers, the CTA's own partials staying in registers (32-row tiles).
  static constexpr int red_slots = C == 1 ? 1 : (R == 32 ? C - 1 : C);
  static_assert(R == 16 || (R == 32 && C == 2), "32-row tiles run on 2-CTA clusters");
  static_assert(nf1 >= 1 && nhb >= 1 && own >= 1, "split");
  __device__ static __forceinline__ uint32_t dcol(int db) { return R == 32 ? 480u : (db ? 496u : 240u); }
};

struct SplitMaps {
  CUtensorMap in_proj, qkv, o, ffn1, ffn2, head;
};

// Attention exchange between the two warps of a TMEM lane quadrant (scratch
// in the union).
struct SplitAttn {
  float s[2][kHeads][32][8];
  float o[kHeads][32][32];
};

template <int C, int R>
struct __align__(1024) SplitSmem {
  using K = Cfg<C, R>;
  bf16 ring[K::slots][kChunkElems];  // weight chunks (1024-byte aligned panels)
  bf16 xa[4 * K::op_panel];          // LN output (B operand); with 32-row tiles also the head
                                     // values of the other CTA's sessions before sending
  bf16 ab[4 * K::op_panel];          // attention output / residual stream copy (B operand)
  union U {
    bf16 src[(12 / K::in_pieces) * K::op_panel];  // in-projection input rows (B operand, K = 768 or a piece)
    SplitAttn att;                              // attention exchange
    bf16 hid[K::hid_elems];                     // FFN hidden slice (B operand)
    struct {
      uint16_t own[K::own][kVocab];             // constrained values of the owned sessions
      uint16_t out[C > 1 && R == 16 ? K::S : 1][C > 1 && R == 16 ? K::vs : 8];  // other sessions, before sending
    } v;
  } u;
  bf16 x[R * kLdX];  // residual stream (row-major)
  union Q {
    bf16 qkv[K::qkv_elems];                                  // q | k | v of the CTA's heads
    unsigned char lists[K::own][kListBytes];                 // sampler scratch (one warp per session)
    GroupScratch grp[K::own];                                // sampler scratch (warp groups)
  } q;
  float red[K::red_slots][R][C > 1 ? K::of : 1];  // FFN2 partial sums of the owned features, by sender
  __align__(16) bf16 hb[K::vs];                   // head p bias, this CTA's vocabulary slice
  int32_t tok[K::S][kPositions];
  int32_t sess[K::S];
  uint32_t flags[K::S];  // bit 0 unfinished, bit 1 finished, bit 2 forbid_eos
  uint32_t nf[K::S];     // non-finite guided logit in this CTA's vocabulary slice, per session
  uint32_t vmax[K::S];   // largest order key of this CTA's vocabulary slice, per session
  uint32_t peer_nf[C][K::own];  // from each peer: non-finite flag << 16 | its slice's largest key
  int64_t ctr[K::own];
  int64_t seed[K::own];
  int32_t inv[K::own];
  int32_t last_issued[kMaxSlots];
  int32_t n_sess;
  int32_t err;
  int32_t producer_done;
  int32_t mma_done;
  uint32_t tmem;
  unsigned long long full[kMaxSlots];
  unsigned long long empty[kMaxSlots];
  unsigned long long dfull[2];
  unsigned long long dempty[2];
  unsigned long long opready;
  unsigned long long srcfree;  // the MMAs have read an in-projection input piece
  unsigned long long mmafin;
  unsigned long long xbar[2];
};

template <int C, int R>
constexpr size_t split_smem_bytes() {
  return sizeof(SplitSmem<C, R>) + 1024;
}
static_assert(split_smem_bytes<1, 16>() <= 232448 && split_smem_bytes<2, 16>() <= 232448 &&
                  split_smem_bytes<4, 16>() <= 232448 && split_smem_bytes<8, 16>() <= 232448 &&
                  split_smem_bytes<2, 32>() <= 232448,
              "split kernel shared memory");

template <int C, int R>
__device__ __forceinline__ int err_flag(const SplitSmem<C, R>& sm) {
  return *reinterpret_cast<const volatile int*>(&sm.err);
}
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Phase clock stamp of the first CTA (library trace hook: mtt_b200_test_frame_trace).
__device__ __forceinline__ void s_stamp(const Frame& f, bool tracer, int p, int i) {
  if (tracer) f.trace[kPositions * p + i] = static_cast<uint64_t>(clock64());
}

// Byte offset of element (row r, column k) of an R-row operand stored as
// 64-column panels with the 128-byte swizzle.
template <int R>
__device__ __forceinline__ int op_off(int r, int k) {
  return (k >> 6) * (R * 128) + r * 128 + ((((k & 63) >> 3) ^ (r & 7)) << 4) + ((k & 7) << 1);
}
template <int R>
__device__ __forceinline__ void op_store(bf16* base, int r, int k, bf16 v) {
  *reinterpret_cast<bf16*>(reinterpret_cast<unsigned char*>(base) + op_off<R>(r, k)) = v;
}
// 16-byte unit (8 columns from k, k % 8 == 0).
template <int R>
__device__ __forceinline__ uint4* op_unit(bf16* base, int r, int k) {
  return reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(base) + op_off<R>(r, k));
}

// ---------------------------------------------------------------------------
// the per-position GEMM schedule (producer and MMA warp walk it in the same order)
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool has_in_projection(bool folded, int p) { return p == 0 || !folded; }

template <int C, int R>
__device__ __forceinline__ int gemm_blocks(int g) {
  using K = Cfg<C, R>;
  switch (g) {
    case G_IN: return 2;
    case G_QKV: return K::nq;
    case G_O: return K::no;
    case G_F1: return K::nf1;
    case G_F2: return 2;
    default: return K::nhb;
  }
}

template <int C, int R>
__device__ __forceinline__ int gemm_kchunks(int g) {
  return g == G_IN ? kEmbed / kChunkK : (g == G_F2 ? Cfg<C, R>::f1 / kChunkK : kD / kChunkK);
}

// First (global) head of CTA c: nh heads each, or with 8 CTAs head c / 2
// for the pair 2h, 2h + 1 (both compute it; each sends half of its rows).
template <int C, int R>
__device__ __forceinline__ int head_base(int c) {
  return C <= kHeads ? c * Cfg<C, R>::nh : c / 2;
}

// Weight rows of the head group gi (q groups, then k, then v; nh per type).
template <int C, int R>
__device__ __forceinline__ int qkv_group_row(int c, int gi) {
  using K = Cfg<C, R>;
  return kD * (gi / K::nh) + kHeadDim * (head_base<C, R>(c) + gi % K::nh);
}

// Tensor map and origins of chunk (M-block b, K-chunk k) of GEMM g: K column
// x0, rows ra (A rows 0..63) and rb (A rows 64..127).
template <int C, int R>
__device__ __forceinline__ const CUtensorMap* chunk_box(const SplitMaps& m, int c, int p, int g, int b, int k, int* x0,
                                                        int* ra, int* rb) {
  using K = Cfg<C, R>;
  *x0 = kChunkK * k;
  switch (g) {
    case G_IN:
      *ra = 128 * b;
      *rb = 128 * b + 64;
      return &m.in_proj;
    case G_QKV: {
      const int ga = 2 * b, gb = 2 * b + 1 < 3 * K::nh ? 2 * b + 1 : 2 * b;
      *ra = qkv_group_row<C, R>(c, ga);
      *rb = qkv_group_row<C, R>(c, gb);
      return &m.qkv;
    }
    case G_O: {
      const int base = K::of * c + 128 * b;
      *ra = base;
      *rb = K::of >= 128 ? base + 64 : base;
      return &m.o;
    }
    case G_F1: {
      const int base = K::f1 * c + 128 * b;
      *ra = base;
      *rb = base + 64;
      return &m.ffn1;
    }
    case G_F2:
      *x0 = K::f1 * c + kChunkK * k;
      *ra = 128 * b;
      *rb = 128 * b + 64;
      return &m.ffn2;
    default: {
      const int base = p * kVocab + K::vs * c + 128 * b;  // the last block may overhang (ignored / zero fill)
      *ra = base;
      *rb = base + 64;
      return &m.head;
    }
  }
}

template <int C, int R>
__device__ void producer(SplitSmem<C, R>& sm, const SplitMaps& maps, int c, bool folded) {
  int it = 0;
  for (int p = 0; p < kPositions; ++p) {
    for (int g = has_in_projection(folded, p) ? G_IN : G_QKV; g <= G_HEAD; ++g) {
      const int nb = gemm_blocks<C, R>(g), nk = gemm_kchunks<C, R>(g);
      for (int b = 0; b < nb; ++b) {
        for (int k = 0; k < nk; ++k, ++it) {
          constexpr int kSl = Cfg<C, R>::slots;
          const int slot = it % kSl;
          if (it >= kSl && err_flag(sm) == 0 && !mbar_wait(&sm.empty[slot], ((it / kSl) - 1) & 1)) sm.err = 1;
          if (err_flag(sm)) return;
          int x0, ra, rb;
          const CUtensorMap* map = chunk_box<C, R>(maps, c, p, g, b, k, &x0, &ra, &rb);
          mbar_expect_tx(&sm.full[slot], kChunkBytes);
          bf16* dst = sm.ring[slot];
          tma_load_2d(dst, map, x0, ra, &sm.full[slot]);
          tma_load_2d(dst + kBoxRows * 64, map, x0, rb, &sm.full[slot]);
          tma_load_2d(dst + kPanelElems, map, x0 + 64, ra, &sm.full[slot]);
          tma_load_2d(dst + kPanelElems + kBoxRows * 64, map, x0 + 64, rb, &sm.full[slot]);
          sm.last_issued[slot] = it;
        }
      }
    }
  }
}

template <int C, int R>
__device__ __forceinline__ const bf16* gemm_operand(SplitSmem<C, R>& sm, int g) {
  switch (g) {
    case G_IN: return sm.u.src;
    case G_QKV: return sm.xa;
    case G_O: return sm.ab;
    case G_F1: return sm.xa;
    case G_F2: return sm.u.hid;
    default: return sm.ab;
  }
}

// The MMA warp's single thread: for every GEMM, wait until the consumers have
// written its B operand, then per M-block wait for a free accumulator buffer,
// per chunk wait for the weights, issue 8 MMAs (K = 128) and free the slot.
// With 32-row tiles the in-projection input comes in three 256-column pieces
// per M-block: each piece has its own operand-ready phase, and a commit on
// `srcfree` tells the consumers when its MMAs have read it.
template <int C, int R>
__device__ void mma_issuer(SplitSmem<C, R>& sm, bool folded) {
  using K = Cfg<C, R>;
  int it = 0, mb = 0, gn = 0;
  auto wait_operand = [&]() {
    const bool ok = mbar_wait(&sm.opready, gn & 1);
    ++gn;
    if (!ok) sm.err = 1;
    tmem_fence_after_sync();
    return ok;
  };
  for (int p = 0; p < kPositions && err_flag(sm) == 0; ++p) {
    for (int g = has_in_projection(folded, p) ? G_IN : G_QKV; g <= G_HEAD && err_flag(sm) == 0; ++g) {
      const bool pieces = g == G_IN && K::in_pieces > 1;
      if (!pieces && !wait_operand()) break;
      const bf16* bop = gemm_operand(sm, g);
      const int nb = gemm_blocks<C, R>(g), nk = gemm_kchunks<C, R>(g);
      for (int b = 0; b < nb && err_flag(sm) == 0; ++b, ++mb) {
        const int db = mb % K::nbuf, use = mb / K::nbuf;
        if (use >= 1 && !mbar_wait(&sm.dempty[db], (use - 1) & 1)) {
          sm.err = 1;
          break;
        }
        tmem_fence_after_sync();
        const uint32_t d = sm.tmem + K::dcol(db);
        if (pieces) {
          for (int k = 0; k < nk; ++k, ++it) {
            if ((k & 1) == 0 && !wait_operand()) break;
            const int kc = k & 1;  // K-chunk within the operand piece
            const int slot = it % K::slots;
            if (!mbar_wait(&sm.full[slot], (it / K::slots) & 1)) {
              sm.err = 1;
              break;
            }
            tmem_fence_after_sync();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t a = umma_desc_sw128(sm.ring[slot] + (kk >> 2) * kPanelElems) + 2 * (kk & 3);
              const uint64_t bd = umma_desc_sw128(bop + (2 * kc + (kk >> 2)) * K::op_panel) + 2 * (kk & 3);
              umma_bf16(d, a, bd, K::idesc, (k | kk) != 0);
            }
            umma_commit(&sm.empty[slot]);
            if ((k & 1) == 1) umma_commit(&sm.srcfree);
          }
        } else {
          // two chunks (K = 256) at a time: wait for both, then their 16 MMAs
          // as one straight-line burst (a branch between tcgen05.mma
          // instructions halves their issue rate)
          for (int k = 0; k < nk; k += 2) {
            const bool two = k + 1 < nk;
            const int s0 = it % K::slots, s1 = (it + 1) % K::slots;
            bool ok = mbar_wait(&sm.full[s0], (it / K::slots) & 1);
            if (two) ok = ok && mbar_wait(&sm.full[s1], ((it + 1) / K::slots) & 1);
            if (!ok) {
              sm.err = 1;
              break;
            }
            tmem_fence_after_sync();
            const uint64_t a0 = umma_desc_sw128(sm.ring[s0]), a1 = umma_desc_sw128(sm.ring[s1]);
            const uint64_t b0 = umma_desc_sw128(bop + 2 * k * K::op_panel);
            constexpr uint64_t kPanelStep = kPanelElems * 2 / 16, kOpStep = K::op_panel * 2 / 16;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              umma_bf16(d, a0 + (kk >> 2) * kPanelStep + 2 * (kk & 3), b0 + (kk >> 2) * kOpStep + 2 * (kk & 3),
                        K::idesc, (k | kk) != 0);
            }
            if (two) {
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                umma_bf16(d, a1 + (kk >> 2) * kPanelStep + 2 * (kk & 3),
                          b0 + (2 + (kk >> 2)) * kOpStep + 2 * (kk & 3), K::idesc, true);
              }
            }
            umma_commit(&sm.empty[s0]);
            if (two) umma_commit(&sm.empty[s1]);
            it += two ? 2 : 1;
          }
        }
        umma_commit(&sm.dfull[db]);
      }
    }
  }
  // every MMA this thread issued has completed before the CTA frees TMEM
  umma_commit(&sm.mmafin);
  mbar_wait(&sm.mmafin, 0);
  atomicExch(&sm.mma_done, 1);
}

// Two loads of N TMEM columns (lanes of this warp's quadrant) and one wait.
template <int N>
__device__ __forceinline__ void tmem_ld_pair(uint32_t (&v)[2 * N], uint32_t ta, uint32_t tb) {
  static_assert(N == 4 || N == 8, "width");
  if constexpr (N == 4) {
    tmem_ld4x2(v, ta, tb);
  } else {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(ta)
                 : "memory");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                   "=r"(v[15])
                 : "r"(tb)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                   "+r"(v[15])
                 :
                 : "memory");
  }
}

// Epilogue helpers: warp w reads TMEM lanes [32 (w % 4), +32) (A rows m),
// the columns of session slots [S/2 (w / 4), +S/2): v[i] = row S/2 (w / 4) + i
// (conditional), v[S/2 + i] = row S + S/2 (w / 4) + i (unconditional).
template <int C, int R>
__device__ __forceinline__ void load_block(SplitSmem<C, R>& sm, int mb, float (&v)[R / 2]) {
  using K = Cfg<C, R>;
  constexpr int H = R / 4;  // sessions per warp half
  const int warp = threadIdx.x >> 5;
  const int db = mb % K::nbuf, use = mb / K::nbuf;
  if (err_flag(sm) == 0 && !mbar_wait(&sm.dfull[db], use & 1)) sm.err = 1;
  tmem_fence_after_sync();
  const uint32_t ta = sm.tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + K::dcol(db) + H * (warp >> 2);
  uint32_t r[R / 2];
  tmem_ld_pair<H>(r, ta, ta + R / 2);
  tmem_fence_before_sync();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.dempty[db]);
#pragma unroll
  for (int i = 0; i < R / 2; ++i) v[i] = __uint_as_float(r[i]);
}

template <int R>
__device__ __forceinline__ int epi_row(int i) {
  constexpr int H = R / 4;
  const int sh = (threadIdx.x >> 5) >> 2;
  return i < H ? H * sh + i : R / 2 + H * sh + (i - H);
}

// B operand written: order the generic writes before the MMA warp's reads.
template <int C, int R>
__device__ __forceinline__ void operand_ready(SplitSmem<C, R>& sm) {
  fence_proxy_async();
  cbar();
  if (threadIdx.x == 0) mbar_arrive(&sm.opready);
}

// LayerNorm (no bias, eps 1e-5) of the R rows of x into the B operand xa;
// lane holds weights g of columns [8 lane, +8); warp w: rows R/8 w + [0, R/8).
template <int R>
__device__ __forceinline__ void layer_norm_op(const bf16* x, bf16* xa, const float (&g)[8]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int rr = 0; rr < R / 8; ++rr) {
    const int r = (R / 8) * warp + rr;
    float v[8];
    unpack8(*reinterpret_cast<const uint4*>(x + r * kLdX + lane * 8), v);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += v[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(kD);
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) var += (v[j] - mean) * (v[j] - mean);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    const float rstd = 1.0f / sqrtf(var / static_cast<float>(kD) + 1.0e-5f);
    float out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = ((v[j] - mean) * rstd) * g[j];
    *op_unit<R>(xa, r, lane * 8) = pack8(out);
  }
}

// x (row-major) -> the B operand ab (the head's input).
template <int R>
__device__ __forceinline__ void x_to_operand(const bf16* x, bf16* ab) {
  for (int i = threadIdx.x; i < R * (kD / 8); i += kSC) {
    const int r = i / (kD / 8), k8 = 8 * (i % (kD / 8));
    *op_unit<R>(ab, r, k8) = *reinterpret_cast<const uint4*>(x + r * kLdX + k8);
  }
}

// ---------------------------------------------------------------------------
// exchange rounds
// ---------------------------------------------------------------------------

// Wait for round rd: this CTA announces on its own round barrier the bytes
// its peers push to it in this round (every peer pushes to every other CTA
// in every round), and the round completes when they have all landed.  No
// CTA arrives on another's barrier: a peer's data arriving already shows
// that the peer finished the phase before it, because every push follows
// the pusher's last use of the buffers the round before it filled.
template <int C, int R>
__device__ __forceinline__ void finish_round(SplitSmem<C, R>& sm, uint32_t& rd, uint32_t bytes_in) {
  cbar();
  const int bar = static_cast<int>(rd & 1u);
  if (threadIdx.x == 0) mbar_expect_tx(&sm.xbar[bar], bytes_in);
  if (err_flag(sm) == 0 && !mbar_wait(&sm.xbar[bar], (rd >> 1) & 1u)) sm.err = 1;
  ++rd;
}

// Vocabulary values CTA j of the cluster holds of each session (its slice of
// the head output, clipped to the vocabulary).
template <int C, int R>
__host__ __device__ constexpr int slice_len(int j) {
  return Cfg<C, R>::vs * (j + 1) <= kVocab ? Cfg<C, R>::vs : kVocab - Cfg<C, R>::vs * j;
}

// Bytes CTA c receives in the head-values round: from every peer j, its
// slice of each of c's sessions plus one non-finite flag per session.
template <int C, int R>
__device__ __forceinline__ uint32_t values_bytes_in(int c) {
  uint32_t b = 0;
#pragma unroll
  for (int j = 0; j < C; ++j) {
    if (j != c) b += static_cast<uint32_t>(Cfg<C, R>::own * (slice_len<C, R>(j) * 2 + 4));
  }
  return b;
}

// ---------------------------------------------------------------------------
// attention over the TMEM KV cache for the CTA's heads: warp w reads lane
// quadrant q = w % 4, which holds local head q (16-row tiles) or head q / 2,
// rows 16 (q % 2).. (32-row tiles); part = w / 4 takes the positions of
// parity part; thread t: row t / 2 of the quadrant, head dims
// [32 (t % 2), +32).  Output to the operand ab at the global head's columns,
// and pushed to every peer.
// ---------------------------------------------------------------------------

// Four 32-bit TMEM columns of lane (lane field of taddr) + t stored by thread t.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3])
               : "memory");
}

// 32 columns of the warp's lanes, then the wait (one wait for the whole load).
__device__ __forceinline__ void tmem_ld32w(uint32_t (&v)[32], uint32_t taddr) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
                 "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]),
                 "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                 "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

// Attention with one head per CTA and 16-row tiles (C = 4, 8), spread over
// all four TMEM lane quadrants so that all eight consumer warps attend: lane
// 32 q + l holds row 4 q + l / 8, head dims [8 (l % 8), +8); K of position j
// at columns 4 b(j), V at 64 + 4 b(j) (b(j) = 8 (j mod 2) + j / 2, so each
// parity's positions are 32 contiguous columns); positions 0..15 all cached.
// Warp w reads quadrant w % 4 and takes the positions of parity w / 4; the
// score of a position is summed over the 8 lanes of its row, rounded as the
// reference rounds it (bf16, x 1/8, bf16); the softmax sum runs over the
// positions in order; the odd warp's partial output joins the even warp's.
template <int C, int R>
__device__ __forceinline__ void attention_spread(SplitSmem<C, R>& sm, int p, int c, uint32_t rd) {
  using K = Cfg<C, R>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q4 = warp & 3, part = warp >> 2;
  const int r = 4 * q4 + (lane >> 3), u = lane & 7;
  const uint32_t tl = sm.tmem + (static_cast<uint32_t>(32 * q4) << 16);
  const bf16* qrow = sm.q.qkv + r * K::ldq + 8 * u;  // the CTA's head: q, then k, then v
  {  // append k (part 0) or v (part 1) of position p
    const uint4 t = *reinterpret_cast<const uint4*>(qrow + kHeadDim * (1 + part));
    const uint32_t kv[4] = {t.x, t.y, t.z, t.w};
    tmem_st4(tl + 64u * static_cast<uint32_t>(part) + 4u * static_cast<uint32_t>(tmem_block(p)), kv);
    tmem_wait_st();
  }
  float q[8];
  unpack8(*reinterpret_cast<const uint4*>(qrow), q);
  tmem_fence_before_sync();
  cbar();
  tmem_fence_after_sync();
  float s[8];
  {
    uint32_t kv[32];
    tmem_ld32w(kv, tl + 32u * static_cast<uint32_t>(part));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const float2 t0 = __bfloat1622float2(bf2_of(kv[4 * i + e]));
        const float2 t1 = __bfloat1622float2(bf2_of(kv[4 * i + e + 1]));
        d0 = fmaf(q[2 * e], t0.x, d0);
        d0 = fmaf(q[2 * e + 1], t0.y, d0);
        d1 = fmaf(q[2 * e + 2], t1.x, d1);
        d1 = fmaf(q[2 * e + 3], t1.y, d1);
      }
      float dot = d0 + d1;
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      s[i] = 2 * i + part <= p ? round_bf16(__fmul_rn(round_bf16(dot), 0.125f)) : -CUDART_INF_F;
    }
  }
  float* my_s = sm.u.att.s[part][q4][lane];
#pragma unroll
  for (int m = 0; m < 8; ++m) my_s[m] = s[m];
  cbar();
  float all[kPositions];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    all[2 * m] = sm.u.att.s[0][q4][lane][m];
    all[2 * m + 1] = sm.u.att.s[1][q4][lane][m];
  }
  float mx = all[0];
#pragma unroll
  for (int j = 1; j < kPositions; ++j) mx = fmaxf(mx, all[j]);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPositions; ++j) {
    all[j] = j <= p ? expf(all[j] - mx) : 0.f;
    sum += all[j];
  }
  float o[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) o[d] = 0.f;
  {
    uint32_t vv[32];
    tmem_ld32w(vv, tl + 64u + 32u * static_cast<uint32_t>(part));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (2 * i + part <= p) {
        // select between two compile-time indices (a runtime index would put `all` in local memory)
        const float e = part ? all[2 * i + 1] : all[2 * i];
        const float prob = round_bf16(e / sum);
#pragma unroll
        for (int d = 0; d < 4; ++d) {
          const float2 t = __bfloat1622float2(bf2_of(vv[4 * i + d]));
          o[2 * d] = fmaf(prob, t.x, o[2 * d]);
          o[2 * d + 1] = fmaf(prob, t.y, o[2 * d + 1]);
        }
      }
    }
  }
  if (part == 1) {
    float* dst = sm.u.att.o[q4][lane];
#pragma unroll
    for (int d = 0; d < 8; ++d) dst[d] = o[d];
  }
  cbar();
  if (part == 0) {
    const float* src = sm.u.att.o[q4][lane];
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d] += src[d];
    const int col = kHeadDim * head_base<C, R>(c) + 8 * u;
    const bool send = C <= kHeads || (r >> 3) == (c & 1);
    const uint4 w = pack8(o);
    uint4* dst = op_unit<R>(sm.ab, r, col);
    *dst = w;
    if (send) {
#pragma unroll
      for (int jc = 0; jc < C; ++jc) {
        if (jc != c) st_async_v4(cluster_addr(dst, jc), w, cluster_addr(&sm.xbar[rd & 1u], jc));
      }
    }
  }
}

template <int C, int R>
__device__ __forceinline__ void attention(SplitSmem<C, R>& sm, int p, int c, uint32_t rd) {
  using K = Cfg<C, R>;
  if constexpr (K::nh == 1 && R == 16) {
    attention_spread<C, R>(sm, p, c, rd);
    return;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q4 = warp & 3, part = warp >> 2;
  const int lh = R == 32 ? q4 >> 1 : q4;  // local head of this quadrant
  const bool active = lh < K::nh;
  const int r = (R == 32 ? 16 * (q4 & 1) : 0) + (lane >> 1), half = lane & 1;
  const uint32_t tl = sm.tmem + (static_cast<uint32_t>(32 * q4) << 16);
  const bf16* qrow = sm.q.qkv + r * K::ldq + kHeadDim * lh + 32 * half;
  const bf16* krow = qrow + K::nh * kHeadDim;
  const bf16* vrow = krow + K::nh * kHeadDim;
  float q[32];
  if (active) {
    if (p < kPositions - 1) {  // append k (part 0) or v (part 1) of position p
      const bf16* src = part == 0 ? krow : vrow;
      uint32_t kv[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 t = *reinterpret_cast<const uint4*>(src + 8 * j);
        kv[4 * j] = t.x;
        kv[4 * j + 1] = t.y;
        kv[4 * j + 2] = t.z;
        kv[4 * j + 3] = t.w;
      }
      tmem_st16(tl + K::kv_v * part + 16 * tmem_block(p), kv);
      tmem_wait_st();
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float f8[8];
      unpack8(*reinterpret_cast<const uint4*>(qrow + 8 * j), f8);
#pragma unroll
      for (int e = 0; e < 8; ++e) q[8 * j + e] = f8[e];
    }
  }
  tmem_fence_before_sync();
  cbar();
  tmem_fence_after_sync();

  float s[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) s[m] = -CUDART_INF_F;
  if (active) {
#pragma unroll
    for (int g4 = 0; g4 < 2; ++g4) {
      if (8 * g4 + part <= p) {
        uint32_t k[64];
        tmem_ld64(k, tl + 16 * (8 * part + 4 * g4));
        if (p == kPositions - 1 && part == 1 && g4 == 1) {  // position 15: k from shared memory
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 t = *reinterpret_cast<const uint4*>(krow + 8 * j);
            k[48 + 4 * j] = t.x;
            k[48 + 4 * j + 1] = t.y;
            k[48 + 4 * j + 2] = t.z;
            k[48 + 4 * j + 3] = t.w;
          }
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          float d0 = 0.f, d1 = 0.f;  // two chains
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const float2 t0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&k[16 * jj + e]));
            const float2 t1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&k[16 * jj + e + 1]));
            d0 = fmaf(q[2 * e], t0.x, d0);
            d0 = fmaf(q[2 * e + 1], t0.y, d0);
            d1 = fmaf(q[2 * e + 2], t1.x, d1);
            d1 = fmaf(q[2 * e + 3], t1.y, d1);
          }
          float dot = d0 + d1;
          dot += __shfl_xor_sync(0xffffffffu, dot, 1);
          if (2 * (4 * g4 + jj) + part <= p) s[4 * g4 + jj] = round_bf16(__fmul_rn(round_bf16(dot), 0.125f));
        }
      }
    }
    float* my_s = sm.u.att.s[part][q4][lane];
#pragma unroll
    for (int m = 0; m < 8; ++m) my_s[m] = s[m];
  }
  cbar();
  float o[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) o[d] = 0.f;
  if (active) {
    float all[kPositions];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      all[2 * m] = sm.u.att.s[0][q4][lane][m];
      all[2 * m + 1] = sm.u.att.s[1][q4][lane][m];
    }
    float mx = all[0];
#pragma unroll
    for (int j = 1; j < kPositions; ++j) mx = fmaxf(mx, all[j]);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kPositions; ++j) {
      all[j] = j <= p ? expf(all[j] - mx) : 0.f;
      sum += all[j];
    }
#pragma unroll
    for (int g4 = 0; g4 < 2; ++g4) {
      if (8 * g4 + part <= p) {
        uint32_t v[64];
        tmem_ld64(v, tl + K::kv_v + 16 * (8 * part + 4 * g4));
        if (p == kPositions - 1 && part == 1 && g4 == 1) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 t = *reinterpret_cast<const uint4*>(vrow + 8 * j);
            v[48 + 4 * j] = t.x;
            v[48 + 4 * j + 1] = t.y;
            v[48 + 4 * j + 2] = t.z;
            v[48 + 4 * j + 3] = t.w;
          }
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = 2 * (4 * g4 + jj) + part;
          if (j <= p) {
            // select between two compile-time indices (a runtime index would
            // put `all` in local memory)
            const float e = part ? all[2 * (4 * g4 + jj) + 1] : all[2 * (4 * g4 + jj)];
            const float prob = round_bf16(e / sum);
#pragma unroll
            for (int d = 0; d < 16; ++d) {
              const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v[16 * jj + d]));
              o[2 * d] = fmaf(prob, t.x, o[2 * d]);
              o[2 * d + 1] = fmaf(prob, t.y, o[2 * d + 1]);
            }
          }
        }
      }
    }
    if (part == 1) {
      float* dst = sm.u.att.o[q4][lane];
#pragma unroll
      for (int d = 0; d < 32; ++d) dst[d] = o[d];
    }
  }
  cbar();
  if (active && part == 0) {
    const float* src = sm.u.att.o[q4][lane];
#pragma unroll
    for (int d = 0; d < 32; ++d) o[d] += src[d];
    const int col = kHeadDim * (head_base<C, R>(c) + lh) + 32 * half;
    const bool send = C <= kHeads || (r >> 3) == (c & 1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float f8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f8[e] = o[8 * j + e];
      const uint4 u = pack8(f8);
      uint4* dst = op_unit<R>(sm.ab, r, col + 8 * j);
      *dst = u;
      if constexpr (C > 1) {
        if (send) {
#pragma unroll
          for (int jc = 0; jc < C; ++jc) {
            if (jc != c) st_async_v4(cluster_addr(dst, jc), u, cluster_addr(&sm.xbar[rd & 1u], jc));
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

template <int C, int R>
__device__ __forceinline__ int64_t input_token(const Frame& f, const SplitSmem<C, R>& sm, int slot, int p) {
  if (f.forced) {
    const int64_t t = f.forced[static_cast<int64_t>(sm.sess[slot]) * kPositions + p];
    return t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
  }
  return sm.tok[slot][p];
}

template <int C, int R>
__global__ void __launch_bounds__(kSThreads, 1) split_frame_kernel(Frame f, const __grid_constant__ SplitMaps maps) {
  using K = Cfg<C, R>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
  SplitSmem<C, R>& sm = *reinterpret_cast<SplitSmem<C, R>*>(smem_raw + pad);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rp = f.rp;
  const bool folded = f.emb_proj != nullptr;
  int c = 0;
  if constexpr (C > 1) c = static_cast<int>(cg::this_cluster().block_rank());
  const int tile = static_cast<int>(blockIdx.x) / C;

  // ---- sessions [S tile, +S) of the active list (every CTA of the cluster)
  if (warp == 0) {
    int seen = 0;
    const int first = K::S * tile;
    for (int base = 0; base < f.n; base += 32) {
      const int s = base + lane;
      const bool act = s < f.n && (f.active == nullptr || f.active[s]);
      const unsigned m = __ballot_sync(0xffffffffu, act);
      const int rank = seen + __popc(m & ((1u << lane) - 1u));
      if (act && rank >= first && rank < first + K::S) sm.sess[rank - first] = s;
      seen += __popc(m);
    }
    if (lane == 0) {
      const int left = seen - first;
      sm.n_sess = left <= 0 ? 0 : (left < K::S ? left : K::S);
      sm.err = 0;
      sm.producer_done = 0;
      sm.mma_done = 0;
    }
  }
  __syncthreads();
  const int n_sess = sm.n_sess;
  if (n_sess == 0) return;  // the same in every CTA of the cluster: none touches another
  // row r belongs to session slot r % S (sub-row r / S)
  auto live = [&](int r) { return (r % K::S) < n_sess && (r / K::S) < rp; };
  const int own0 = K::own * c;
  const int n_own = n_sess - own0 <= 0 ? 0 : (n_sess - own0 < K::own ? n_sess - own0 : K::own);

  if (threadIdx.x == 0) {
    for (int s = 0; s < K::slots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
      sm.last_issued[s] = -1;
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.dfull[b], 1);
      mbar_init(&sm.dempty[b], kSW);
      mbar_init(&sm.xbar[b], 1);
    }
    mbar_init(&sm.opready, 1);
    mbar_init(&sm.srcfree, 1);
    mbar_init(&sm.mmafin, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(&sm.tmem, 512);
    tmem_relinquish();
  }
  if (threadIdx.x < n_sess) {
    const int sid = sm.sess[threadIdx.x];
    sm.flags[threadIdx.x] = (f.unfinished[sid] ? 1u : 0u) | (f.finished[sid] ? 2u : 0u) | (f.forbid[sid] ? 4u : 0u);
  }
  if (threadIdx.x < n_own) {  // per-session state and EOS registration of the owned sessions
    const int ls = threadIdx.x;
    const int sid = sm.sess[own0 + ls];
    sm.ctr[ls] = f.counter_io[sid];
    sm.seed[ls] = f.seed[sid];
    int32_t inv = 0;
    bool en = !f.unfinished[sid] && !f.finished[sid] && !f.forbid[sid];
    if (en && f.final_w == nullptr) {
      inv = 2;
      en = false;
    }
    sm.inv[ls] = inv;
    if (en) {
      const int slot = atomicAdd(f.eos_count, 1);
      f.eos_list[slot] = sid;
      f.eos_slot[sid] = slot;
    } else {
      f.eos_slot[sid] = -1;
    }
  }
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  if constexpr (C > 1) cg::this_cluster().sync();  // every CTA's barriers exist before any push

  if (warp >= kSW) {  // control warpgroup
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kSProducerRegs));
    if (warp == kSW && lane == 0) {
      producer<C, R>(sm, maps, c, folded);
      // no copy may still be writing when the CTA leaves
      for (int s = 0; s < K::slots; ++s) {
        const int last = sm.last_issued[s];
        if (last >= 0) mbar_wait(&sm.full[s], (last / K::slots) & 1);
      }
      atomicExch(&sm.producer_done, 1);
    } else if (warp == kSW + 1 && lane == 0) {
      mma_issuer<C, R>(sm, folded);
    }
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSConsumerRegs));
  {
    float g1[8], g2[8];
    unpack8(*reinterpret_cast<const uint4*>(f.ln1 + lane * 8), g1);
    unpack8(*reinterpret_cast<const uint4*>(f.ln2 + lane * 8), g2);
    const int q4 = warp & 3, sh = warp >> 2;
    const int m_lane = 32 * q4 + lane;  // A row of an M-block held by this thread
    const bool cfg = rp == 2;
    const float cfg_scale = f.prm.cfg_scale, uncond_scale = __fsub_rn(1.0f, f.prm.cfg_scale);
    int mb = 0;          // M-blocks consumed
    uint32_t rd = 0;     // exchange rounds
    int src_pieces = 0;  // in-projection input pieces staged (32-row tiles)
    const bool tracer = f.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
    if (tracer) f.trace[256] = static_cast<uint64_t>(clock64()), f.trace[257] = global_ns();
    for (int p = 0; p < kPositions; ++p) {
      // ---------------- input rows
      s_stamp(f, tracer, p, 0);
      if (has_in_projection(folded, p)) {
        // the rows' 768 inputs (p = 0: decoder hidden; else the sampled token's
        // embedding), whole or in pieces of 256 columns per M-block
        auto stage_src = [&](int piece) {
          constexpr int kw = kEmbed / K::in_pieces;
          for (int i = threadIdx.x; i < R * (kw / 8); i += kSC) {
            const int r = i / (kw / 8), k8 = 8 * (i % (kw / 8));
            uint4 v = make_uint4(0, 0, 0, 0);
            if (live(r)) {
              const int slot = r % K::S, sub = r / K::S;
              const bf16* src;
              if (p == 0) {
                src = f.hidden + (static_cast<int64_t>(sm.sess[slot]) * rp + sub) * kEmbed;
              } else {
                src = f.emb + (static_cast<int64_t>(p - 1) * kVocab + input_token(f, sm, slot, p - 1)) * kEmbed;
              }
              v = *reinterpret_cast<const uint4*>(src + kw * piece + k8);
            }
            *op_unit<R>(sm.u.src, r, k8) = v;
          }
        };
        if constexpr (K::in_pieces == 1) {
          stage_src(0);
          operand_ready(sm);
        }
        const bf16* pos = f.pos + static_cast<int64_t>(p) * kD;
        for (int b = 0; b < 2; ++b, ++mb) {
          if constexpr (K::in_pieces > 1) {
            for (int piece = 0; piece < K::in_pieces; ++piece, ++src_pieces) {
              // the MMAs of the previous piece have read the buffer
              if (src_pieces > 0 && err_flag(sm) == 0 && !mbar_wait(&sm.srcfree, (src_pieces - 1) & 1)) sm.err = 1;
              stage_src(piece);
              operand_ready(sm);
            }
          }
          float v[R / 2];
          load_block(sm, mb, v);
          const int n = 128 * b + m_lane;
          const float bias = bf2f(f.in_b[n]), pe = bf2f(pos[n]);
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            const float y = round_bf16(__fadd_rn(v[i], bias));
            sm.x[epi_row<R>(i) * kLdX + n] = f2bf(__fadd_rn(y, pe));
          }
        }
      }
      // head p bias slice; per-position flags
      {
        const bf16* hbp = f.head_b + static_cast<int64_t>(p) * kVocab;
        for (int i = threadIdx.x; i < K::vs / 8; i += kSC) {
          const int v0 = K::vs * c + 8 * i;
          uint4 u = make_uint4(0, 0, 0, 0);
          if (v0 < kVocab) u = *reinterpret_cast<const uint4*>(hbp + v0);  // kVocab % 8 == 0
          *reinterpret_cast<uint4*>(sm.hb + 8 * i) = u;
        }
        if (threadIdx.x < K::S) {
          sm.nf[threadIdx.x] = 0;
          sm.vmax[threadIdx.x] = 0;
        }
      }
      cbar();

      // ---------------- LN1 (with the folded tables done by the previous
      // position's row gather), qkv of the CTA's heads
      if (has_in_projection(folded, p)) layer_norm_op<R>(sm.x, sm.xa, g1);
      operand_ready(sm);
      s_stamp(f, tracer, p, 1);
      for (int b = 0; b < K::nq; ++b, ++mb) {
        float v[R / 2];
        load_block(sm, mb, v);
        const int gi = 2 * b + (m_lane >> 6);
        if (gi < 3 * K::nh) {
          const int col = kHeadDim * gi + (m_lane & 63);  // (type, local head) major, as the staging layout
#pragma unroll
          for (int i = 0; i < R / 2; ++i) sm.q.qkv[epi_row<R>(i) * K::ldq + col] = f2bf(v[i]);
        }
      }
      cbar();

      s_stamp(f, tracer, p, 2);
      // ---------------- attention (R1: the heads' outputs to every CTA)
      attention<C, R>(sm, p, c, rd);
      s_stamp(f, tracer, p, 3);
      if constexpr (C > 1) {
        finish_round(sm, rd, static_cast<uint32_t>((C - 1) * K::att_rows * kHeadDim * K::nh * 2));
        fence_proxy_async();
      }
      operand_ready(sm);

      s_stamp(f, tracer, p, 4);
      // ---------------- o-projection + residual (R2: the CTA's features to every CTA)
      for (int b = 0; b < K::no; ++b, ++mb) {
        float v[R / 2];
        load_block(sm, mb, v);
        const int nl = 128 * b + m_lane;
        if (nl < K::of) {
          const int n = K::of * c + nl;
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            bf16* xr = sm.x + epi_row<R>(i) * kLdX + n;
            *xr = f2bf(__fadd_rn(bf2f(*xr), round_bf16(v[i])));
          }
        }
      }
      cbar();
      // rows of the CTA's feature slice of x to every peer, 16-byte units
      auto push_x_slice = [&]() {
        constexpr int upr = K::of / 8;
        for (int i = threadIdx.x; i < R * upr; i += kSC) {
          const int r = i / upr, k8 = K::of * c + 8 * (i % upr);
          const uint4* src = reinterpret_cast<const uint4*>(sm.x + r * kLdX + k8);
          const uint4 u = *src;
#pragma unroll
          for (int j = 0; j < C; ++j) {
            if (j != c) st_async_v4(cluster_addr(src, j), u, cluster_addr(&sm.xbar[rd & 1u], j));
          }
        }
      };
      if constexpr (C > 1) {
        push_x_slice();
        finish_round(sm, rd, static_cast<uint32_t>((C - 1) * R * K::of * 2));
      }

      s_stamp(f, tracer, p, 5);
      // ---------------- LN2, FFN1 + GELU
      layer_norm_op<R>(sm.x, sm.xa, g2);
      operand_ready(sm);
      s_stamp(f, tracer, p, 6);
      for (int b = 0; b < K::nf1; ++b, ++mb) {
        float v[R / 2];
        load_block(sm, mb, v);
        const int fl = 128 * b + m_lane;
#pragma unroll
        for (int i = 0; i < R / 2; ++i) op_store<R>(sm.u.hid, epi_row<R>(i), fl, f2bf(gelu_tanh(round_bf16(v[i]))));
      }
      operand_ready(sm);

      s_stamp(f, tracer, p, 7);
      // ---------------- FFN2 (+ R3 reduce-scatter, R4 all-gather) + residual
      float own_part[R / 2];  // 32-row tiles: this CTA's partials of its own features
#pragma unroll
      for (int i = 0; i < R / 2; ++i) own_part[i] = 0.f;
      for (int b = 0; b < 2; ++b, ++mb) {
        float v[R / 2];
        load_block(sm, mb, v);
        const int n = 128 * b + m_lane;
        if constexpr (C == 1) {
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            bf16* xr = sm.x + epi_row<R>(i) * kLdX + n;
            *xr = f2bf(__fadd_rn(bf2f(*xr), round_bf16(v[i])));
          }
        } else {
          const int owner = n / K::of, nl = n % K::of;
          // receive slot of this CTA at the owner: every CTA (16-row tiles), or
          // the peers only (32-row tiles: the owner keeps its own in registers)
          const int slot_at = K::red_slots == C ? c : (c < owner ? c : c - 1);
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            if (owner == c) {
              if constexpr (K::red_slots == C) {
                sm.red[c][epi_row<R>(i)][nl] = v[i];
              } else {
                own_part[i] = v[i];
              }
            } else {
              st_async_b32(cluster_addr(&sm.red[slot_at][epi_row<R>(i)][nl], owner), __float_as_uint(v[i]),
                           cluster_addr(&sm.xbar[rd & 1u], owner));
            }
          }
        }
      }
      if constexpr (C > 1) {
        s_stamp(f, tracer, p, 8);
        finish_round(sm, rd, static_cast<uint32_t>((C - 1) * R * K::of * 4));
        s_stamp(f, tracer, p, 9);
        if constexpr (K::red_slots == C) {
          constexpr int upr = K::of / 8;
          for (int i = threadIdx.x; i < R * upr; i += kSC) {
            const int r = i / upr, k8 = 8 * (i % upr);
            float s8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) s8[e] = 0.f;
#pragma unroll
            for (int j = 0; j < C; ++j) {
#pragma unroll
              for (int e = 0; e < 8; ++e) s8[e] += sm.red[j][r][k8 + e];
            }
            uint4* xr = reinterpret_cast<uint4*>(sm.x + r * kLdX + K::of * c + k8);
            float xv[8];
            unpack8(*xr, xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) xv[e] = __fadd_rn(xv[e], round_bf16(s8[e]));
            *xr = pack8(xv);
          }
        } else {
          // two CTAs: own + the peer's partial (f32 addition of two terms is
          // the same in either order), + residual
          static_assert(C == 2, "32-row tiles run on 2-CTA clusters");
          const int n = K::of * c + m_lane;
#pragma unroll
          for (int i = 0; i < R / 2; ++i) {
            bf16* xr = sm.x + epi_row<R>(i) * kLdX + n;
            const float sum = __fadd_rn(own_part[i], sm.red[0][epi_row<R>(i)][m_lane]);
            *xr = f2bf(__fadd_rn(bf2f(*xr), round_bf16(sum)));
          }
        }
        cbar();
        push_x_slice();
        finish_round(sm, rd, static_cast<uint32_t>((C - 1) * R * K::of * 2));
      } else {
        cbar();
      }
      x_to_operand<R>(sm.x, sm.ab);
      operand_ready(sm);

      s_stamp(f, tracer, p, 10);
      // ---------------- head p: bias, CFG combine, constraints (R5: values to the owners)
      {
        bf16* lo_base = f.logits_out;
        // with 32-row tiles the other CTA's sessions' values wait in xa (free
        // between FFN1 and the next position's LN1), [non-owned slot][vs]
        uint16_t* out32 = reinterpret_cast<uint16_t*>(sm.xa);
        constexpr int H = R / 4;  // sessions per warp half
        uint32_t fl[H];           // flags of the thread's sessions H sh + i (0 for dead slots)
#pragma unroll
        for (int i = 0; i < H; ++i) fl[i] = H * sh + i < n_sess ? sm.flags[H * sh + i] : 0u;
        for (int b = 0; b < K::nhb; ++b, ++mb) {
          float v[R / 2];
          load_block(sm, mb, v);
          const int vl = 128 * b + m_lane;
          const int t = K::vs * c + vl;
          const bool in_vocab = t < kVocab;
          const float bias = bf2f(sm.hb[vl]);
          uint32_t nfm = 0;   // non-finite guided logit, bit i: session H sh + i
          uint32_t keys[H];
#pragma unroll
          for (int i = 0; i < H; i += 2) {  // sessions H sh + i and + 1 as the halves of bf16x2 values
            const uint32_t c2 = pack2_rn(__fadd_rn(v[i], bias), __fadd_rn(v[i + 1], bias));
            const uint32_t u2 = pack2_rn(__fadd_rn(v[H + i], bias), __fadd_rn(v[H + i + 1], bias));
            if (lo_base && in_vocab) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int slot = H * sh + i + h;
                if (slot < n_sess) {
                  uint16_t* lr = reinterpret_cast<uint16_t*>(lo_base) +
                                 (static_cast<int64_t>(sm.sess[slot]) * kPositions + p) * rp * kVocab;
                  lr[t] = static_cast<uint16_t>(h ? c2 >> 16 : c2 & 0xffffu);
                  if (cfg) lr[kVocab + t] = static_cast<uint16_t>(h ? u2 >> 16 : u2 & 0xffffu);
                }
              }
            }
            const uint32_t g2 = cfg ? guided_value2(c2, u2, cfg_scale, uncond_scale) : c2;
            uint32_t g0 = g2 & 0xffffu, g1 = g2 >> 16;
            // constraints only where they can change a value: specials, non-finite values, finished rows
            if (t >= kCodebook || (g0 & 0x7f80u) == 0x7f80u || (g1 & 0x7f80u) == 0x7f80u || ((fl[i] | fl[i + 1]) & 2u)) {
              bool n0 = false, n1 = false;
              g0 = constrain(g0, t, fl[i] & 1u, (fl[i] & 2u) != 0, (fl[i] & 4u) != 0, n0);
              g1 = constrain(g1, t, fl[i + 1] & 1u, (fl[i + 1] & 2u) != 0, (fl[i + 1] & 4u) != 0, n1);
              nfm |= (n0 ? 1u : 0u) << i | (n1 ? 1u : 0u) << (i + 1);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int slot = H * sh + i + h;
              const uint32_t val = h ? g1 : g0;
              const bool live = in_vocab && slot < n_sess;
              keys[i + h] = live ? sample_key(val) : 0u;
              if (!live) continue;
              const int owner = slot / K::own;
              if (owner == c) {
                sm.u.v.own[slot - own0][t] = static_cast<uint16_t>(val);
              } else if constexpr (R == 16) {
                sm.u.v.out[slot][vl] = static_cast<uint16_t>(val);
              } else {
                out32[(slot < own0 ? slot : slot - K::own) * K::vs + vl] = static_cast<uint16_t>(val);
              }
            }
          }
          if (!in_vocab) nfm = 0;
          nfm &= (1u << (n_sess - H * sh < 0 ? 0 : (n_sess - H * sh < H ? n_sess - H * sh : H))) - 1u;
          const uint32_t any = __reduce_or_sync(0xffffffffu, nfm);
          if (lane == 0 && any != 0) {
#pragma unroll
            for (int i = 0; i < H; ++i) {
              if (any & (1u << i)) atomicOr(&sm.nf[H * sh + i], 1u);
            }
          }
          if constexpr (K::sw > 1) {  // the group sampler takes the row maximum from here
#pragma unroll
            for (int i = 0; i < H; ++i) {
              const uint32_t km = __reduce_max_sync(0xffffffffu, keys[i]);
              if (lane == 0 && km != 0) atomicMax(&sm.vmax[H * sh + i], km);
            }
          }
        }
        cbar();
        s_stamp(f, tracer, p, 11);
        if constexpr (C > 1) {
          // the other CTAs' sessions: this CTA's vocabulary slice of each, and its non-finite flags
          constexpr int full_units = K::vs / 8;
          const int len = slice_len<C, R>(c);  // a multiple of 8
          const int units = len / 8;
          const int n_other = K::S - K::own;
          for (int i = threadIdx.x; i < n_other * full_units; i += kSC) {
            const int oi = i / full_units, u = i % full_units;
            if (u < units) {
              const int slot = oi < own0 ? oi : oi + K::own;  // skip the owned slots
              const int owner = slot / K::own;
              uint4 val;
              if constexpr (R == 16) {
                val = *reinterpret_cast<const uint4*>(&sm.u.v.out[slot][8 * u]);
              } else {
                val = *reinterpret_cast<const uint4*>(&out32[oi * K::vs + 8 * u]);
              }
              st_async_v4(cluster_addr(&sm.u.v.own[slot - K::own * owner][K::vs * c + 8 * u], owner), val,
                          cluster_addr(&sm.xbar[rd & 1u], owner));
            }
          }
          if (threadIdx.x < K::S) {
            const int slot = threadIdx.x;
            const int owner = slot / K::own;
            if (owner != c) {
              st_async_b32(cluster_addr(&sm.peer_nf[c][slot - K::own * owner], owner),
                           (sm.nf[slot] << 16) | sm.vmax[slot], cluster_addr(&sm.xbar[rd & 1u], owner));
            }
          }
          finish_round(sm, rd, values_bytes_in<C, R>(c));
        }
      }
      s_stamp(f, tracer, p, 12);

      // ---------------- sampling (R6: the token to every CTA): one warp per owned
      // session, or a group of 8 / own >= 4 warps per session
      {
        constexpr int W = K::sw;
        const int ls = warp / W;
        if (ls < n_own) {
          const int slot = own0 + ls;
          uint32_t nfs = sm.nf[slot], M = sm.vmax[slot];
          if constexpr (C > 1) {
#pragma unroll
            for (int j = 0; j < C; ++j) {
              if (j != c) {
                const uint32_t pk = sm.peer_nf[j][ls];
                nfs |= pk >> 16;
                M = (pk & 0xffffu) > M ? (pk & 0xffffu) : M;
              }
            }
          }
          RowSample rs;
          rs.vals = sm.u.v.own[ls];
          rs.flags = sm.flags[slot];
          rs.nonfinite = nfs != 0;
          rs.seed = sm.seed[ls];
          rs.counter = sm.ctr[ls];
          int invalid = 0;
          int token;
          if constexpr (W == 1) {
            uint16_t* list = reinterpret_cast<uint16_t*>(sm.q.lists[ls]);
            token = sample_row(rs, f.prm, list, list + kListCap + 16, &invalid);
          } else {
            uint32_t* list32 = reinterpret_cast<uint32_t*>(sm.xa) + ls * kListCap;
            token = sample_group<W>(rs, M < kKeyNegInf ? kKeyNegInf : M, f.prm, list32, sm.q.grp[ls], 2 + ls,
                                    &invalid);
          }
          __syncwarp();
          if (warp % W == 0 && lane == 0) {
            const int64_t counter = sm.ctr[ls];
            sm.tok[slot][p] = token;
            sm.inv[ls] |= invalid;
            const bool counter_valid = counter >= 0 && counter <= kMaxCounter;
            if (!f.prm.argmax && counter_valid) sm.ctr[ls] = counter + 1;
            if constexpr (C > 1) {
              if (p + 1 < kPositions) {
#pragma unroll
                for (int j = 0; j < C; ++j) {
                  if (j != c) {
                    st_async_b32(cluster_addr(&sm.tok[slot][p], j), static_cast<uint32_t>(token),
                                 cluster_addr(&sm.xbar[rd & 1u], j));
                  }
                }
              }
            }
          }
        }
      }
      s_stamp(f, tracer, p, 13);
      if constexpr (C > 1) {
        if (p + 1 < kPositions) {
          // dead owned slots still announce their 4 bytes: push a zero token for them
          if (threadIdx.x >= n_own && threadIdx.x < K::own) {
            const int slot = own0 + threadIdx.x;
            sm.tok[slot][p] = 0;
#pragma unroll
            for (int j = 0; j < C; ++j) {
              if (j != c) st_async_b32(cluster_addr(&sm.tok[slot][p], j), 0u, cluster_addr(&sm.xbar[rd & 1u], j));
            }
          }
          finish_round(sm, rd, static_cast<uint32_t>((C - 1) * K::own * 4));
        } else {
          cbar();
        }
      } else {
        cbar();
      }

      s_stamp(f, tracer, p, 14);
      // ---------------- next input rows (folded tables), every CTA, all sessions
      if (folded && p + 1 < kPositions) {
        for (int slot = warp; slot < n_sess; slot += kSW) {
          const int64_t tin = input_token(f, sm, slot, p);
          float e8[8], p8[8];
          unpack8(
              *reinterpret_cast<const uint4*>(f.emb_proj + (static_cast<int64_t>(p) * kVocab + tin) * kD + lane * 8),
              e8);
          unpack8(*reinterpret_cast<const uint4*>(f.pos + static_cast<int64_t>(p + 1) * kD + lane * 8), p8);
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = __fadd_rn(e8[e], p8[e]);
          const uint4 row = pack8(y);
          *reinterpret_cast<uint4*>(sm.x + slot * kLdX + lane * 8) = row;
          if (rp == 2) *reinterpret_cast<uint4*>(sm.x + (slot + K::S) * kLdX + lane * 8) = row;
          // the next position's LN1 of the row, from registers (the same arithmetic as
          // layer_norm_op; the conditional and unconditional rows are the same row)
          float v[8];
          unpack8(row, v);
          float sum = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) sum += v[j];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          const float mean = sum / static_cast<float>(kD);
          float var = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) var += (v[j] - mean) * (v[j] - mean);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
          const float rstd = 1.0f / sqrtf(var / static_cast<float>(kD) + 1.0e-5f);
          float out[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) out[j] = ((v[j] - mean) * rstd) * g1[j];
          const uint4 ln = pack8(out);
          *op_unit<R>(sm.xa, slot, lane * 8) = ln;
          if (rp == 2) *op_unit<R>(sm.xa, slot + K::S, lane * 8) = ln;
        }
      }
      cbar();
      s_stamp(f, tracer, p, 15);
    }

    if (tracer) f.trace[258] = static_cast<uint64_t>(clock64()), f.trace[259] = global_ns();
    // ---- commit (owned sessions): tokens, counters, flags, next-frame embedding
    for (int i = threadIdx.x; i < n_own * kPositions; i += kSC) {
      const int ls = i / kPositions, pp = i % kPositions;
      const int slot = own0 + ls;
      const int sid = sm.sess[slot];
      const int32_t t = sm.tok[slot][pp];
      f.codec_tokens[codec_index(f, sid, pp)] = t;
      f.tokens[static_cast<int64_t>(sid) * kPositions + pp] = t;
    }
    if (threadIdx.x < n_own) {
      const int ls = threadIdx.x;
      const int sid = sm.sess[own0 + ls];
      f.counter_io[sid] = sm.ctr[ls];
      f.invalid_rows[sid] = sm.inv[ls] | (err_flag(sm) ? 4 : 0);
      if (f.eos_slot[sid] < 0) commit_end(f, sid, f.finished[sid] ? 0 : -1);
    }
    for (int i = threadIdx.x; i < n_own * (kEmbed / 8); i += kSC) {
      const int ls = i / (kEmbed / 8), k8 = 8 * (i % (kEmbed / 8));
      const int slot = own0 + ls;
      float acc[8];
#pragma unroll
      for (int pp = 0; pp < kPositions; ++pp) {
        float v[8];
        unpack8(*reinterpret_cast<const uint4*>(f.emb + (static_cast<int64_t>(pp) * kVocab + sm.tok[slot][pp]) * kEmbed +
                                                k8),
                v);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = pp == 0 ? v[e] : round_bf16(__fadd_rn(acc[e], v[e]));
      }
      float out[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = __fdiv_rn(acc[e], 16.0f);
      *reinterpret_cast<uint4*>(f.next_emb + static_cast<int64_t>(sm.sess[slot]) * kEmbed + k8) = pack8(out);
    }

    // ---- teardown: the control warps' copies and MMAs have finished (bounded)
    if (threadIdx.x == 0) {
      const unsigned long long t0 = global_ns();
      while ((*reinterpret_cast<volatile int*>(&sm.producer_done) == 0 ||
              *reinterpret_cast<volatile int*>(&sm.mma_done) == 0) &&
             global_ns() - t0 < 20000000ull) {
        __nanosleep(1000);
      }
    }
    tmem_fence_before_sync();
    cbar();
    if (warp == 0) {
      tmem_fence_after_sync();
      tmem_dealloc(sm.tmem, 512);
    }
  }
  if constexpr (C > 1) cg::this_cluster().sync();  // no CTA leaves while a peer may still push into it
}

template <int C, int R>
int split_clusters() {
  static PerDeviceInt cache;  // the opt-in below is per device context
  return cache.get([] {
    int clusters = 0;
    if (cudaFuncSetAttribute(split_frame_kernel<C, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(split_smem_bytes<C, R>())) == cudaSuccess) {
      if constexpr (C == 1) {
        int blocks = 0;
        int dev = 0, sms = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, split_frame_kernel<C, R>, kSThreads,
                                                          split_smem_bytes<C, R>()) == cudaSuccess &&
            cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && blocks >= 1) {
          clusters = blocks * sms;
        }
      } else {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = C;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(C);
        cfg.blockDim = dim3(kSThreads);
        cfg.dynamicSmemBytes = split_smem_bytes<C, R>();
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, split_frame_kernel<C, R>, &cfg) != cudaSuccess) clusters = 0;
      }
    }
    cudaGetLastError();
    return clusters;
  });
}

template <int C, int R>
cudaError_t launch_split(const Frame& f, const SplitMaps& maps, cudaStream_t stream) {
  const int tiles = (f.n + Cfg<C, R>::S - 1) / Cfg<C, R>::S;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(tiles * C);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = split_smem_bytes<C, R>();
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, split_frame_kernel<C, R>, f, maps);
}

}  // namespace

int split_frame_clusters(int split, int rows) {
  if (rows == 32) return split == 2 ? split_clusters<2, 32>() : 0;
  switch (split) {
    case 1: return split_clusters<1, 16>();
    case 2: return split_clusters<2, 16>();
    case 4: return split_clusters<4, 16>();
    case 8: return split_clusters<8, 16>();
    default: return 0;
  }
}

bool split_frame_supported(const Frame& f, int split, int rows) {
  if (f.d != kD || f.H != kHeads || f.F != kF || f.L != 1 || !f.in_proj || (f.rp != 1 && f.rp != 2)) return false;
  return split_frame_clusters(split, rows) > 0;
}

cudaError_t launch_split_frame(const Frame& f, int split, int rows, cudaStream_t stream) {
  SplitMaps maps;
  if (!make_weight_map(&maps.in_proj, f.in_w, kEmbed, kD, kBoxRows) ||
      !make_weight_map(&maps.qkv, f.qkv, kD, 3 * kD, kBoxRows) || !make_weight_map(&maps.o, f.o, kD, kD, kBoxRows) ||
      !make_weight_map(&maps.ffn1, f.w1, kD, kF, kBoxRows) || !make_weight_map(&maps.ffn2, f.w2, kF, kD, kBoxRows) ||
      !make_weight_map(&maps.head, f.head_w, kD, static_cast<uint64_t>(kPositions) * kVocab, kBoxRows)) {
    return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaMemsetAsync(f.eos_count, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  if (rows == 32) {
    if (split != 2) return cudaErrorInvalidValue;
    e = launch_split<2, 32>(f, maps, stream);
  } else {
    switch (split) {
      case 1: e = launch_split<1, 16>(f, maps, stream); break;
      case 2: e = launch_split<2, 16>(f, maps, stream); break;
      case 4: e = launch_split<4, 16>(f, maps, stream); break;
      case 8: e = launch_split<8, 16>(f, maps, stream); break;
      default: return cudaErrorInvalidValue;
    }
  }
  if (e != cudaSuccess) return e;
  return launch_frame_eos(f, stream);
}

}  // namespace mtt
