// Quad frame kernel: a 4-CTA thread-block cluster runs all 16 positions of a
// Local AR frame for a tile of 16 sessions (32 rows with CFG), CTA c owning
// attention head c.  It is the throughput path for the benchmark shape:
// 32-row tiles give each tcgen05.mma (M = 128 weight rows, N = 32 tile rows,
// K = 16) twice the work of a 16-row tile for the same ~46-cycle cost, and
// with one head per CTA the tile's key/value cache fits in tensor memory
// next to eight accumulator buffers, so the MMA warp never waits for an
// epilogue to free one.
//
// Reference ops per position (local_ar_wrapper.py:609-751,
// transformer_2501.py:405-442,761-851,1153-1232; sampling
// local_ar_plugins.cu:1211-1370; embedding sum main_decoder_wrapper.py:796-810),
// in CTA c of the cluster:
//
//   input rows: p = 0 (every p without the folded tables) the in-projection
//     of all rows, x = bf16(bf16(W_in h + b) + pos[p]); p >= 1 the folded
//     rows x = bf16(emb_proj[p-1][token] + pos[p]), gathered by every CTA
//   LN1 of all rows; q|k|v of head c; k, v appended to the TMEM cache;
//     attention of head c for the 32 rows;                       round R1
//       (head c's output columns to every CTA)
//   o-projection of all 256 features (every CTA: no round) + residual; LN2
//   FFN1 features [256 c, +256) + GELU-tanh; FFN2 partial sums of all 256
//     outputs over those features, each CTA's 64-feature slice to its owner
//                                                                round R3
//   own features: the four partials in CTA order, + residual     round R4
//       (x'' columns to every CTA: the head's input)
//   head p vocabulary [512 c, +512): bias, CFG combine, constraints; the
//     other CTAs' sessions' values to their owners (sessions [4 c, +4) are
//     sampled by CTA c)                                          round R5
//   one warp per owned session samples it (sample_row) and sends the token
//     to every CTA                                               round R6
//
// GEMMs (swap-AB): D[128 weight rows][32 tile rows] = W[128][K] x X[32][K]^T,
// tcgen05.mma kind::f16 M=128 N=32 K=16, A a weight chunk and B the
// activation panels, both in shared memory (K-major, 128-byte swizzle).  A
// weight chunk is 128 rows x 64 K columns (16 KB) as two 64-row TMA boxes
// (no multicast) that may come from different rows of a matrix (head c's q
// and k rows); the weights stream through a ring filled by a producer warp
// that runs ahead across GEMMs and positions.  One thread issues the MMAs;
// tcgen05.commit frees the ring slots and signals an accumulator full.
//
// Tensor memory (512 columns x 128 lanes): lane 32 q + l holds row
// 8 q + l / 4, head dims [16 (l % 4), +16); K of position j at columns
// [8 j, +8), V at [128 + 8 j, +8) (bf16 pairs); eight 32-column accumulator
// buffers at column 256 + 32 b, taken by M-block in turn.
//
// Rows: row 2 s + u of the tile is session slot s's conditional (u = 0) or
// unconditional (u = 1) row, so an epilogue lane holds both rows of a
// session.
//
// Exchanges push data with st.async into the receivers' shared memory and
// complete on the receiver's round mbarrier, which the receiver arms with the
// bytes it expects; every CTA pushes to every other in every round, so a
// completed round also shows every peer finished the phase before it.  Two
// round barriers alternate.  Every push lands in a buffer the receiver does
// not use between the round before and the round it belongs to.  Every wait
// is bounded; a timeout sets invalid bit 4 for the CTA's sessions.
#include <cooperative_groups.h>
#include <cuda.h>

#include "frame_common.cuh"
#include "ptx.cuh"
#include "tile_common.cuh"

namespace cg = cooperative_groups;

namespace mtt {
namespace {

constexpr int kQR = 32;                // tile rows
constexpr int kQS = 16;                // session slots per tile
constexpr int kQW = 8;                 // consumer warps
constexpr int kQT = kQW * 32;          // consumer threads
constexpr int kQThreads = kQT + 128;   // + the control warpgroup (producer warp, MMA warp)
constexpr int kQProducerRegs = 40;
constexpr int kQConsumerRegs = 232;
static_assert(128 * kQProducerRegs + kQT * kQConsumerRegs <= kQThreads * 168, "register split");
constexpr int kQD = 256;
constexpr int kQF = 1024;
constexpr int kQSlots = 8;             // weight ring slots
constexpr int kQGroups = kQSlots / 4;  // ring groups of 4 chunks (one M-block's K = 256), one barrier pair each
constexpr int kQNbuf = 8;              // accumulator buffers
constexpr int kQChunkK = 64;
constexpr int kQChunkElems = 128 * kQChunkK;            // 16 KB
constexpr uint32_t kQChunkBytes = kQChunkElems * 2;
constexpr int kQBoxRows = 64;
constexpr int kQPanel = kQR * 64;                       // one 32-row x 64-column operand panel (4 KB)
constexpr int kQLdX = kQD + 8;
constexpr int kQLdQkv = 3 * kHeadDim + 8;
constexpr uint32_t kQIdesc = umma_idesc_bf16(128, kQR);
constexpr uint32_t kQAcc0 = 256;  // first accumulator column

// What one CTA of a C-CTA cluster (C = 4: quad kernel, C = 8: octo kernel) owns.
template <int C>
struct QK {
  static_assert(C == 4 || C == 8, "4- or 8-CTA clusters");
  static constexpr int kOwn = kQS / C;   // sessions sampled per CTA
  static constexpr int kF1 = kQF / C;    // FFN features per CTA (FFN2 K per CTA)
  static constexpr int kOf = kQD / C;    // residual features owned per CTA (o-projection, FFN2 reduction)
  static constexpr int kVs = 2048 / C;   // vocabulary slice per CTA
  static constexpr int kPerHead = C / 4; // CTAs computing one attention head
  // attention head of CTA c; with two CTAs per head each sends the peers its half of the rows
  __host__ __device__ static constexpr int head(int c) { return c / kPerHead; }
};

enum QGemm { Q_IN = 0, Q_QKV, Q_O, Q_F1, Q_F2, Q_HEAD };

struct QuadMaps {
  CUtensorMap in_proj, qkv, o, ffn1, ffn2, head;
};

// Shared-memory buffers that live in turn: the in-projection input (its
// MMAs finish before LN1 writes xa) and the position's working buffers.
// Peers push only into ab and v, never while the receiver's src is live (the
// first push of a position, R1, follows the receiver's attention).
// Attention exchange between the two warps of a TMEM lane quadrant (even and
// odd positions): their exponentials, the odd warp's partial outputs, the
// partial maxima.
struct QuadAttn {
  float e[128][17];
  float o[128][17];
  float m[2][128];
};

template <int C>
union QuadWork {
  using K = QK<C>;
  bf16 src[12 * kQPanel];  // in-projection input rows (B operand, K = 768)
  struct {
    union {
      struct {
        bf16 xa[4 * kQPanel];   // LayerNorm output (B operand)
        bf16 hid[4 * kQPanel];  // FFN hidden slice (B operand)
      };
      QuadAttn att;  // between the q|k|v MMAs and LN2 / FFN1
    };
    union V {
      bf16 qkv[kQR * kQLdQkv];     // q | k | v of the CTA's head
      float red[C - 1][K::kOf][kQR];  // FFN2 partial sums of the owned features from the peers (sender order)
      uint16_t vals[K::kOwn][2048];  // constrained values of the owned sessions
    } v;
  } a;
};

template <int C>
struct __align__(1024) QuadSmem {
  using K = QK<C>;
  bf16 ring[kQSlots][kQChunkElems];  // weight chunks (1024-byte aligned)
  bf16 ab[4 * kQPanel];              // attention output, then x'' (B operands; peers push into it)
  QuadWork<C> u;
  union X {
    bf16 x[kQR * kQLdX];                       // residual stream (row-major)
    uint16_t stage[kQS][K::kVs];                 // head values of the other CTAs' sessions, before sending
    uint16_t lists[K::kOwn][2 * kListCap + 16];  // sampler scratch (one warp per owned session)
  } xr;
  __align__(16) bf16 hb[2][K::kVs];  // head bias of positions p (p % 2) and p + 1, this CTA's vocabulary slice
  int32_t tok[kQS][kPositions];
  int32_t sess[kQS];
  uint32_t flags[kQS];                  // bit 0 unfinished, bit 1 finished, bit 2 forbid_eos
  uint32_t nf[kQS];                     // non-finite guided logit in this CTA's slice, per session
  uint32_t peer_nf[C][K::kOwn];         // from each peer: its non-finite flag of each owned session
  int64_t ctr[K::kOwn];
  int64_t seed[K::kOwn];
  int32_t inv[K::kOwn];
  int32_t last_issued[kQGroups];
  int32_t n_sess;
  int32_t err;
  int32_t producer_done;
  int32_t mma_done;
  uint32_t tmem;
  unsigned long long full[kQGroups];
  unsigned long long empty[kQGroups];
  unsigned long long dfull[kQNbuf];
  unsigned long long dempty[kQNbuf];
  unsigned long long opready;
  unsigned long long mmafin;
  unsigned long long xbar[2];
  uint32_t r1_sink;  // the head partner's attention-round word (never read)
};

template <int C>
constexpr size_t quad_smem_bytes() { return sizeof(QuadSmem<C>) + 1024; }
static_assert(quad_smem_bytes<4>() <= 232448 && quad_smem_bytes<8>() <= 232448, "quad / octo kernel shared memory");
static_assert(sizeof(QuadSmem<4>::X) >= sizeof(uint16_t) * kQS * QK<4>::kVs, "staging");
static_assert(sizeof(QuadSmem<8>::X) >= sizeof(uint16_t) * kQS * QK<8>::kVs, "staging");

template <int C>
__device__ __forceinline__ int qerr(const QuadSmem<C>& sm) { return *reinterpret_cast<const volatile int*>(&sm.err); }
__device__ __forceinline__ void qbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Byte offset of element (row r, column k) of a 32-row operand stored as
// 64-column panels with the 128-byte swizzle.
__device__ __forceinline__ int qop_off(int r, int k) {
  return (k >> 6) * (kQR * 128) + r * 128 + ((((k & 63) >> 3) ^ (r & 7)) << 4) + ((k & 7) << 1);
}
__device__ __forceinline__ uint4* qop_unit(bf16* base, int r, int k) {
  return reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(base) + qop_off(r, k));
}
__device__ __forceinline__ void qop_store(bf16* base, int r, int k, bf16 v) {
  *reinterpret_cast<bf16*>(reinterpret_cast<unsigned char*>(base) + qop_off(r, k)) = v;
}

// ---------------------------------------------------------------------------
// the per-position GEMM schedule (producer and MMA warp walk it in the same order)
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool q_has_in(bool folded, int p) { return p == 0 || !folded; }
// M-blocks (128 weight rows each) of GEMM g, and K chunks (64 columns) per M-block.
template <int C>
__device__ __forceinline__ int q_blocks(int g) {
  using K = QK<C>;
  switch (g) {
    case Q_O: return 1;
    case Q_F1: return K::kF1 / 128;
    case Q_HEAD: return K::kVs / 128;
    default: return 2;  // in-projection, q|k|v, FFN2
  }
}
template <int C>
__device__ __forceinline__ int q_kchunks(int g) {
  return g == Q_IN ? kEmbed / kQChunkK : (g == Q_F2 ? QK<C>::kF1 / kQChunkK : 4);
}
// Ring groups of GEMM g, 4 chunks each: one M-block's K = 256 (three groups
// for K = 768); with 8 CTAs FFN2's two M-blocks have K = 128 and share one.
template <int C>
__device__ __forceinline__ int q_groups(int g) { return q_blocks<C>(g) * q_kchunks<C>(g) / 4; }
// Chunk k (0..3) of ring group gr of GEMM g: its M-block b and K chunk kc.
template <int C>
__device__ __forceinline__ void q_group_chunk(int g, int gr, int k, int* b, int* kc) {
  const int per_block = q_kchunks<C>(g);
  if (per_block >= 4) {
    *b = gr / (per_block / 4);
    *kc = 4 * (gr % (per_block / 4)) + k;
  } else {
    *b = 2 * gr + k / 2;
    *kc = k % 2;
  }
}

// Tensor map and origins of chunk (M-block b, K-chunk k) of GEMM g: K column
// x0, rows ra (A rows 0..63) and rb (A rows 64..127); rb < 0 when the block
// has 64 weight rows only (A rows 64..127 keep stale weights, and the
// epilogue ignores their lanes).
template <int C>
__device__ __forceinline__ const CUtensorMap* q_chunk(const QuadMaps& m, int c, int p, int g, int b, int k, int* x0,
                                                      int* ra, int* rb) {
  using K = QK<C>;
  const int h = K::head(c);
  *x0 = kQChunkK * k;
  switch (g) {
    case Q_IN:
      *ra = 128 * b;
      *rb = 128 * b + 64;
      return &m.in_proj;
    case Q_QKV:  // block 0: head h's q and k rows; block 1: its v rows
      *ra = b == 0 ? kHeadDim * h : 2 * kQD + kHeadDim * h;
      *rb = b == 0 ? kQD + kHeadDim * h : -1;
      return &m.qkv;
    case Q_O:  // output features [kOf c, +kOf) in one 64-row box (8 CTAs: its upper 32 rows unused,
               // past the matrix for the last CTA: zero fill)
      *ra = K::kOf * c;
      *rb = -1;
      return &m.o;
    case Q_F1:
      *ra = K::kF1 * c + 128 * b;
      *rb = *ra + 64;
      return &m.ffn1;
    case Q_F2:
      *x0 = K::kF1 * c + kQChunkK * k;
      *ra = 128 * b;
      *rb = 128 * b + 64;
      return &m.ffn2;
    default: {
      const int base = p * kVocab + K::kVs * c + 128 * b;  // the last CTA's last block overhangs (ignored / zero fill)
      *ra = base;
      *rb = base + 64;
      return &m.head;
    }
  }
}

// The producer fills the ring a group of 4 chunks at a time, all four landing
// on the group's one barrier.
template <int C>
__device__ void q_producer(QuadSmem<C>& sm, const QuadMaps& maps, int c, bool folded) {
  int git = 0;  // groups issued
  for (int p = 0; p < kPositions; ++p) {
    for (int g = q_has_in(folded, p) ? Q_IN : Q_QKV; g <= Q_HEAD; ++g) {
      const int ng = q_groups<C>(g);
      for (int gr = 0; gr < ng; ++gr, ++git) {
        const int gi = git % kQGroups;
        if (git >= kQGroups && qerr(sm) == 0 && !mbar_wait_cta(&sm.empty[gi], ((git / kQGroups) - 1) & 1)) {
          sm.err = 1;
        }
        if (qerr(sm)) return;
        int b, kc, x0, ra, rb;
        q_group_chunk<C>(g, gr, 0, &b, &kc);
        q_chunk<C>(maps, c, p, g, b, kc, &x0, &ra, &rb);
        mbar_expect_tx(&sm.full[gi], 4 * (rb < 0 ? kQChunkBytes / 2 : kQChunkBytes));
#pragma unroll 1
        for (int k = 0; k < 4; ++k) {
          q_group_chunk<C>(g, gr, k, &b, &kc);
          const CUtensorMap* map = q_chunk<C>(maps, c, p, g, b, kc, &x0, &ra, &rb);
          bf16* dst = sm.ring[4 * gi + k];
          tma_load_2d(dst, map, x0, ra, &sm.full[gi]);
          if (rb >= 0) tma_load_2d(dst + kQBoxRows * 64, map, x0, rb, &sm.full[gi]);
        }
        sm.last_issued[gi] = git;
      }
    }
  }
}

template <int C>
__device__ __forceinline__ const bf16* q_operand(QuadSmem<C>& sm, int g) {
  switch (g) {
    case Q_IN: return sm.u.src;
    case Q_QKV: return sm.u.a.xa;
    case Q_O: return sm.ab;
    case Q_F1: return sm.u.a.xa;
    case Q_F2: return sm.u.a.hid;
    default: return sm.ab;
  }
}

// The MMA warp's single thread: per GEMM wait until the consumers have
// written its B operand; per M-block wait for a free accumulator buffer; per
// ring group (4 weight chunks) wait on the group's barrier, then issue its 16
// MMAs as one straight-line burst (a branch between tcgen05.mma instructions
// halves their issue rate) and free the group.  The ring is consumed in
// order by this one thread, so every parity wait is for the phase right
// after the one it last saw complete.
template <int C>
__device__ void q_mma(QuadSmem<C>& sm, bool folded) {
  constexpr uint64_t kSlotStep = kQChunkElems * 2 / 16, kPanelStep = kQPanel * 2 / 16;
  int git = 0, mb = 0, gn = 0;
  for (int p = 0; p < kPositions && qerr(sm) == 0; ++p) {
    for (int g = q_has_in(folded, p) ? Q_IN : Q_QKV; g <= Q_HEAD && qerr(sm) == 0; ++g) {
      if (!mbar_wait_cta(&sm.opready, gn & 1)) {
        sm.err = 1;
        break;
      }
      ++gn;
      tmem_fence_after_sync();
      const bf16* bop = q_operand(sm, g);
      const int nb = q_blocks<C>(g), per_block = q_kchunks<C>(g);
      bool ok = true;
      if (per_block >= 4) {
        const int ng = per_block / 4;
        for (int b = 0; b < nb; ++b, ++mb) {
          const int db = mb % kQNbuf, use = mb / kQNbuf;
          ok = use < 1 || mbar_wait_cta(&sm.dempty[db], (use - 1) & 1);
          const uint32_t d = sm.tmem + kQAcc0 + 32u * static_cast<uint32_t>(db);
          for (int gr = 0; gr < ng && ok; ++gr, ++git) {
            const int gi = git % kQGroups;
            ok = mbar_wait_cta(&sm.full[gi], (git / kQGroups) & 1);
            if (!ok) break;
            tmem_fence_after_sync();
            const uint64_t b0 = umma_desc_sw128(bop + 4 * gr * kQPanel);
            const uint64_t a0 = umma_desc_sw128(sm.ring[4 * gi]);
            const bool acc0 = gr != 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                umma_bf16(d, a0 + k * kSlotStep + 2 * kk, b0 + k * kPanelStep + 2 * kk, kQIdesc,
                          acc0 || (k | kk) != 0);
              }
            }
            umma_commit(&sm.empty[gi]);
          }
          if (!ok) break;
          umma_commit(&sm.dfull[db]);
        }
      } else {
        // one group holds two M-blocks of K = 128 (FFN2 with 8 CTAs): chunks
        // 0, 1 accumulate into block mb's buffer, chunks 2, 3 into mb + 1's
        const int db0 = mb % kQNbuf, db1 = (mb + 1) % kQNbuf;
        const int use0 = mb / kQNbuf, use1 = (mb + 1) / kQNbuf;
        ok = use0 < 1 || mbar_wait_cta(&sm.dempty[db0], (use0 - 1) & 1);
        ok = ok && (use1 < 1 || mbar_wait_cta(&sm.dempty[db1], (use1 - 1) & 1));
        const int gi = git % kQGroups;
        ok = ok && mbar_wait_cta(&sm.full[gi], (git / kQGroups) & 1);
        if (ok) {
          tmem_fence_after_sync();
          const uint32_t d0 = sm.tmem + kQAcc0 + 32u * static_cast<uint32_t>(db0);
          const uint32_t d1 = sm.tmem + kQAcc0 + 32u * static_cast<uint32_t>(db1);
          const uint64_t b0 = umma_desc_sw128(bop);
          const uint64_t a0 = umma_desc_sw128(sm.ring[4 * gi]);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              umma_bf16(k < 2 ? d0 : d1, a0 + k * kSlotStep + 2 * kk, b0 + (k & 1) * kPanelStep + 2 * kk, kQIdesc,
                        ((k & 1) | kk) != 0);
            }
          }
          umma_commit(&sm.empty[gi]);
          umma_commit(&sm.dfull[db0]);
          umma_commit(&sm.dfull[db1]);
        }
        ++git;
        mb += 2;
      }
      if (!ok) {
        sm.err = 1;
        break;
      }
    }
  }
  umma_commit(&sm.mmafin);
  mbar_wait_cta(&sm.mmafin, 0);
  atomicExch(&sm.mma_done, 1);
}

// ---------------------------------------------------------------------------
// consumer helpers
// ---------------------------------------------------------------------------

// Epilogue read of M-block mb: warp w takes TMEM lanes [32 (w % 4), +32) (A
// rows m) and columns [16 (w / 4), +16): v[i] = tile row 16 (w / 4) + i.
template <int C>
__device__ __forceinline__ void q_load_block(QuadSmem<C>& sm, int mb, float (&v)[16]) {
  const int warp = threadIdx.x >> 5;
  const int db = mb % kQNbuf, use = mb / kQNbuf;
  if (qerr(sm) == 0 && !mbar_wait_cta(&sm.dfull[db], use & 1)) sm.err = 1;
  tmem_fence_after_sync();
  uint32_t r[16];
  tmem_ld16(r, sm.tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + kQAcc0 + 32u * db + 16u * (warp >> 2));
  tmem_fence_before_sync();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.dempty[db]);
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// B operand written: order the generic writes before the MMA warp's reads.
template <int C>
__device__ __forceinline__ void q_operand_ready(QuadSmem<C>& sm) {
  fence_proxy_async();
  qbar();
  if (threadIdx.x == 0) mbar_arrive(&sm.opready);
}

// LayerNorm (no bias, eps 1e-5) of the 32 rows of x into the B operand xa;
// lane holds weights g of columns [8 lane, +8); warp w: rows [4 w, +4).
// LayerNorm (no bias, eps 1e-5) of the warp's rows [4 w, +4), held by lane
// as columns [8 lane, +8) in v, into the B operand xa (lane holds weights g).
__device__ __forceinline__ void q_layer_norm_rows(float (&v)[kQR / kQW][8], bf16* xa, const float (&g)[8]) {
  constexpr int kRows = kQR / kQW;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float sum[kRows], var[kRows];
#pragma unroll
  for (int rr = 0; rr < kRows; ++rr) {
    sum[rr] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum[rr] += v[rr][j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr) sum[rr] += __shfl_xor_sync(0xffffffffu, sum[rr], o);
  }
#pragma unroll
  for (int rr = 0; rr < kRows; ++rr) {
    const float mean = sum[rr] / static_cast<float>(kQD);
    sum[rr] = mean;
    var[rr] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) var[rr] += (v[rr][j] - mean) * (v[rr][j] - mean);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr) var[rr] += __shfl_xor_sync(0xffffffffu, var[rr], o);
  }
#pragma unroll
  for (int rr = 0; rr < kRows; ++rr) {
    const float mean = sum[rr];
    const float rstd = 1.0f / sqrtf(var[rr] / static_cast<float>(kQD) + 1.0e-5f);
    float out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = ((v[rr][j] - mean) * rstd) * g[j];
    *qop_unit(xa, kRows * warp + rr, lane * 8) = pack8(out);
  }
}

// LayerNorm of the 32 rows of x (row-major) into xa; warp w: rows [4 w, +4).
__device__ __forceinline__ void q_layer_norm(const bf16* x, bf16* xa, const float (&g)[8]) {
  constexpr int kRows = kQR / kQW;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float v[kRows][8];
#pragma unroll
  for (int rr = 0; rr < kRows; ++rr) unpack8(*reinterpret_cast<const uint4*>(x + (kRows * warp + rr) * kQLdX + lane * 8), v[rr]);
  q_layer_norm_rows(v, xa, g);
}

// Wait for round rd: this CTA announces on its own round barrier the bytes
// its peers push to it in this round, and the round completes when they have
// all landed.
template <int C>
__device__ __forceinline__ void q_round(QuadSmem<C>& sm, uint32_t& rd, uint32_t bytes_in) {
  qbar();
  const int bar = static_cast<int>(rd & 1u);
  if (threadIdx.x == 0) mbar_expect_tx(&sm.xbar[bar], bytes_in);
  if (qerr(sm) == 0 && !mbar_wait(&sm.xbar[bar], (rd >> 1) & 1u)) sm.err = 1;
  ++rd;
}

template <int C>
__device__ __forceinline__ uint32_t q_round_bar(QuadSmem<C>& sm, uint32_t rd, int peer) {
  return cluster_addr(&sm.xbar[rd & 1u], peer);
}

// Vocabulary values CTA j holds of each session (its slice, clipped to the vocabulary).
template <int C>
__host__ __device__ constexpr int q_slice_len(int j) {
  return QK<C>::kVs * (j + 1) <= kVocab ? QK<C>::kVs : kVocab - QK<C>::kVs * j;
}

// Bytes CTA c receives in the head-values round: from every peer j its slice
// of each of c's sessions plus one non-finite flag per session.
template <int C>
__device__ __forceinline__ uint32_t q_values_bytes_in(int c) {
  using K = QK<C>;
  uint32_t b = 0;
#pragma unroll
  for (int j = 0; j < C; ++j) {
    if (j != c) b += static_cast<uint32_t>(K::kOwn * (q_slice_len<C>(j) * 2 + 4));
  }
  return b;
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// TMEM column block of cached position j: even positions in blocks 0..7,
// odd ones in 8..15, so each of the two attention warps of a lane quadrant
// reads its positions with one 64-column load.
__device__ __forceinline__ uint32_t q_kv_block(int j) { return 8u * static_cast<uint32_t>(j & 1) + (j >> 1); }

// Attention of the CTA's head h for the tile's 32 rows at position p, all 8
// consumer warps: warp w reads TMEM lane quadrant q = w % 4 and takes the
// positions of parity w / 4; thread (w, l) = row 8 q + l / 4, head dims
// [16 (l % 4), +16).  This position's k and v go into the TMEM cache (K at
// column 8 b(j), V at 128 + 8 b(j)); scores, exponentials and the softmax sum
// as the reference takes them (sum over positions in order); each warp sums
// its positions' values; the even warp adds the odd warp's partial output and
// writes the output columns into ab and the peers' ab.  With two CTAs per
// head (C = 8) both compute all 32 rows and each sends the other six CTAs its
// half of them (rows [16 (c % 2), +16)).
template <int C>
__device__ __forceinline__ void q_attention(QuadSmem<C>& sm, int p, int c, uint32_t rd) {
  using K = QK<C>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q4 = warp & 3, part = warp >> 2;
  const int r = 8 * q4 + (lane >> 2), u = lane & 3;
  const int t128 = 32 * q4 + lane;
  const uint32_t tl = sm.tmem + (static_cast<uint32_t>(32 * q4) << 16);
  const bf16* row = sm.u.a.v.qkv + r * kQLdQkv;
  QuadAttn& at = sm.u.a.att;
  float q[16];
  {
    uint32_t kk[8], vv[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 qa = *reinterpret_cast<const uint4*>(row + 16 * u + 8 * h);
      float f8[8];
      unpack8(qa, f8);
#pragma unroll
      for (int e = 0; e < 8; ++e) q[8 * h + e] = f8[e];
      const uint4 ka = *reinterpret_cast<const uint4*>(row + kHeadDim + 16 * u + 8 * h);
      const uint4 va = *reinterpret_cast<const uint4*>(row + 2 * kHeadDim + 16 * u + 8 * h);
      kk[4 * h] = ka.x, kk[4 * h + 1] = ka.y, kk[4 * h + 2] = ka.z, kk[4 * h + 3] = ka.w;
      vv[4 * h] = va.x, vv[4 * h + 1] = va.y, vv[4 * h + 2] = va.z, vv[4 * h + 3] = va.w;
    }
    // the warp that takes position p's parity caches it (only that warp reads it)
    if ((p & 1) == part) {
      tmem_st8(tl + 8u * q_kv_block(p), kk);
      tmem_st8(tl + 128u + 8u * q_kv_block(p), vv);
      tmem_wait_st();
    }
  }
  // scores of this warp's positions j = 2 i + part <= p
  float s[8];
  float mloc = -CUDART_INF_F;
  {
    uint32_t kv[64];
    tmem_ld64(kv, tl + 64u * part);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float2 t0 = __bfloat1622float2(bf2_of(kv[8 * i + e]));
        const float2 t1 = __bfloat1622float2(bf2_of(kv[8 * i + e + 1]));
        d0 = fmaf(q[2 * e], t0.x, d0);
        d0 = fmaf(q[2 * e + 1], t0.y, d0);
        d1 = fmaf(q[2 * e + 2], t1.x, d1);
        d1 = fmaf(q[2 * e + 3], t1.y, d1);
      }
      float dot = d0 + d1;
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      s[i] = 2 * i + part <= p ? round_bf16(__fmul_rn(round_bf16(dot), 0.125f)) : -CUDART_INF_F;
      mloc = fmaxf(mloc, s[i]);
    }
  }
  at.m[part][t128] = mloc;
  qbar();
  const float mx = fmaxf(at.m[0][t128], at.m[1][t128]);
  float e[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    e[i] = 2 * i + part <= p ? expf(s[i] - mx) : 0.f;
    at.e[t128][2 * i + part] = e[i];
  }
  qbar();
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPositions; ++j) sum += at.e[t128][j];
  float o[16];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d] = 0.f;
  {
    uint32_t kv[64];
    tmem_ld64(kv, tl + 128u + 64u * part);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (2 * i + part <= p) {
        const float pr = round_bf16(e[i] / sum);
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          const float2 t = __bfloat1622float2(bf2_of(kv[8 * i + d]));
          o[2 * d] = fmaf(pr, t.x, o[2 * d]);
          o[2 * d + 1] = fmaf(pr, t.y, o[2 * d + 1]);
        }
      }
    }
  }
  if (part == 1) {
#pragma unroll
    for (int d = 0; d < 16; ++d) at.o[t128][d] = o[d];
  }
  qbar();
  if (part == 0) {
    float lo[8], hi[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      lo[d] = o[d] + at.o[t128][d];
      hi[d] = o[8 + d] + at.o[t128][8 + d];
    }
    const int k0 = kHeadDim * K::head(c) + 16 * u;
    uint4* d0 = qop_unit(sm.ab, r, k0);
    uint4* d1 = qop_unit(sm.ab, r, k0 + 8);
    const uint4 w0 = pack8(lo), w1 = pack8(hi);
    *d0 = w0;
    *d1 = w1;
    if (K::kPerHead == 1 || (q4 >> 1) == (c & 1)) {
#pragma unroll
      for (int j = 0; j < C; ++j) {
        if (K::head(j) != K::head(c)) {
          const uint32_t bar = q_round_bar(sm, rd, j);
          st_async_v4(cluster_addr(d0, j), w0, bar);
          st_async_v4(cluster_addr(d1, j), w1, bar);
        }
      }
    }
  }
  // The head partner sends no rows in this round, only a word, so that this
  // round, like every other, completes only after every peer has reached it
  // (no CTA runs a round ahead into buffers its partner still uses).
  if (K::kPerHead > 1 && threadIdx.x == 0) {
    st_async_b32(cluster_addr(&sm.r1_sink, c ^ 1), 0u, q_round_bar(sm, rd, c ^ 1));
  }
}

template <int C>
__device__ __forceinline__ int64_t q_input_token(const Frame& f, const QuadSmem<C>& sm, int slot, int p) {
  if (f.forced) {
    const int64_t t = f.forced[static_cast<int64_t>(sm.sess[slot]) * kPositions + p];
    return t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
  }
  return sm.tok[slot][p];
}

__device__ __forceinline__ void q_stamp(const Frame& f, bool tracer, int p, int i) {
  if (tracer) f.trace[kPositions * p + i] = static_cast<uint64_t>(clock64());
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

template <int C>
__global__ void __launch_bounds__(kQThreads, 1) quad_frame_kernel(Frame f, const __grid_constant__ QuadMaps maps) {
  using K = QK<C>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
  QuadSmem<C>& sm = *reinterpret_cast<QuadSmem<C>*>(smem_raw + pad);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rp = f.rp;
  const bool folded = f.emb_proj != nullptr;
  const int c = static_cast<int>(cg::this_cluster().block_rank());
  const int tile = static_cast<int>(blockIdx.x) / C;
  const bool tracer = f.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0;

  // ---- sessions [16 tile, +16) of the active list (every CTA of the cluster)
  if (warp == 0) {
    int seen = 0;
    const int first = kQS * tile;
    for (int base = 0; base < f.n; base += 32) {
      const int s = base + lane;
      const bool act = s < f.n && (f.active == nullptr || f.active[s]);
      const unsigned m = __ballot_sync(0xffffffffu, act);
      const int rank = seen + __popc(m & ((1u << lane) - 1u));
      if (act && rank >= first && rank < first + kQS) sm.sess[rank - first] = s;
      seen += __popc(m);
    }
    if (lane == 0) {
      const int left = seen - first;
      sm.n_sess = left <= 0 ? 0 : (left < kQS ? left : kQS);
      sm.err = 0;
      sm.producer_done = 0;
      sm.mma_done = 0;
    }
  }
  __syncthreads();
  const int n_sess = sm.n_sess;
  if (n_sess == 0) return;  // the same in every CTA of the cluster: none touches another
  auto live = [&](int r) { return (r >> 1) < n_sess && (r & 1) < rp; };
  const int own0 = K::kOwn * c;
  const int n_own = n_sess - own0 <= 0 ? 0 : (n_sess - own0 < K::kOwn ? n_sess - own0 : K::kOwn);
  if (tracer) f.trace[256] = static_cast<uint64_t>(clock64()), f.trace[257] = global_ns();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQGroups; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
      sm.last_issued[s] = -1;
    }
    for (int b = 0; b < kQNbuf; ++b) {
      mbar_init(&sm.dfull[b], 1);
      mbar_init(&sm.dempty[b], kQW);
    }
    mbar_init(&sm.xbar[0], 1);
    mbar_init(&sm.xbar[1], 1);
    mbar_init(&sm.opready, 1);
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
  cg::this_cluster().sync();  // every CTA's barriers exist before any push

  if (warp >= kQW) {  // control warpgroup
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kQProducerRegs));
    if (warp == kQW && lane == 0) {
      q_producer(sm, maps, c, folded);
      // no copy may still be writing when the CTA leaves
      for (int s = 0; s < kQGroups; ++s) {
        const int last = sm.last_issued[s];
        if (last >= 0) mbar_wait_cta(&sm.full[s], (last / kQGroups) & 1);
      }
      atomicExch(&sm.producer_done, 1);
    } else if (warp == kQW + 1 && lane == 0) {
      q_mma(sm, folded);
    }
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kQConsumerRegs));
  {
    float g1[8], g2[8];
    unpack8(*reinterpret_cast<const uint4*>(f.ln1 + lane * 8), g1);
    unpack8(*reinterpret_cast<const uint4*>(f.ln2 + lane * 8), g2);
    const int q4 = warp & 3, sh = warp >> 2;
    const int m_lane = 32 * q4 + lane;  // A row of an M-block held by this thread
    const bool cfg = rp == 2;
    const float cfg_scale = f.prm.cfg_scale, uncond_scale = __fsub_rn(1.0f, f.prm.cfg_scale);
    int mb = 0;       // M-blocks consumed
    uint32_t rd = 0;  // exchange rounds
    if (threadIdx.x < K::kVs / 8) {  // head bias of position 0
      const int v0 = K::kVs * c + 8 * threadIdx.x;
      const uint4 z = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sm.hb[0] + 8 * threadIdx.x) = v0 < kVocab ? *reinterpret_cast<const uint4*>(f.head_b + v0) : z;
      *reinterpret_cast<uint4*>(sm.hb[1] + 8 * threadIdx.x) = z;
    }
    // flags of the 8 sessions whose rows this thread holds in the head epilogue
    uint32_t fl8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) fl8[i] = 8 * sh + i < n_sess ? sm.flags[8 * sh + i] : 0u;
    for (int p = 0; p < kPositions; ++p) {
      q_stamp(f, tracer, p, 0);
      // ---------------- input rows
      if (q_has_in(folded, p)) {
        // the rows' 768 inputs: p = 0 the decoder hidden, else the sampled token's embedding
        for (int i = threadIdx.x; i < kQR * (kEmbed / 8); i += kQT) {
          const int r = i / (kEmbed / 8), k8 = 8 * (i % (kEmbed / 8));
          uint4 v = make_uint4(0, 0, 0, 0);
          if (live(r)) {
            const int slot = r >> 1, sub = r & 1;
            const bf16* src;
            if (p == 0) {
              src = f.hidden + (static_cast<int64_t>(sm.sess[slot]) * rp + sub) * kEmbed;
            } else {
              src = f.emb + (static_cast<int64_t>(p - 1) * kVocab + q_input_token(f, sm, slot, p - 1)) * kEmbed;
            }
            v = *reinterpret_cast<const uint4*>(src + k8);
          }
          *qop_unit(sm.u.src, r, k8) = v;
        }
        q_operand_ready(sm);
        const bf16* pos = f.pos + static_cast<int64_t>(p) * kQD;
        for (int b = 0; b < 2; ++b, ++mb) {
          float v[16];
          q_load_block(sm, mb, v);
          const int n = 128 * b + m_lane;
          const float bias = bf2f(f.in_b[n]), pe = bf2f(pos[n]);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float y = round_bf16(__fadd_rn(v[i], bias));
            sm.xr.x[(16 * sh + i) * kQLdX + n] = f2bf(__fadd_rn(y, pe));
          }
        }
      }
      // head bias: position p's slice has landed (issued a position ahead),
      // position p + 1's is issued now; per-position flags
      if (threadIdx.x < K::kVs / 8) {
        const int v0 = K::kVs * c + 8 * threadIdx.x;
        if (v0 < kVocab) {  // kVocab % 8 == 0; the slice's tail past the vocabulary stays zero
          cp_async_wait_all();
          if (p + 1 < kPositions) {
            cp_async16(sm.hb[(p + 1) & 1] + 8 * threadIdx.x, f.head_b + static_cast<int64_t>(p + 1) * kVocab + v0);
          }
        }
      }
      if (threadIdx.x < kQS) sm.nf[threadIdx.x] = 0;

      // ---------------- LN1 (with the folded tables done by the previous
      // position's row gather), q|k|v of head c
      if (q_has_in(folded, p)) {
        qbar();
        q_layer_norm(sm.xr.x, sm.u.a.xa, g1);
      }
      q_operand_ready(sm);
      q_stamp(f, tracer, p, 1);
      for (int b = 0; b < 2; ++b, ++mb) {
        float v[16];
        q_load_block(sm, mb, v);
        if (b == 0 || m_lane < kHeadDim) {
          const int col = b == 0 ? m_lane : 2 * kHeadDim + m_lane;  // q | k | v
#pragma unroll
          for (int i = 0; i < 16; ++i) sm.u.a.v.qkv[(16 * sh + i) * kQLdQkv + col] = f2bf(v[i]);
        }
      }
      qbar();
      q_stamp(f, tracer, p, 2);

      // ---------------- attention (R1: head c's output columns to every CTA)
      q_attention(sm, p, c, rd);
      q_stamp(f, tracer, p, 3);
      q_round(sm, rd, static_cast<uint32_t>((C - K::kPerHead) * (kQR / K::kPerHead) * kHeadDim * 2 +
                                            (K::kPerHead > 1 ? 4 : 0)));
      fence_proxy_async();
      q_operand_ready(sm);
      q_stamp(f, tracer, p, 4);

      // ---------------- o-projection features [64 c, +64) + residual (R2: the slice to every CTA), LN2
      {
        float v[16];
        q_load_block(sm, mb, v);
        ++mb;
        if (m_lane < K::kOf) {
          const int n = K::kOf * c + m_lane;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            bf16* xr = sm.xr.x + (16 * sh + i) * kQLdX + n;
            *xr = f2bf(__fadd_rn(bf2f(*xr), round_bf16(v[i])));
          }
        }
      }
      qbar();
      if (8 * warp < K::kOf) {
        // thread: row lane, features [kOf c + 8 warp, +8)
        const uint4* src = reinterpret_cast<const uint4*>(sm.xr.x + lane * kQLdX + K::kOf * c + 8 * warp);
        const uint4 w = *src;
#pragma unroll
        for (int j = 0; j < C; ++j) {
          if (j != c) st_async_v4(cluster_addr(src, j), w, q_round_bar(sm, rd, j));
        }
      }
      q_round(sm, rd, static_cast<uint32_t>((C - 1) * kQR * K::kOf * 2));
      q_stamp(f, tracer, p, 5);
      q_layer_norm(sm.xr.x, sm.u.a.xa, g2);
      q_operand_ready(sm);
      q_stamp(f, tracer, p, 6);

      // ---------------- FFN1 + GELU (features [kF1 c, +kF1))
      for (int b = 0; b < K::kF1 / 128; ++b, ++mb) {
        float v[16];
        q_load_block(sm, mb, v);
        const int fl = 128 * b + m_lane;
#pragma unroll
        for (int i = 0; i < 16; ++i) qop_store(sm.u.a.hid, 16 * sh + i, fl, f2bf(gelu_tanh(round_bf16(v[i]))));
      }
      q_operand_ready(sm);
      q_stamp(f, tracer, p, 7);

      // ---------------- FFN2 partials (R3 to the feature owners), sum, + residual (R4)
      for (int b = 0; b < 2; ++b, ++mb) {
        float v[16];
        q_load_block(sm, mb, v);
        const int n = 128 * b + m_lane;
        const int owner = n / K::kOf, nl = n % K::kOf;
        // the owner keeps its own partials in xa (free after the FFN1 MMAs), the
        // peers' in red[slot], slot = the sender's rank skipping the owner's
        float* dst = owner == c ? reinterpret_cast<float*>(sm.u.a.xa) + nl * kQR + 16 * sh
                                : &sm.u.a.v.red[c < owner ? c : c - 1][nl][16 * sh];
        if (owner == c) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
          const uint32_t bar = q_round_bar(sm, rd, owner);
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            st_async_v4(cluster_addr(dst + i, owner),
                        make_uint4(__float_as_uint(v[i]), __float_as_uint(v[i + 1]), __float_as_uint(v[i + 2]),
                                   __float_as_uint(v[i + 3])),
                        bar);
          }
        }
      }
      q_stamp(f, tracer, p, 8);
      q_round(sm, rd, static_cast<uint32_t>((C - 1) * K::kOf * kQR * 4));
      q_stamp(f, tracer, p, 9);
      if (8 * warp < K::kOf) {
        // thread: row lane, features [8 warp, +8) of this CTA's kOf
        const int r = lane, nl = 8 * warp;
        const int k0 = K::kOf * c + nl;
        float xv[8];
        unpack8(*reinterpret_cast<const uint4*>(sm.xr.x + r * kQLdX + k0), xv);
        // the C partials in CTA order: this CTA's own in xa, the peers' in red
        const float* src[C];
#pragma unroll
        for (int j = 0; j < C; ++j) {
          src[j] = (j == c ? reinterpret_cast<const float*>(sm.u.a.xa) : &sm.u.a.v.red[j < c ? j : j - 1][0][0]) +
                   nl * kQR + r;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float s = src[0][e * kQR];
#pragma unroll
          for (int j = 1; j < C; ++j) s = __fadd_rn(s, src[j][e * kQR]);
          xv[e] = __fadd_rn(xv[e], round_bf16(s));
        }
        const uint4 w = pack8(xv);
        uint4* d = qop_unit(sm.ab, r, k0);
        *d = w;
#pragma unroll
        for (int j = 0; j < C; ++j) {
          if (j != c) st_async_v4(cluster_addr(d, j), w, q_round_bar(sm, rd, j));
        }
      }
      q_round(sm, rd, static_cast<uint32_t>((C - 1) * kQR * K::kOf * 2));
      fence_proxy_async();
      q_operand_ready(sm);
      q_stamp(f, tracer, p, 10);

      // ---------------- head p: bias, CFG combine, constraints (R5: values to the owners)
      {
        bf16* lo_base = f.logits_out;
        const bf16* hbp = sm.hb[p & 1];
        for (int b = 0; b < K::kVs / 128; ++b, ++mb) {
          float v[16];
          q_load_block(sm, mb, v);
          const int vl = 128 * b + m_lane;
          const int t = K::kVs * c + vl;
          const bool in_vocab = t < kVocab;
          const float bias = bf2f(hbp[vl]);
          uint32_t nfm = 0;
#pragma unroll
          for (int i2 = 0; i2 < 4; ++i2) {
            // sessions 8 sh + 2 i2 (low halves) and + 1 (high halves): rows 2 s, 2 s + 1
            const uint32_t cc = pack2_rn(__fadd_rn(v[4 * i2], bias), __fadd_rn(v[4 * i2 + 2], bias));
            const uint32_t uu = pack2_rn(__fadd_rn(v[4 * i2 + 1], bias), __fadd_rn(v[4 * i2 + 3], bias));
            const int s0 = 8 * sh + 2 * i2;
            if (lo_base != nullptr && in_vocab) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (s0 + h < n_sess) {
                  uint16_t* lr = reinterpret_cast<uint16_t*>(lo_base) +
                                 (static_cast<int64_t>(sm.sess[s0 + h]) * kPositions + p) * rp * kVocab;
                  lr[t] = static_cast<uint16_t>(h ? cc >> 16 : cc & 0xffffu);
                  if (cfg) lr[kVocab + t] = static_cast<uint16_t>(h ? uu >> 16 : uu & 0xffffu);
                }
              }
            }
            const uint32_t g = cfg ? guided_value2(cc, uu, cfg_scale, uncond_scale) : cc;
            uint32_t g0 = g & 0xffffu, g1 = g >> 16;
            const uint32_t f0 = fl8[2 * i2], f1 = fl8[2 * i2 + 1];
            if (t >= kCodebook || (g0 & 0x7f80u) == 0x7f80u || (g1 & 0x7f80u) == 0x7f80u || ((f0 | f1) & 2u)) {
              bool n0 = false, n1 = false;
              g0 = constrain(g0, t, f0 & 1u, (f0 & 2u) != 0, (f0 & 4u) != 0, n0);
              g1 = constrain(g1, t, f1 & 1u, (f1 & 2u) != 0, (f1 & 4u) != 0, n1);
              if (in_vocab) nfm |= (n0 ? 1u : 0u) << (2 * i2) | (n1 ? 1u : 0u) << (2 * i2 + 1);
            }
            if (in_vocab) {
              // slots s0, s0 + 1 share their owner (owners hold 4 aligned slots)
              const int owner = s0 / K::kOwn;
              if (owner == c) {
                sm.u.a.v.vals[s0 - own0][t] = static_cast<uint16_t>(g0);
                sm.u.a.v.vals[s0 + 1 - own0][t] = static_cast<uint16_t>(g1);
              } else {
                sm.xr.stage[s0][vl] = static_cast<uint16_t>(g0);
                sm.xr.stage[s0 + 1][vl] = static_cast<uint16_t>(g1);
              }
            }
          }
          const uint32_t any = __reduce_or_sync(0xffffffffu, nfm);
          if (lane == 0 && any != 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              if (any & (1u << i)) atomicOr(&sm.nf[8 * sh + i], 1u);
            }
          }
        }
        qbar();
        q_stamp(f, tracer, p, 11);
        // the other CTAs' sessions: this CTA's vocabulary slice of each (all
        // four slots of every owner, live or not), and its non-finite flags
        const int units = q_slice_len<C>(c) / 8;
        constexpr int kOther = kQS - K::kOwn;
        for (int i = threadIdx.x; i < kOther * (K::kVs / 8); i += kQT) {
          const int oi = i / (K::kVs / 8), un = i % (K::kVs / 8);
          if (un < units) {
            const int slot = oi < own0 ? oi : oi + K::kOwn;  // skip the owned slots
            const int owner = slot / K::kOwn;
            const uint4 val = *reinterpret_cast<const uint4*>(&sm.xr.stage[slot][8 * un]);
            st_async_v4(cluster_addr(&sm.u.a.v.vals[slot - K::kOwn * owner][K::kVs * c + 8 * un], owner), val,
                        q_round_bar(sm, rd, owner));
          }
        }
        if (threadIdx.x < kQS) {
          const int slot = threadIdx.x;
          const int owner = slot / K::kOwn;
          if (owner != c) {
            st_async_b32(cluster_addr(&sm.peer_nf[c][slot - K::kOwn * owner], owner), sm.nf[slot],
                         q_round_bar(sm, rd, owner));
          }
        }
        q_round(sm, rd, q_values_bytes_in<C>(c));
      }
      q_stamp(f, tracer, p, 12);

      // ---------------- sampling (R6: the token to every CTA): one warp per owned
      // session (two warps per session with sample_group measured slower here)
      if (warp < n_own) {
        const int ls = warp, slot = own0 + ls;
        uint32_t nfs = sm.nf[slot];
#pragma unroll
        for (int j = 0; j < C; ++j) {
          if (j != c) nfs |= sm.peer_nf[j][ls];
        }
        RowSample rs;
        rs.vals = sm.u.a.v.vals[ls];
        rs.flags = sm.flags[slot];
        rs.nonfinite = nfs != 0;
        rs.seed = sm.seed[ls];
        rs.counter = sm.ctr[ls];
        int invalid = 0;
        uint16_t* list = sm.xr.lists[ls];
        const int token = sample_row(rs, f.prm, list, list + kListCap + 16, &invalid);
        __syncwarp();
        if (lane == 0) {
          const int64_t counter = sm.ctr[ls];
          sm.tok[slot][p] = token;
          sm.inv[ls] |= invalid;
          const bool counter_valid = counter >= 0 && counter <= kMaxCounter;
          if (!f.prm.argmax && counter_valid) sm.ctr[ls] = counter + 1;
          if (p + 1 < kPositions) {
#pragma unroll
            for (int j = 0; j < C; ++j) {
              if (j != c) {
                st_async_b32(cluster_addr(&sm.tok[slot][p], j), static_cast<uint32_t>(token),
                             q_round_bar(sm, rd, j));
              }
            }
          }
        }
      }
      q_stamp(f, tracer, p, 13);
      if (p + 1 < kPositions) {
        // dead owned slots still announce their 4 bytes: push a zero token for them
        if (threadIdx.x >= n_own && threadIdx.x < K::kOwn) {
          const int slot = own0 + threadIdx.x;
          sm.tok[slot][p] = 0;
#pragma unroll
          for (int j = 0; j < C; ++j) {
            if (j != c) st_async_b32(cluster_addr(&sm.tok[slot][p], j), 0u, q_round_bar(sm, rd, j));
          }
        }
        q_round(sm, rd, static_cast<uint32_t>((C - 1) * K::kOwn * 4));
      } else {
        qbar();
      }
      q_stamp(f, tracer, p, 14);

      // ---------------- next input rows (folded tables), every CTA, all rows,
      // and their LN1 for the next position's q|k|v (warp w: rows [4 w, +4))
      if (folded && p + 1 < kPositions) {
        constexpr int kRows = kQR / kQW;
        float v[kRows][8];
        uint4 ev[kRows];
#pragma unroll
        for (int rr = 0; rr < kRows; ++rr) {
          const int r = kRows * warp + rr;
          ev[rr] = make_uint4(0, 0, 0, 0);
          if (live(r)) {
            const int64_t tin = q_input_token(f, sm, r >> 1, p);
            ev[rr] = *reinterpret_cast<const uint4*>(f.emb_proj + (static_cast<int64_t>(p) * kVocab + tin) * kQD +
                                                     lane * 8);
          }
        }
        float p8[8];
        unpack8(*reinterpret_cast<const uint4*>(f.pos + static_cast<int64_t>(p + 1) * kQD + lane * 8), p8);
#pragma unroll
        for (int rr = 0; rr < kRows; ++rr) {
          const int r = kRows * warp + rr;
          uint4 row = make_uint4(0, 0, 0, 0);
          if (live(r)) {
            float e8[8], y[8];
            unpack8(ev[rr], e8);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = __fadd_rn(e8[e], p8[e]);
            row = pack8(y);
          }
          *reinterpret_cast<uint4*>(sm.xr.x + r * kQLdX + lane * 8) = row;
          unpack8(row, v[rr]);
        }
        q_layer_norm_rows(v, sm.u.a.xa, g1);
      }
      qbar();
      q_stamp(f, tracer, p, 15);
    }

    // ---- commit (owned sessions): tokens, counters, flags, next-frame embedding
    for (int i = threadIdx.x; i < n_own * kPositions; i += kQT) {
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
      f.invalid_rows[sid] = sm.inv[ls] | (qerr(sm) ? 4 : 0);
      if (f.eos_slot[sid] < 0) commit_end(f, sid, f.finished[sid] ? 0 : -1);
    }
    for (int i = threadIdx.x; i < n_own * (kEmbed / 8); i += kQT) {
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
    qbar();
    if (warp == 0) {
      tmem_fence_after_sync();
      tmem_dealloc(sm.tmem, 512);
    }
    if (tracer) f.trace[258] = static_cast<uint64_t>(clock64()), f.trace[259] = global_ns();
  }
  cg::this_cluster().sync();  // no CTA leaves while a peer may still push into it
}

template <int C>
int clusters_of() {
  static PerDeviceInt cache;  // the opt-in below is per device context
  return cache.get([] {
    int clusters = 0;
    if (cudaFuncSetAttribute(quad_frame_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(quad_smem_bytes<C>())) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = C;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(C);
      cfg.blockDim = dim3(kQThreads);
      cfg.dynamicSmemBytes = quad_smem_bytes<C>();
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&clusters, quad_frame_kernel<C>, &cfg) != cudaSuccess) clusters = 0;
    }
    cudaGetLastError();
    return clusters;
  });
}

bool shape_supported(const Frame& f) {
  return f.d == kQD && f.H == 4 && f.F == kQF && f.L == 1 && f.in_proj && (f.rp == 1 || f.rp == 2);
}

template <int C>
cudaError_t launch(const Frame& f, cudaStream_t stream) {
  QuadMaps maps;
  if (!make_weight_map(&maps.in_proj, f.in_w, kEmbed, kQD, kQBoxRows) ||
      !make_weight_map(&maps.qkv, f.qkv, kQD, 3 * kQD, kQBoxRows) ||
      !make_weight_map(&maps.o, f.o, kQD, kQD, kQBoxRows) || !make_weight_map(&maps.ffn1, f.w1, kQD, kQF, kQBoxRows) ||
      !make_weight_map(&maps.ffn2, f.w2, kQF, kQD, kQBoxRows) ||
      !make_weight_map(&maps.head, f.head_w, kQD, static_cast<uint64_t>(kPositions) * kVocab, kQBoxRows)) {
    return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaMemsetAsync(f.eos_count, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  const int tiles = (f.n + kQS - 1) / kQS;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(tiles * C);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = quad_smem_bytes<C>();
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, quad_frame_kernel<C>, f, maps);
  if (e != cudaSuccess) return e;
  return launch_frame_eos(f, stream);
}

}  // namespace

int quad_frame_clusters() { return clusters_of<4>(); }
bool quad_frame_supported(const Frame& f) { return shape_supported(f) && quad_frame_clusters() > 0; }
cudaError_t launch_quad_frame(const Frame& f, cudaStream_t stream) { return launch<4>(f, stream); }

int octo_frame_clusters() { return clusters_of<8>(); }
bool octo_frame_supported(const Frame& f) { return shape_supported(f) && octo_frame_clusters() > 0; }
cudaError_t launch_octo_frame(const Frame& f, cudaStream_t stream) { return launch<8>(f, stream); }

}  // namespace mtt
