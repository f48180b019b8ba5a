// Pair frame kernel: a 2-CTA thread-block cluster runs all 16 positions of a
// Local AR frame for up to 16 sessions (32 rows with CFG).  This is the
// throughput path for large batches: compared with one CTA per 8 sessions
// (frame_tile.cu) each SM streams half as many weight bytes per session, and
// every weight fragment it reads feeds two 16-row MMA tiles.
//
// Per position (reference ops as in frame_tile.cu), CTA c of the pair (c = 0, 1):
//   input rows: in-projection output features [128c, +128) (p = 0, or every p
//     without the folded tables) or x = bf16(emb_proj[p-1][token] + pos[p])
//     written by the sampling warps of both CTAs;             exchange R0 / R6
//   LN1 (all rows, both CTAs); q|k|v of heads 2c, 2c+1 only (no exchange);
//   k/v appended to this CTA's TMEM KV cache; attention for its two heads;
//     the two heads' outputs go to the peer;                  exchange R1
//   o-projection features [128c, +128) + residual;            exchange R2
//   LN2; FFN1 features [512c, +512) + GELU-tanh; FFN2 partial sums over
//     those 512 hidden features: the peer's output features go to the peer
//     (reduce-scatter, f32);                                  exchange R3
//   own output features = CTA 0's partial + CTA 1's partial, + residual;
//                                                             exchange R4
//   head p vocabulary [1012c, +1012) for all 16 sessions (bias, CFG, the
//     constraints): sessions 8c..8c+7 stay, the other eight sessions' values
//     and non-finite flags go to the peer;                    exchange R5
//   one warp per session samples sessions 8c..8c+7 and sends the peer the
//     token and the session's next input rows.                exchange R6
//
// Exchanges are pushes (st.async into the peer's shared memory, completing on
// the peer's round mbarrier, which the receiver arms with the bytes it
// expects); two barriers alternate by round parity.  A CTA can be at most one round ahead
// of its peer, so each round's pushes land in buffers the receiver does not
// touch during the phase before that round (x columns it does not own, the
// peer-attention buffer xr, the FFN2 receive buffer red, the value columns of
// the other vocabulary half).  Weights stream through a four-slot TMA ring
// (no multicast) filled by a producer warp.  GEMMs are mma.sync m16n8k16 with
// the 32-row A operand in registers, except the head: tcgen05.mma with 128
// vocabulary rows on M and the 32 tile rows on N, accumulating in TMEM
// columns of the KV cache that no position has written yet.  TMEM holds the
// KV cache of the CTA's two heads: lane 32q + t, quadrant q = (local head
// q/2, rows 16(q%2)..+16), t = 2 (row % 16) + half; columns as in the tile
// kernel.  Every wait is bounded; a timeout sets invalid bit 4 for the pair's
// sessions.
#include <cooperative_groups.h>
#include <cuda.h>

#include <mutex>

#include "frame_common.cuh"
#include "ptx.cuh"
#include "tile_common.cuh"

namespace cg = cooperative_groups;

namespace mtt {
namespace {

constexpr int kPR = 32;                      // rows per pair
constexpr int kPS = 16;                      // session slots per pair
constexpr int kPOwn = 8;                     // slots each CTA samples
constexpr int kPW = 8;                       // consumer warps
constexpr int kPC = kPW * 32;                // consumer threads
constexpr int kPThreads = kPC + 128;         // + the control warpgroup (TMA producer, head MMA thread)
constexpr int kPProducerRegs = 56;   // the producer and head MMA threads
constexpr int kPConsumerRegs = 224;
static_assert(128 * kPProducerRegs + kPC * kPConsumerRegs <= kPThreads * 168, "register split");
constexpr int kD = 256;
constexpr int kF = 1024;
constexpr int kHeads = 4;
constexpr int kCRows = 64;
constexpr int kCK = 256;
constexpr int kCPanel = 64;
constexpr int kCElems = kCRows * kCK;
constexpr uint32_t kCBytes = kCElems * 2;
constexpr int kPSlots = 4;
constexpr int kHeadRows = 128;  // head chunks: 128 vocabulary rows x 128 K columns (tcgen05 M = 128)
constexpr int kLdX = kD + 8;    // 264
constexpr int kLdR = 128 + 8;   // 136: the peer's two heads
constexpr int kLdQ = 384 + 8;   // 392: this CTA's q | k | v
constexpr int kLdH = 512 + 8;   // 520: this CTA's half of the FFN hidden
constexpr int kHalf = kVocab / 2;  // 1012
constexpr int kTmemCols = 512;
constexpr int kListBytes = (2 * kListCap + 8) * 2;  // candidate (+ scratch entry) + eligible lists
static_assert(kPOwn * kListBytes <= kPR * kLdX * 2, "sampler lists in xa");

struct PairMaps {
  CUtensorMap in_proj, qkv, o, ffn1, ffn2, head;
};

struct PairAttn {
  float s[2][4][32][8];
  float o[4][32][32];
};

union PairU {
  bf16 src[kPR * kLdX];            // one 256-column block of the in-projection input
  bf16 qkv[kPR * kLdQ];            // this CTA's heads: q | k | v
  PairAttn att;                    // after q/k/v are consumed
  bf16 hid[kPR * kLdH];            // this CTA's half of the FFN hidden
  uint16_t val[kPOwn * kVocab];    // constrained logits of the sessions this CTA samples
};

struct __align__(1024) PairSmem {
  bf16 ring[kPSlots][kCElems];
  bf16 xa[kPR * kLdX];  // LN output / this CTA's attention heads / the head's B operand / sampler lists
  bf16 x[kPR * kLdX];   // residual stream (all rows, all features)
  bf16 xr[kPR * kLdR];  // the peer's attention heads
  PairU u;
  float red[kPR][128];  // the peer's FFN2 partial sums of this CTA's output features
  __align__(16) bf16 hb[1016];  // this CTA's half of head p's bias
  int32_t tok[kPS][kPositions];
  int32_t sess[kPS];
  uint32_t flags[kPS];  // bit 0 unfinished, bit 1 finished, bit 2 forbid_eos
  int64_t ctr[kPOwn];
  int64_t seed[kPOwn];
  int32_t inv[kPOwn];
  uint32_t nonfinite[kPOwn];        // this CTA's half, own sessions
  uint32_t stage_nonfinite[kPOwn];  // this CTA's half, the peer's sessions, before sending
  uint32_t peer_nonfinite[kPOwn];   // the peer's half, own sessions (sent by the peer)
  int32_t last_issued[kPSlots];
  int32_t n_sess;
  int32_t err;
  uint32_t tmem;
  unsigned long long full[kPSlots];
  unsigned long long empty[kPSlots];
  unsigned long long xbar[2];
  unsigned long long hbar[2];   // head accumulator buffer b holds a finished M-block (tcgen05.commit)
  unsigned long long hfree[2];  // every consumer warp has read head buffer b
  unsigned long long hop;       // the head's B operand of this position is in xa
  unsigned long long hfin;      // every head MMA has completed (teardown)
  int32_t mma_done;
  uint32_t sink;  // round token (never read)
};
// xa follows the ring at a 1024-byte boundary: the head reads it as a
// swizzled tcgen05 operand (8-row, 1024-byte swizzle atoms).
static_assert((kPSlots * kCElems * 2) % 1024 == 0 && kPR * 64 * 2 * 4 <= kPR * kLdX * 2, "head operand in xa");
constexpr size_t kPSmemBytes = sizeof(PairSmem) + 1024;
static_assert(kPSmemBytes <= 232448, "pair kernel shared memory");

__device__ __forceinline__ int err_flag(const PairSmem& sm) { return *reinterpret_cast<const volatile int*>(&sm.err); }
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Phase clock stamp of the first CTA (library trace hook: mtt_b200_test_frame_trace).
__device__ __forceinline__ void p_stamp(const Frame& f, bool tracer, int p, int i) {
  if (tracer) f.trace[kPositions * p + i] = static_cast<uint64_t>(clock64());
}

// ---------------------------------------------------------------------------
// weight stream
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool has_in_projection(bool folded, int p) { return p == 0 || !folded; }

__device__ __forceinline__ int chunks_in_position(bool folded, int p) {
  return (has_in_projection(folded, p) ? 6 : 0) + 6 + 2 + 8 + 8 + 16;
}

// Chunk k of position p for CTA c: tensor map and box origin (x = K column, y = row).
__device__ __forceinline__ const CUtensorMap* chunk_origin(const PairMaps& m, int c, bool folded, int p, int k, int* x,
                                                           int* y) {
  if (has_in_projection(folded, p)) {
    if (k < 6) {  // (kb, nb): K block kb of 768, features [128c + 64 nb, +64)
      *x = kCK * (k / 2);
      *y = 128 * c + kCRows * (k % 2);
      return &m.in_proj;
    }
    k -= 6;
  }
  *x = 0;
  if (k < 6) {  // q, k, v rows of heads 2c, 2c+1
    *y = kD * (k >> 1) + 128 * c + kCRows * (k & 1);
    return &m.qkv;
  }
  k -= 6;
  if (k < 2) {
    *y = 128 * c + kCRows * k;
    return &m.o;
  }
  k -= 2;
  if (k < 8) {
    *y = 512 * c + kCRows * k;
    return &m.ffn1;
  }
  k -= 8;
  if (k < 8) {  // (kb, nb): hidden features [512c + 256 kb, +256), outputs [64 nb, +64)
    *x = 512 * c + kCK * (k / 4);
    *y = kCRows * (k % 4);
    return &m.ffn2;
  }
  k -= 8;
  // head: M-block k / 2 (vocabulary rows [128 (k / 2), +128) of this CTA's
  // half; rows past the half are ignored), K columns [128 (k % 2), +128)
  *x = 128 * (k & 1);
  *y = p * kVocab + kHalf * c + 128 * (k >> 1);
  return &m.head;
}

__device__ void producer(PairSmem& sm, const PairMaps& maps, int c, bool folded) {
  int it = 0;
  for (int p = 0; p < kPositions; ++p) {
    const int n = chunks_in_position(folded, p);
    for (int k = 0; k < n; ++k, ++it) {
      const int slot = it % kPSlots;
      if (it >= kPSlots && !mbar_wait(&sm.empty[slot], ((it / kPSlots) - 1) & 1)) sm.err = 1;
      if (err_flag(sm)) return;
      int x, y;
      const CUtensorMap* map = chunk_origin(maps, c, folded, p, k, &x, &y);
      fence_proxy_async();
      mbar_expect_tx(&sm.full[slot], kCBytes);
      if (map == &maps.head) {  // two 128-row x 64-column panels
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          tma_load_2d(sm.ring[slot] + b * (kHeadRows * kCPanel), map, x + b * kCPanel, y, &sm.full[slot]);
        }
      } else {  // four 64-row x 64-column panels
#pragma unroll
        for (int b = 0; b < kCK / kCPanel; ++b) {
          tma_load_2d(sm.ring[slot] + b * (kCRows * kCPanel), map, x + b * kCPanel, y, &sm.full[slot]);
        }
      }
      sm.last_issued[slot] = it;
    }
  }
}

__device__ __forceinline__ const bf16* acquire(PairSmem& sm, int it) {
  const int slot = it % kPSlots;
  if (err_flag(sm) == 0 && !mbar_wait(&sm.full[slot], (it / kPSlots) & 1)) sm.err = 1;
  return sm.ring[slot];
}

__device__ __forceinline__ void release(PairSmem& sm, int it) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.empty[it % kPSlots]);
}

// ---------------------------------------------------------------------------
// 32-row GEMM pieces: A = two 16-row m-tiles in registers
// ---------------------------------------------------------------------------

__device__ __forceinline__ void load_a2(uint32_t (&a)[2][16][4], const bf16* A, int lda) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const bf16* p = A + (16 * m + (lane & 7) + 8 * ((lane >> 3) & 1)) * lda + 8 * (lane >> 4);
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) ldsm_x4(a[m][ks], p + 16 * ks);
  }
}

// A of the o-projection: dims [128c, +128) from xa, the other half from xr.
__device__ __forceinline__ void load_a2_attn(uint32_t (&a)[2][16][4], const bf16* xa, const bf16* xr, int c) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const int row = 16 * m + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      const bf16* p = ((ks >> 3) == c) ? xa + row * kLdX + 16 * ks : xr + row * kLdR + 16 * (ks & 7);
      ldsm_x4(a[m][ks], p + 8 * (lane >> 4));
    }
  }
}

template <int CH>
__device__ __forceinline__ void mma_chunk2(float (&cc)[2][CH][4], const uint32_t (&a)[2][16][4], const bf16* chunk) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = 8 * warp + (lane & 7);
  const int q = lane >> 3;
  const bf16* row = chunk + n * kCPanel;
  const int swz = n & 7;
#pragma unroll
  for (int ks2 = 0; ks2 < 8; ++ks2) {
    uint32_t b[4];
    ldsm_x4(b, row + (ks2 >> 1) * (kCRows * kCPanel) + (((4 * (ks2 & 1) + q) ^ swz) << 3));
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      mma16816(cc[m][(2 * ks2) % CH], a[m][2 * ks2], b[0], b[1]);
      mma16816(cc[m][(2 * ks2 + 1) % CH], a[m][2 * ks2 + 1], b[2], b[3]);
    }
  }
}

// C[32][64 nb_count] = A W^T; epi(nb, acc[m][e]) per chunk.  (Running the
// epilogue one chunk behind, as the 16-row kernels do, costs spills at 32 rows.)
template <typename Epi>
__device__ __forceinline__ void gemm_n2(PairSmem& sm, int& it, const uint32_t (&a)[2][16][4], int nb_count, Epi epi) {
  for (int nb = 0; nb < nb_count; ++nb, ++it) {
    const bf16* chunk = acquire(sm, it);
    float cur[2][2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int j = 0; j < 2; ++j) cur[m][j][0] = cur[m][j][1] = cur[m][j][2] = cur[m][j][3] = 0.f;
    mma_chunk2<2>(cur, a, chunk);
    release(sm, it);
    float acc[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][e] = cur[m][0][e] + cur[m][1][e];
    epi(nb, acc);
  }
}

// ---------------------------------------------------------------------------
// head on tcgen05: D[vocabulary row m][tile row n] in TMEM lane m, with the
// accumulators in key/value columns no position has written yet.  Position j
// keeps its keys in columns 16 tmem_block(j) + [0, 16) and its values 256
// higher; blocks 14 and 15 (positions 13 and 15) are adjacent.  Positions
// 0..12, and 15 once its attention has read the cache: two N = 32 buffers,
// columns [224, 256) and [480, 512).  Position 13: the key / value blocks of
// positions 15 (buffer 0) and 14 (buffer 1), each buffer two N = 16 halves
// (tile rows 0..15 in the key block, 16..31 in the value block).  Position
// 14: position 15's blocks, one buffer.
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool head_wide(int p) { return p <= 12 || p == 15; }
__device__ __forceinline__ int head_nbuf(int p) { return p == 14 ? 1 : 2; }
// Columns of buffer b: tile rows 0..15 from ca, rows 16..31 from cb.
__device__ __forceinline__ void head_cols(int p, int b, uint32_t& ca, uint32_t& cb) {
  if (head_wide(p)) {
    ca = b ? 480u : 224u;
    cb = ca + 16u;
  } else {
    ca = 16u * static_cast<uint32_t>(tmem_block(b ? 14 : 15));
    cb = ca + 256u;
  }
}

// The head MMA thread: the MMAs of head M-block mb (chunks it0 + 2 mb: K 0..127 and
// it0 + 2 mb + 1: K 128..255) into buffer b, then a commit to hbar[b], also
// after an error (the waiting warps always see the phase complete).
__device__ __forceinline__ void issue_head_block(PairSmem& sm, int it0, int mb, int p, int b) {
  const bf16* c0 = acquire(sm, it0 + 2 * mb);
  const bf16* c1 = acquire(sm, it0 + 2 * mb + 1);
  if (err_flag(sm) == 0) {
    tmem_fence_after_sync();
    uint32_t ca, cb;
    head_cols(p, b, ca, cb);
    const uint32_t da = sm.tmem + ca, db = sm.tmem + cb;
    const uint64_t a0 = umma_desc_sw128(c0), a1 = umma_desc_sw128(c1), b0 = umma_desc_sw128(sm.xa);
    constexpr uint64_t kPanelStep = kHeadRows * kCPanel * 2 / 16;  // 128-row weight panel
    constexpr uint64_t kOpStep = kPR * kCPanel * 2 / 16;           // 32-row operand panel
    constexpr uint64_t kHalfRows = 16 * 128 / 16;                  // operand rows 16..31
    // straight-line bursts (a branch between tcgen05.mma instructions slows their issue)
    if (head_wide(p)) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, 32);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        umma_bf16(da, a0 + (kk >> 2) * kPanelStep + 2 * (kk & 3), b0 + (kk >> 2) * kOpStep + 2 * (kk & 3), idesc,
                  kk != 0);
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        umma_bf16(da, a1 + (kk >> 2) * kPanelStep + 2 * (kk & 3), b0 + (2 + (kk >> 2)) * kOpStep + 2 * (kk & 3),
                  idesc, true);
      }
    } else {
      // positions 13 and 14 only: a rolled loop keeps this thread within its registers
      constexpr uint32_t idesc = umma_idesc_bf16(128, 16);
#pragma unroll 1
      for (int kk = 0; kk < 16; ++kk) {
        const uint64_t a = ((kk >> 3) ? a1 : a0) + ((kk >> 2) & 1) * kPanelStep + 2 * (kk & 3);
        const uint64_t bd = b0 + (kk >> 2) * kOpStep + 2 * (kk & 3);
        umma_bf16(da, a, bd, idesc, kk != 0);
        umma_bf16(db, a, bd + kHalfRows, idesc, kk != 0);
      }
    }
  }
  umma_commit(&sm.hbar[b]);
}

// Two 8-column loads (lanes of this warp's quadrant) and one wait.
__device__ __forceinline__ void tmem_ld8x2(uint32_t (&v)[16], uint32_t ta, uint32_t tb) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(ta)
               : "memory");
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
               : "r"(tb)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

// The head MMA thread (one lane of the control warpgroup): per position,
// once the consumers have put the B operand in xa, the eight M-blocks
// alternate over the position's buffers; a buffer is reused after every
// consumer warp has read it.  Waits are skipped after an error (all bounded).
__device__ void head_mma(PairSmem& sm, bool folded) {
  int it = 0, u0 = 0, u1 = 0;  // chunks before this position, uses of buffers 0 and 1
  for (int p = 0; p < kPositions; ++p) {
    const int n = chunks_in_position(folded, p);
    const int it0 = it + n - 2 * 8;  // the head's 16 chunks end the position
    it += n;
    if (err_flag(sm) == 0 && !mbar_wait_cta(&sm.hop, p & 1)) sm.err = 1;
    const int nb = head_nbuf(p);
    for (int mb = 0; mb < 8; ++mb) {
      const int b = nb == 2 ? (mb & 1) : 0;
      const int u = b ? u1 : u0;
      if (u >= 1 && err_flag(sm) == 0 && !mbar_wait_cta(&sm.hfree[b], (u - 1) & 1)) sm.err = 1;
      if (b) {
        ++u1;
      } else {
        ++u0;
      }
      issue_head_block(sm, it0, mb, p, b);
    }
  }
  umma_commit(&sm.hfin);
  mbar_wait_cta(&sm.hfin, 0);
  atomicExch(&sm.mma_done, 1);
}

__device__ __forceinline__ void layer_norm_rows32(const bf16* x, bf16* xa, const float (&g)[8]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    const int r = 4 * warp + rr;
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
    *reinterpret_cast<uint4*>(xa + r * kLdX + lane * 8) = pack8(out);
  }
}

// ---------------------------------------------------------------------------
// exchange rounds (two CTAs)
// ---------------------------------------------------------------------------

struct Round {
  uint32_t r = 0;
  __device__ __forceinline__ int bar() const { return static_cast<int>(r & 1u); }
  __device__ __forceinline__ uint32_t parity() const { return (r >> 1) & 1u; }
};

__device__ __forceinline__ uint32_t peer_bar(const PairSmem& sm, const Round& rd, int peer) {
  return cluster_addr(&sm.xbar[rd.bar()], peer);
}

// Wait for this CTA's round: it arms its own round barrier with the bytes
// the peer pushes to it in this round, and the round completes when they
// have landed.  The peer pushes something in every round (a 4-byte token in
// the token round), so a completed round also shows the peer finished the
// phase before it.
__device__ __forceinline__ void finish_round(PairSmem& sm, Round& rd, uint32_t bytes_in) {
  cbar();
  if (threadIdx.x == 0) mbar_expect_tx(&sm.xbar[rd.bar()], bytes_in);
  if (err_flag(sm) == 0 && !mbar_wait(&sm.xbar[rd.bar()], rd.parity())) sm.err = 1;
  ++rd.r;
}

__device__ __forceinline__ void push_b32(const void* local_addr_in_peer_layout, int peer, uint32_t v, uint32_t bar) {
  st_async_b32(cluster_addr(local_addr_in_peer_layout, peer), v, bar);
}

// ---------------------------------------------------------------------------
// attention: warp w -> quadrant q = w % 4 (local head q / 2, rows 16 (q % 2)..),
// part = w / 4 (positions of parity part); thread t: row 16 (q % 2) + t / 2,
// dims [32 (t % 2), +32) of the head
// ---------------------------------------------------------------------------

__device__ __forceinline__ void attention_pair(PairSmem& sm, int p, int c, int peer, uint32_t rbar) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = warp & 3, part = warp >> 2;
  const int hl = q >> 1;
  const int row = 16 * (q & 1) + (lane >> 1), half = lane & 1;
  const uint32_t tl = sm.tmem + (static_cast<uint32_t>(32 * q) << 16);
  const bf16* qrow = sm.u.qkv + row * kLdQ + kHeadDim * hl + 32 * half;
  {  // append k (part 0) or v (part 1) of position p (its columns may have held a head accumulator)
    tmem_fence_after_sync();
    uint32_t kv[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 t = *reinterpret_cast<const uint4*>(qrow + 128 * (1 + part) + 8 * j);
      kv[4 * j] = t.x;
      kv[4 * j + 1] = t.y;
      kv[4 * j + 2] = t.z;
      kv[4 * j + 3] = t.w;
    }
    tmem_st16(tl + 256 * part + 16 * tmem_block(p), kv);
    tmem_wait_st();
  }
  float qv[32];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float f8[8];
    unpack8(*reinterpret_cast<const uint4*>(qrow + 8 * j), f8);
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[8 * j + e] = f8[e];
  }
  tmem_fence_before_sync();
  cbar();
  tmem_fence_after_sync();
  float s[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) s[m] = -CUDART_INF_F;
#pragma unroll
  for (int g4 = 0; g4 < 2; ++g4) {
    if (8 * g4 + part <= p) {
      uint32_t k[64];
      tmem_ld64(k, tl + 16 * (8 * part + 4 * g4));
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&k[16 * jj + e]));
          dot = fmaf(qv[2 * e], t.x, dot);
          dot = fmaf(qv[2 * e + 1], t.y, dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        if (2 * (4 * g4 + jj) + part <= p) s[4 * g4 + jj] = round_bf16(__fmul_rn(round_bf16(dot), 0.125f));
      }
    }
  }
  float* my_s = sm.u.att.s[part][q][lane];
#pragma unroll
  for (int m = 0; m < 8; ++m) my_s[m] = s[m];
  cbar();
  float all[kPositions];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    all[2 * m] = sm.u.att.s[0][q][lane][m];
    all[2 * m + 1] = sm.u.att.s[1][q][lane][m];
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
  float o[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) o[d] = 0.f;
#pragma unroll
  for (int g4 = 0; g4 < 2; ++g4) {
    if (8 * g4 + part <= p) {
      uint32_t v[64];
      tmem_ld64(v, tl + 256 + 16 * (8 * part + 4 * g4));
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
    float* dst = sm.u.att.o[q][lane];
#pragma unroll
    for (int d = 0; d < 32; ++d) dst[d] = o[d];
  }
  cbar();
  if (part == 0) {
    const float* src = sm.u.att.o[q][lane];
#pragma unroll
    for (int d = 0; d < 32; ++d) o[d] += src[d];
    bf16* out = sm.xa + row * kLdX + kHeadDim * (2 * c + hl) + 32 * half;
    const bf16* remote = sm.xr + row * kLdR + kHeadDim * hl + 32 * half;  // same place in the peer
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float f8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f8[e] = o[8 * j + e];
      const uint4 u = pack8(f8);
      *reinterpret_cast<uint4*>(out + 8 * j) = u;
      st_async_v4(cluster_addr(remote + 8 * j, peer), u, rbar);
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

__device__ __forceinline__ int64_t clamp_token(int64_t t) { return t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t); }

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    pair_frame_kernel(Frame f, const __grid_constant__ PairMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
  PairSmem& sm = *reinterpret_cast<PairSmem*>(smem_raw + pad);
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int peer = c ^ 1;
  const int pair = static_cast<int>(blockIdx.x) / 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rp = f.rp;
  const bool folded = f.emb_proj != nullptr;

  // ---- sessions [16 pair, +16) of the active list (both CTAs find the same)
  if (warp == 0) {
    int seen = 0;
    const int first = kPS * pair;
    for (int base = 0; base < f.n; base += 32) {
      const int s = base + lane;
      const bool act = s < f.n && (f.active == nullptr || f.active[s]);
      const unsigned m = __ballot_sync(0xffffffffu, act);
      const int rank = seen + __popc(m & ((1u << lane) - 1u));
      if (act && rank >= first && rank < first + kPS) sm.sess[rank - first] = s;
      seen += __popc(m);
    }
    if (lane == 0) {
      const int left = seen - first;
      sm.n_sess = left <= 0 ? 0 : (left < kPS ? left : kPS);
      sm.err = 0;
      sm.mma_done = 0;
    }
  }
  __syncthreads();
  const int n_sess = sm.n_sess;
  if (n_sess == 0) return;  // same in both CTAs: neither touches the other
  const int own0 = kPOwn * c;
  const int n_own = n_sess - own0 <= 0 ? 0 : (n_sess - own0 < kPOwn ? n_sess - own0 : kPOwn);
  const int n_peer = n_sess - kPOwn * peer <= 0 ? 0 : (n_sess - kPOwn * peer < kPOwn ? n_sess - kPOwn * peer : kPOwn);
  auto live = [&](int r) { return (r & 15) < n_sess && (r >> 4) < rp; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kPW);
      sm.last_issued[s] = -1;
    }
    mbar_init(&sm.xbar[0], 1);
    mbar_init(&sm.xbar[1], 1);
    mbar_init(&sm.hbar[0], 1);
    mbar_init(&sm.hbar[1], 1);
    mbar_init(&sm.hfree[0], kPW);
    mbar_init(&sm.hfree[1], kPW);
    mbar_init(&sm.hop, 1);
    mbar_init(&sm.hfin, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(&sm.tmem, kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x < n_sess) {
    const int sid = sm.sess[threadIdx.x];
    sm.flags[threadIdx.x] = (f.unfinished[sid] ? 1u : 0u) | (f.finished[sid] ? 2u : 0u) | (f.forbid[sid] ? 4u : 0u);
  }
  if (threadIdx.x < n_own) {  // per-session state and EOS registration of the sessions this CTA samples
    const int s = threadIdx.x;
    const int sid = sm.sess[own0 + s];
    sm.ctr[s] = f.counter_io[sid];
    sm.seed[s] = f.seed[sid];
    int32_t inv = 0;
    bool en = !f.unfinished[sid] && !f.finished[sid] && !f.forbid[sid];
    if (en && f.final_w == nullptr) {
      inv = 2;
      en = false;
    }
    sm.inv[s] = inv;
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
  cluster.sync();  // both CTAs' barriers are initialised before any push

  if (warp >= kPW) {  // control warpgroup: the TMA producer and the head MMA thread
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPProducerRegs));
    if (warp == kPW && lane == 0) producer(sm, maps, c, folded);
    if (warp == kPW + 1 && lane == 0) head_mma(sm, folded);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPConsumerRegs));
    float g1[8], g2[8];
    unpack8(*reinterpret_cast<const uint4*>(f.ln1 + lane * 8), g1);
    unpack8(*reinterpret_cast<const uint4*>(f.ln2 + lane * 8), g2);
    Round rd;
    int it = 0;
    const bool tracer = f.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
    if (tracer) f.trace[256] = static_cast<uint64_t>(clock64()), f.trace[257] = global_ns();
    for (int p = 0; p < kPositions; ++p) {
      // ---------------- input rows
      p_stamp(f, tracer, p, 0);
      if (has_in_projection(folded, p)) {
        float acc[2][2][2][4];  // nb, m-tile, chain
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int j = 0; j < 2; ++j) acc[nb][m][j][0] = acc[nb][m][j][1] = acc[nb][m][j][2] = acc[nb][m][j][3] = 0.f;
        for (int kb = 0; kb < 3; ++kb) {
          cbar();  // the previous block's A fragments are loaded
          for (int i = threadIdx.x; i < kPR * (kCK / 8); i += kPC) {
            const int r = i / (kCK / 8), ch = i % (kCK / 8);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (live(r)) {
              const int slot = r & 15, sub = r >> 4;
              const bf16* src;
              if (p == 0) {
                src = f.hidden + (static_cast<int64_t>(sm.sess[slot]) * rp + sub) * kEmbed;
              } else {
                const int64_t t = f.forced ? clamp_token(f.forced[static_cast<int64_t>(sm.sess[slot]) * kPositions + p - 1])
                                           : static_cast<int64_t>(sm.tok[slot][p - 1]);
                src = f.emb + (static_cast<int64_t>(p - 1) * kVocab + t) * kEmbed;
              }
              v = *reinterpret_cast<const uint4*>(src + kCK * kb + ch * 8);
            }
            *reinterpret_cast<uint4*>(sm.u.src + r * kLdX + ch * 8) = v;
          }
          cbar();
          uint32_t a[2][16][4];
          load_a2(a, sm.u.src, kLdX);
#pragma unroll
          for (int nb = 0; nb < 2; ++nb, ++it) {
            const bf16* chunk = acquire(sm, it);
            mma_chunk2<2>(acc[nb], a, chunk);
            release(sm, it);
          }
        }
        const bf16* pos = f.pos + static_cast<int64_t>(p) * kD;
        const uint32_t rb = peer_bar(sm, rd, peer);
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          const int n = 128 * c + kCRows * nb + 8 * warp + 2 * (lane & 3);
          const float b0 = bf2f(f.in_b[n]), b1 = bf2f(f.in_b[n + 1]);
          const float q0 = bf2f(pos[n]), q1 = bf2f(pos[n + 1]);
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int r = 16 * m + (lane >> 2) + 8 * hh;
              const float y0 = round_bf16(__fadd_rn(acc[nb][m][0][2 * hh] + acc[nb][m][1][2 * hh], b0));
              const float y1 = round_bf16(__fadd_rn(acc[nb][m][0][2 * hh + 1] + acc[nb][m][1][2 * hh + 1], b1));
              const uint32_t v = pack_bf16x2(__fadd_rn(y0, q0), __fadd_rn(y1, q1));
              bf16* xr_ = sm.x + r * kLdX + n;
              *reinterpret_cast<uint32_t*>(xr_) = v;
              push_b32(xr_, peer, v, rb);
            }
        }
        finish_round(sm, rd, kPR * 128 * 2);  // R0
      }
      // head p bias (this CTA's half), per-position sampling state
      {
        const bf16* hb = f.head_b + static_cast<int64_t>(p) * kVocab + kHalf * c;
        if (threadIdx.x < kHalf / 4) {
          *reinterpret_cast<uint2*>(sm.hb + 4 * threadIdx.x) = *reinterpret_cast<const uint2*>(hb + 4 * threadIdx.x);
        }
        if (threadIdx.x < kPOwn) {
          sm.nonfinite[threadIdx.x] = 0;
          sm.stage_nonfinite[threadIdx.x] = 0;
        }
      }
      // ---------------- LN1, q|k|v of this CTA's heads
      layer_norm_rows32(sm.x, sm.xa, g1);
      cbar();
      p_stamp(f, tracer, p, 1);
      {
        uint32_t a[2][16][4];
        load_a2(a, sm.xa, kLdX);
        gemm_n2(sm, it, a, 6, [&](int nb, const float (&acc)[2][4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int r = 16 * m + (lane >> 2) + 8 * hh;
              *reinterpret_cast<uint32_t*>(sm.u.qkv + r * kLdQ + n) = pack_bf16x2(acc[m][2 * hh], acc[m][2 * hh + 1]);
            }
        });
      }
      cbar();
      p_stamp(f, tracer, p, 2);
      // ---------------- attention of heads 2c, 2c+1; outputs to the peer
      attention_pair(sm, p, c, peer, peer_bar(sm, rd, peer));
      p_stamp(f, tracer, p, 3);
      finish_round(sm, rd, kPR * 128 * 2);  // R1
      p_stamp(f, tracer, p, 4);
      // ---------------- o-projection features [128c, +128) + residual
      {
        uint32_t a[2][16][4];
        load_a2_attn(a, sm.xa, sm.xr, c);
        const uint32_t rb = peer_bar(sm, rd, peer);
        gemm_n2(sm, it, a, 2, [&](int nb, const float (&acc)[2][4]) {
          const int n = 128 * c + kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              bf16* xr_ = sm.x + (16 * m + (lane >> 2) + 8 * hh) * kLdX + n;
              const uint32_t v = pack_bf16x2(__fadd_rn(bf2f(xr_[0]), round_bf16(acc[m][2 * hh])),
                                             __fadd_rn(bf2f(xr_[1]), round_bf16(acc[m][2 * hh + 1])));
              *reinterpret_cast<uint32_t*>(xr_) = v;
              push_b32(xr_, peer, v, rb);
            }
        });
      }
      finish_round(sm, rd, kPR * 128 * 2);  // R2
      p_stamp(f, tracer, p, 5);
      // ---------------- LN2, FFN1 features [512c, +512) + GELU
      layer_norm_rows32(sm.x, sm.xa, g2);
      cbar();
      p_stamp(f, tracer, p, 6);
      {
        uint32_t a[2][16][4];
        load_a2(a, sm.xa, kLdX);
        gemm_n2(sm, it, a, 8, [&](int nb, const float (&acc)[2][4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int r = 16 * m + (lane >> 2) + 8 * hh;
              *reinterpret_cast<uint32_t*>(sm.u.hid + r * kLdH + n) =
                  pack_bf16x2(gelu_tanh(round_bf16(acc[m][2 * hh])), gelu_tanh(round_bf16(acc[m][2 * hh + 1])));
            }
        });
      }
      cbar();
      p_stamp(f, tracer, p, 7);
      // ---------------- FFN2 partial sums over this CTA's 512 hidden features
      float own[2][2][4];  // this CTA's output features (nb = 2c, 2c+1), m-tile
      {
        float acc[4][2][1][4];
#pragma unroll
        for (int nb = 0; nb < 4; ++nb)
#pragma unroll
          for (int m = 0; m < 2; ++m) acc[nb][m][0][0] = acc[nb][m][0][1] = acc[nb][m][0][2] = acc[nb][m][0][3] = 0.f;
        for (int kb = 0; kb < 2; ++kb) {
          uint32_t a[2][16][4];
          load_a2(a, sm.u.hid + kCK * kb, kLdH);
#pragma unroll
          for (int nb = 0; nb < 4; ++nb, ++it) {
            const bf16* chunk = acquire(sm, it);
            mma_chunk2<1>(acc[nb], a, chunk);
            release(sm, it);
          }
        }
        const uint32_t rb = peer_bar(sm, rd, peer);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = kCRows * j + 8 * warp + 2 * (lane & 3);  // within the 128 features of a CTA
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            // this CTA's blocks are nb = 2c + j, the peer's 2 peer + j: select between
            // compile-time indices (a runtime index would put acc in local memory)
            float mine[4], theirs[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              mine[e] = c ? acc[2 + j][m][0][e] : acc[j][m][0][e];
              theirs[e] = c ? acc[j][m][0][e] : acc[2 + j][m][0][e];
              own[j][m][e] = mine[e];
            }
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int r = 16 * m + (lane >> 2) + 8 * hh;
              st_async_v2f(cluster_addr(&sm.red[r][col], peer), theirs[2 * hh], theirs[2 * hh + 1], rb);
            }
          }
        }
      }
      p_stamp(f, tracer, p, 8);
      finish_round(sm, rd, kPR * 128 * 4);  // R3
      p_stamp(f, tracer, p, 9);
      // ---------------- own output features: CTA 0's partial + CTA 1's partial, + residual
      {
        const uint32_t rb = peer_bar(sm, rd, peer);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = kCRows * j + 8 * warp + 2 * (lane & 3);
          const int n = 128 * c + col;
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int r = 16 * m + (lane >> 2) + 8 * hh;
              const float2 rv = *reinterpret_cast<const float2*>(&sm.red[r][col]);
              const float s0 = c == 0 ? own[j][m][2 * hh] + rv.x : rv.x + own[j][m][2 * hh];
              const float s1 = c == 0 ? own[j][m][2 * hh + 1] + rv.y : rv.y + own[j][m][2 * hh + 1];
              bf16* xr_ = sm.x + r * kLdX + n;
              const uint32_t v = pack_bf16x2(__fadd_rn(bf2f(xr_[0]), round_bf16(s0)), __fadd_rn(bf2f(xr_[1]), round_bf16(s1)));
              *reinterpret_cast<uint32_t*>(xr_) = v;
              push_b32(xr_, peer, v, rb);
            }
        }
      }
      finish_round(sm, rd, kPR * 128 * 2);  // R4
      p_stamp(f, tracer, p, 10);
      // ---------------- head p, this CTA's vocabulary half, all 16 sessions
      // (tcgen05: M = 128 vocabulary rows, N = the 32 tile rows, K = 256; one
      // thread of the control warpgroup issues, buffer b's M-block lands on hbar[b])
      {
        // B operand: x as four 32-row x 64-column panels with the 128-byte swizzle
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int q = threadIdx.x + kPC * i;  // 16-byte unit: row q / 32, columns [8 (q % 32), +8)
          const int r = q >> 5, kc = q & 31;
          const uint4 u = *reinterpret_cast<const uint4*>(sm.x + r * kLdX + 8 * kc);
          *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(sm.xa) + (kc >> 3) * (kPR * 128) + r * 128 +
                                    (((kc & 7) ^ (r & 7)) << 4)) = u;
        }
        fence_proxy_async();
        tmem_fence_before_sync();  // the attention's key/value reads come before the MMAs' writes
        cbar();
        if (threadIdx.x == 0) mbar_arrive(&sm.hop);
        const int nbuf = head_nbuf(p);
        // this warp: vocabulary entries [32 (warp % 4), +32) of each M-block,
        // slots 8 g..8 g + 7 (sampled by CTA g); after the lane-pair exchange
        // an even lane holds entries (j, j + 1) of slots 8 g + 0..3, an odd
        // lane entries (j - 1, j) of slots 8 g + 4..7
        const int g = warp >> 2;
        const bool local = g == c, odd = lane & 1;
        const int s0 = 8 * g + 4 * (lane & 1);
        const uint32_t rb = peer_bar(sm, rd, peer);
        const bool cfg = rp == 2;
        const float cfg_scale = f.prm.cfg_scale, uncond_scale = __fsub_rn(1.0f, f.prm.cfg_scale);
        uint32_t fl[4];
        bool live_s[4], nf[4];
        bf16* lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int s = s0 + i;
          fl[i] = sm.flags[s];
          live_s[i] = s < n_sess;
          nf[i] = false;
          lo[i] = (f.logits_out && live_s[i])
                      ? f.logits_out + (static_cast<int64_t>(sm.sess[s]) * kPositions + p) * rp * kVocab : nullptr;
        }
        const uint32_t tl = sm.tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        uint32_t hph = 0;  // bit b: parity of buffer b's next phase
#pragma unroll 1
        for (int mb = 0; mb < 8; ++mb) {
          const int b = nbuf == 2 ? (mb & 1) : 0;
          if (err_flag(sm) == 0 && !mbar_wait_cta(&sm.hbar[b], (hph >> b) & 1u)) sm.err = 1;
          hph ^= 1u << b;
          tmem_fence_after_sync();
          uint32_t ca, cb;
          head_cols(p, b, ca, cb);
          uint32_t v[16];  // v[i]: slot 8 g + i conditional row, v[8 + i]: unconditional
          tmem_ld8x2(v, tl + ca + 8 * g, tl + cb + 8 * g);
          release(sm, it);
          release(sm, it + 1);
          it += 2;
          tmem_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.hfree[b]);  // this warp has read buffer b
          float cv[4][2], uv[4][2];  // [local slot][entry j & ~1, j | 1]
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float mc = __uint_as_float(odd ? v[4 + i] : v[i]);
            const float mu = __uint_as_float(odd ? v[12 + i] : v[8 + i]);
            const float gc = __shfl_xor_sync(0xffffffffu, __uint_as_float(odd ? v[i] : v[4 + i]), 1);
            const float gu = __shfl_xor_sync(0xffffffffu, __uint_as_float(odd ? v[8 + i] : v[12 + i]), 1);
            cv[i][0] = odd ? gc : mc;
            cv[i][1] = odd ? mc : gc;
            uv[i][0] = odd ? gu : mu;
            uv[i][1] = odd ? mu : gu;
          }
          const int jl = 128 * mb + 32 * (warp & 3) + (lane & ~1);
          if (jl < kHalf) {
            const int n = kHalf * c + jl;
            const float2 bias = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sm.hb + jl));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              if (!live_s[i]) continue;
              const uint32_t c2 = pack2_rn(__fadd_rn(cv[i][0], bias.x), __fadd_rn(cv[i][1], bias.y));
              const uint32_t u2 = pack2_rn(__fadd_rn(uv[i][0], bias.x), __fadd_rn(uv[i][1], bias.y));
              if (lo[i]) {
                *reinterpret_cast<uint32_t*>(lo[i] + n) = c2;
                if (cfg) *reinterpret_cast<uint32_t*>(lo[i] + kVocab + n) = u2;
              }
              const uint32_t gv = cfg ? guided_value2(c2, u2, cfg_scale, uncond_scale) : c2;
              const uint32_t val = constrain2(gv, n, fl[i], nf[i]);
              uint16_t* dst = sm.u.val + ((s0 + i) & 7) * kVocab + n;  // the slot's row in its sampling CTA
              if (local) {
                *reinterpret_cast<uint32_t*>(dst) = val;
              } else {
                push_b32(dst, peer, val, rb);
              }
            }
          }
        }
        tmem_fence_before_sync();
        // the non-finite flags: to this CTA for its own slots, staged for the peer's
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (nf[i]) atomicOr(local ? &sm.nonfinite[(s0 + i) & 7] : &sm.stage_nonfinite[(s0 + i) & 7], 1u);
        }
        cbar();
        if (threadIdx.x < kPOwn) push_b32(&sm.peer_nonfinite[threadIdx.x], peer, sm.stage_nonfinite[threadIdx.x], rb);
      }
      p_stamp(f, tracer, p, 11);
      finish_round(sm, rd, n_own * kHalf * 2 + kPOwn * 4);  // R5: the peer's half of this CTA's sessions
      p_stamp(f, tracer, p, 12);
      // ---------------- sampling of sessions 8c..8c+7; tokens and next input rows to both CTAs
      if (warp < n_own) {
        const int ls = warp, slot = own0 + warp;
        RowSample rs;
        rs.vals = sm.u.val + ls * kVocab;
        rs.flags = sm.flags[slot];
        rs.nonfinite = (sm.nonfinite[ls] | sm.peer_nonfinite[ls]) != 0;
        rs.seed = sm.seed[ls];
        rs.counter = sm.ctr[ls];
        uint16_t* lists = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(sm.xa) + ls * kListBytes);
        int invalid = 0;
        const int token = sample_row(rs, f.prm, lists, lists + kListCap + 8, &invalid);
        __syncwarp();
        const uint32_t rb = peer_bar(sm, rd, peer);
        if (lane == 0) {
          sm.tok[slot][p] = token;
          sm.inv[ls] |= invalid;
          const bool counter_valid = rs.counter >= 0 && rs.counter <= kMaxCounter;
          if (!f.prm.argmax && counter_valid) sm.ctr[ls] = rs.counter + 1;
          if (p + 1 < kPositions) push_b32(&sm.tok[slot][p], peer, static_cast<uint32_t>(token), rb);
        }
        if (folded && p + 1 < kPositions) {
          const int64_t tin = f.forced ? clamp_token(f.forced[static_cast<int64_t>(sm.sess[slot]) * kPositions + p])
                                       : static_cast<int64_t>(token);
          float e8[8], p8[8];
          unpack8(*reinterpret_cast<const uint4*>(f.emb_proj + (static_cast<int64_t>(p) * kVocab + tin) * kD + lane * 8),
                  e8);
          unpack8(*reinterpret_cast<const uint4*>(f.pos + static_cast<int64_t>(p + 1) * kD + lane * 8), p8);
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = __fadd_rn(e8[e], p8[e]);
          const uint4 row = pack8(y);
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            if (sub < rp) {
              bf16* xr_ = sm.x + (slot + 16 * sub) * kLdX + lane * 8;
              *reinterpret_cast<uint4*>(xr_) = row;
              st_async_v4(cluster_addr(xr_, peer), row, rb);
            }
          }
        }
      }
      p_stamp(f, tracer, p, 13);
      if (p + 1 < kPositions) {
        if (threadIdx.x == 0) push_b32(&sm.sink, peer, 0u, peer_bar(sm, rd, peer));  // the round's token
        finish_round(sm, rd, n_peer * (4 + (folded ? rp * kD * 2 : 0)) + 4);  // R6: the peer's tokens and rows
      } else {
        cbar();
      }
      p_stamp(f, tracer, p, 14);
      p_stamp(f, tracer, p, 15);
    }
    if (tracer) f.trace[258] = static_cast<uint64_t>(clock64()), f.trace[259] = global_ns();
    // ---- commit: tokens, counters, flags, next-frame embedding of the sessions this CTA sampled
    if (threadIdx.x == 0 && sm.err) {
      for (int s = 0; s < kPSlots; ++s) {
        const int last = sm.last_issued[s];
        if (last >= 0) mbar_wait(&sm.full[s], (last / kPSlots) & 1);
      }
    }
    for (int i = threadIdx.x; i < n_own * kPositions; i += kPC) {
      const int ls = i / kPositions, pp = i % kPositions;
      const int sid = sm.sess[own0 + ls];
      const int32_t t = sm.tok[own0 + ls][pp];
      f.codec_tokens[codec_index(f, sid, pp)] = t;
      f.tokens[static_cast<int64_t>(sid) * kPositions + pp] = t;
    }
    if (threadIdx.x < n_own) {
      const int ls = threadIdx.x;
      const int sid = sm.sess[own0 + ls];
      f.counter_io[sid] = sm.ctr[ls];
      f.invalid_rows[sid] = sm.inv[ls] | (sm.err ? 4 : 0);
      if (f.eos_slot[sid] < 0) commit_end(f, sid, f.finished[sid] ? 0 : -1);
    }
    for (int i = threadIdx.x; i < n_own * (kEmbed / 8); i += kPC) {
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
    // the head MMA thread's MMAs have completed before TMEM is freed (bounded)
    if (threadIdx.x == 0) {
      const unsigned long long t0 = global_ns();
      while (*reinterpret_cast<volatile int*>(&sm.mma_done) == 0 && global_ns() - t0 < 20000000ull) __nanosleep(1000);
    }
    tmem_fence_before_sync();
    cbar();
    if (warp == 0) {
      tmem_fence_after_sync();
      tmem_dealloc(sm.tmem, kTmemCols);
    }
  }
  cluster.sync();  // no CTA leaves while its peer may still push into it
}

}  // namespace

int pair_frame_clusters() {
  static PerDeviceInt cache;  // the opt-in below is per device context
  return cache.get([] {
    int clusters = 0;
    if (cudaFuncSetAttribute(pair_frame_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPSmemBytes)) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2);
      cfg.blockDim = dim3(kPThreads);
      cfg.dynamicSmemBytes = kPSmemBytes;
      if (cudaOccupancyMaxActiveClusters(&clusters, pair_frame_kernel, &cfg) != cudaSuccess) clusters = 0;
    }
    cudaGetLastError();
    return clusters;
  });
}

bool pair_frame_supported(const Frame& f) {
  if (f.d != kD || f.H != kHeads || f.F != kF || f.L != 1 || !f.in_proj || (f.rp != 1 && f.rp != 2)) return false;
  return pair_frame_clusters() > 0;
}

cudaError_t launch_pair_frame(const Frame& f, cudaStream_t stream) {
  PairMaps maps;
  if (!make_weight_map(&maps.in_proj, f.in_w, kEmbed, kD, kCRows) ||
      !make_weight_map(&maps.qkv, f.qkv, kD, 3 * kD, kCRows) || !make_weight_map(&maps.o, f.o, kD, kD, kCRows) ||
      !make_weight_map(&maps.ffn1, f.w1, kD, kF, kCRows) || !make_weight_map(&maps.ffn2, f.w2, kF, kD, kCRows) ||
      !make_weight_map(&maps.head, f.head_w, kD, static_cast<uint64_t>(kPositions) * kVocab, kHeadRows)) {
    return cudaErrorInvalidValue;
  }
  const int pairs = (f.n + kPS - 1) / kPS;
  cudaError_t e = cudaMemsetAsync(f.eos_count, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  pair_frame_kernel<<<2 * pairs, kPThreads, kPSmemBytes, stream>>>(f, maps);
  return launch_frame_eos(f, stream);
}

}  // namespace mtt
