// Fused Local AR frame: one kernel launch runs all 16 positions of a frame
// for every active session, one 16-CTA thread-block cluster per tile of
// 8 sessions (16 CFG rows).  Clusters never wait on each other.
//
// Per position and per tile (reference ops: tools/export/local_ar_wrapper.py:
// 609-751; transformer_2501.py:405-442,761-851,1153-1232; sampling
// plugins/local_ar_plugins.cu:1211-1370; embedding sum
// main_decoder_wrapper.py:796-810), CTA c of the cluster:
//
//   Ph0 in-projection: at p = 0, features [16c, +16) of bf16(bf16(W_in h + b)
//       + pos[0]) for the 16 decoder-hidden rows, all-gathered into every
//       CTA's x.  At p >= 1 every CTA gathers x = bf16(emb_proj[p-1][token] +
//       pos[p]) locally from the folded tables (fold.cu); without them the
//       sampled token's embedding row is multiplied like the hidden rows.
//   Ph1 LN1(x) (every CTA, all rows); qkv features of head h = c / 4,
//       head-dims [16(c%4), +16): q kept, k/v appended to this CTA's K/V
//       slice; partial q.k over those 16 dims sent to the 4 CTAs of head h.
//   Ph2 attention for head h, dims slice: scores = sum of the 4 partials,
//       bf16 rounding, x 1/8, softmax, probability-weighted V slice;
//       all-gathered into every CTA's attention buffer.
//   Ph3 o-projection features [16c, +16) + residual, all-gathered into x.
//   Ph4 LN2(x); FFN1 features [64c, +64) + GELU-tanh (kept locally); their
//       FFN2 contribution h_c W2[:, 64c:+64]^T (f32) scattered to the owners
//       of the output features.
//   Ph5 the 16 partial sums of features [16c, +16), in CTA order, bf16, +
//       residual, all-gathered into x.
//   Ph6 head_p features [128c, +128) (+bias); each session's logits rows are
//       sent to the CTA that owns the session (CTA s owns session s).
//   Ph7 the owner samples (sampling.cuh) and broadcasts the token; it keeps
//       the RNG counter and the invalid flag, and at the end of the frame
//       forms the next-frame embedding sum from the 16 sampled rows.
//
// Exchanges are pushes, not barriers: the data goes out with st.async to the
// receivers' shared memory and completes on the receiver's round mbarrier,
// which the receiver arms with the bytes it expects; every CTA pushes to
// every CTA in every round (a 4-byte token where it has no data for one), so
// a completed round means every CTA finished the phase before it.  No buffer
// written in a round is read by any CTA during that round, so this ordering
// is enough.  Weight slices stream from global memory
// (L2-resident across frames) through a two-slot ring of TMA tensor copies
// (cp.async.bulk.tensor.2d, 128-byte swizzle, no multicast), one phase
// ahead of use.  The 16-row tiles run on mma.sync m16n8k16 (bf16 in, f32
// accumulate): at 16 rows each layer is a weight-streaming GEMV, below
// tcgen05's 64-row minimum.  Every wait is bounded; a timeout sets invalid
// bit 4 for the tile's sessions instead of hanging.
//
// Supported shape: d_model 256, 4 heads, FFN 1024, 1 layer, in-projection
// (the benchmark shape); others use the phase kernels in frame.cu.
#include <cooperative_groups.h>
#include <cuda.h>

#include <mutex>

#include "eos_proj.cuh"
#include "frame_common.cuh"
#include "ptx.cuh"
#include "sampling.cuh"

namespace cg = cooperative_groups;

namespace mtt {
namespace {

constexpr int kCS = 16;       // CTAs per cluster
constexpr int kM = 16;        // rows per tile
constexpr int kThreads = 256;
constexpr int kD = 256;
constexpr int kHeads = 4;
constexpr int kF = 1024;
constexpr int kDC = kD / kCS;       // 16 residual features per CTA
constexpr int kFC = kF / kCS;       // 64 FFN features per CTA
constexpr int kG = kCS / kHeads;    // 4 CTAs per head
constexpr int kHD = kHeadDim / kG;  // 16 head dims per CTA
constexpr int kLd256 = kD + 8;
constexpr int kLd768 = kEmbed + 8;
constexpr int kLdH = kFC + 8;
constexpr int kHeadCols = 128;  // head features per CTA (the last CTA: 2024 - 15*128 = 104)
constexpr int kPanel = 64;      // TMA box inner extent: 64 bf16 = one 128-byte swizzle row
constexpr int kSlotElems = kHeadCols * kD;  // 64 KB: the largest chunk (head slice)
constexpr unsigned long long kWaitLimitNs = 20000000ull;  // bounded mbarrier wait: 20 ms

static_assert(kHeadDim % kG == 0 && kHD == 16, "head split");
static_assert(16 * kEmbed <= kSlotElems && 48 * kD <= kSlotElems && 64 * kD <= kSlotElems && kD * kFC <= kSlotElems,
              "ring slot");

// TMA descriptors of the weight matrices (2D, bf16, 128-byte swizzle).
struct WeightMaps {
  CUtensorMap in_proj;  // [256][768]    box 64 x 16
  CUtensorMap qkv;      // [768][256]    box 64 x 16
  CUtensorMap o;        // [256][256]    box 64 x 16
  CUtensorMap ffn1;     // [1024][256]   box 64 x 64
  CUtensorMap ffn2;     // [256][1024]   box 64 x 256 (a 64-column K slice)
  CUtensorMap head;     // [16*2024][256] box 64 x 128
};

// Shared buffer reused by phases that never overlap: the in-projection
// source rows (position 0 / unfolded), the FFN2 partial sums received from
// the 16 CTAs, and the sampler's scratch.
union BigBuffer {
  bf16 src[kM * kLd768];
  float recv[kCS][kM][kDC];
  unsigned char sample_scratch[kSampleScratchBytes];
  struct {                           // this CTA's head columns in candidate form, per session
    uint16_t key[kM][kHeadCols];
    float score[kM][kHeadCols];
  } cand_out;
};

struct __align__(1024) Smem {
  bf16 ring[2][kSlotElems];  // 1024-byte aligned panels (128-byte swizzle atoms)
  bf16 x[kM * kLd256];       // residual stream, all rows, all features
  bf16 xa[kM * kLd256];      // LN output / attention output
  BigBuffer big;
  bf16 hc[kM * kLdH];        // this CTA's FFN1 features (GELU output)
  bf16 kv[2][kM][kPositions][kHD];
  bf16 qs[kM][kHD];
  float part[kG][kM][kPositions];  // partial q.k received from the head group
  union {
    struct {                   // this CTA's session row in candidate form (owner), written by all CTAs
      uint16_t key[2048];      // order keys of the constrained values
      float score[2048];       // Philox-Gumbel scores
      uint32_t nf[kCS];        // per sender: a raw value was non-finite
    } cand;
    float red[8][kM * 8 * 2];  // cross-warp K-split partials
  } u;
  bf16 stage[kM * kHeadCols];  // outgoing slice (bf16) or partial scores (f32)
  bf16 hbias[kHeadCols];       // this CTA's head bias slice of the position (fetched at its start)
  alignas(16) bf16 lnw[2][kD];  // LN1 and LN2 weights
  float gum[kM][kHeadCols];      // fast Gumbel noise of this CTA's columns, per live session, this position
  SampleShared samp;
  int32_t tok[kM][kPositions];  // tokens of the tile's sessions (every CTA)
  int32_t sess[kM];             // stream ids of the tile's sessions
  int64_t seed[kM];             // the tile's sessions: Philox seeds,
  int64_t ctrs[kM];             // working RNG counters (every CTA advances them alike),
  uint32_t flags[kM];           // unfinished | finished << 1 | forbid_eos << 2,
  uint32_t cnf[kM];             // and this CTA's non-finite flag of the position
  int32_t inv;                  // owner: invalid flag
  int32_t n_sess;
  int32_t err;
  unsigned long long mbar[2];   // weight ring
  unsigned long long xbar[2];   // exchange rounds, alternating by round parity
  uint32_t sink[kCS];           // round tokens (never read)
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "fused frame shared memory exceeds the per-CTA limit");

// ---------------------------------------------------------------------------
// 16-row GEMM on the tile: C[16][8*NT] = A[16][16*KS] * B[8*NT][16*KS]^T.
// B is the weight slice in the ring: b_rows x (16*KS) stored as 64-column
// panels of b_rows x 128 bytes, 128-byte swizzled (16-byte chunk j of row n at
// chunk j ^ (n & 7)).  Warps split N (WN warps) and, when N is narrow, K (KW
// chunks reduced in a fixed order through shared memory).  Calls
// epi(row, col, v0, v1) once per pair of adjacent output columns (col even).
// ---------------------------------------------------------------------------

template <int NT, int KS, typename Epi>
__device__ __forceinline__ void gemm16(const bf16* A, int lda, const bf16* B, int b_rows, float* red, Epi epi) {
  constexpr int WN = NT < 8 ? NT : 8;
  constexpr int KW = 8 / WN;
  constexpr int NTW = NT / WN;
  constexpr int KSW = KS / KW;
  static_assert(NT % WN == 0 && KS % KW == 0, "gemm16 split");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool active = warp < WN * KW;
  const int wn = warp % WN, wk = warp / WN;
  float acc[NTW][4];
#pragma unroll
  for (int j = 0; j < NTW; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  if (active) {
    const bf16* a_row = A + ((lane & 7) + 8 * ((lane >> 3) & 1)) * lda + 8 * (lane >> 4);
    const int b_r = lane & 7, b_hi = (lane >> 3) & 1;
#pragma unroll 4
    for (int ks = wk * KSW; ks < (wk + 1) * KSW; ++ks) {
      uint32_t a[4];
      ldsm_x4(a, a_row + 16 * ks);
      const bf16* panel = B + (ks >> 2) * (b_rows * kPanel);
      const int chunk = ((ks & 3) << 1) + b_hi;
#pragma unroll
      for (int j = 0; j < NTW; ++j) {
        const int n = 8 * (wn * NTW + j) + b_r;
        uint32_t b[2];
        ldsm_x2(b, panel + n * kPanel + ((chunk ^ (n & 7)) << 3));
        mma16816(acc[j], a, b);
      }
    }
  }
  if constexpr (KW > 1) {
    if (active && wk > 0) {
#pragma unroll
      for (int j = 0; j < NTW; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[(((wk - 1) * WN + wn) * NTW + j) * 128 + e * 32 + lane] = acc[j][e];
    }
    __syncthreads();
    if (active && wk == 0) {
#pragma unroll
      for (int k = 1; k < KW; ++k)
#pragma unroll
        for (int j = 0; j < NTW; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][e] += red[(((k - 1) * WN + wn) * NTW + j) * 128 + e * 32 + lane];
    }
  }
  if (active && wk == 0) {
#pragma unroll
    for (int j = 0; j < NTW; ++j) {
      const int col0 = 8 * (wn * NTW + j) + 2 * (lane & 3);
      epi(lane >> 2, col0, acc[j][0], acc[j][1]);
      epi((lane >> 2) + 8, col0, acc[j][2], acc[j][3]);
    }
  }
  __syncthreads();
}

// LayerNorm (no bias, eps 1e-5) of the 16 rows of x into xa; warp w: rows 2w, 2w+1.
__device__ __forceinline__ void layer_norm16(const bf16* x, bf16* xa, const bf16* w) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float g[8];
  {
    const uint4 gv = *reinterpret_cast<const uint4*>(w + lane * 8);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(g2[j]);
      g[2 * j] = t.x;
      g[2 * j + 1] = t.y;
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = 2 * warp + rr;
    const uint4 xv = *reinterpret_cast<const uint4*>(x + r * kLd256 + lane * 8);
    const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
    float v[8];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(x2[j]);
      v[2 * j] = t.x;
      v[2 * j + 1] = t.y;
      sum += t.x + t.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(kD);
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) var += (v[j] - mean) * (v[j] - mean);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    const float rstd = 1.0f / sqrtf(var / static_cast<float>(kD) + 1.0e-5f);
    __align__(16) bf16 out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = f2bf(((v[j] - mean) * rstd) * g[j]);
    *reinterpret_cast<uint4*>(xa + r * kLd256 + lane * 8) = *reinterpret_cast<const uint4*>(out);
  }
}

__device__ __forceinline__ float gelu_tanh_f(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

// ---------------------------------------------------------------------------
// exchange rounds
// ---------------------------------------------------------------------------

// Exchange round r uses barrier xbar[r & 1]; its (r >> 1)-th phase.  Two
// barriers keep a fast CTA's next-round arrivals off a barrier that is still
// collecting this round (no CTA can start round r + 2 before every CTA has
// finished round r).
struct Round {
  uint32_t r = 0;
  __device__ __forceinline__ int bar() const { return static_cast<int>(r & 1u); }
  __device__ __forceinline__ uint32_t parity() const { return (r >> 1) & 1u; }
};

// Pushes rows [0, rows) of the [16][cols] bf16 staging slice to every CTA's
// buffer at (dst_ld, dst_col) (cols * 2 and dst_col * 2 multiples of 16
// bytes); rows past the tile's sessions are never sent.
__device__ __forceinline__ void push_all16(Smem& sm, const Round& rd, int rows, int cols, const bf16* dst, int dst_ld,
                                           int dst_col) {
  const int per_row = cols / 8;
  const int chunks = rows * per_row;
  for (int i = threadIdx.x; i < chunks * kCS; i += blockDim.x) {
    const int rank = i / chunks, k = i % chunks;
    const int r = k / per_row, cc = k % per_row;
    const uint4 v = *reinterpret_cast<const uint4*>(sm.stage + r * cols + cc * 8);
    st_async_v4(cluster_addr(dst + r * dst_ld + dst_col + cc * 8, rank), v, cluster_addr(&sm.xbar[rd.bar()], rank));
  }
}

// Waits for this CTA's round: it arms its own round barrier with the bytes
// the cluster pushes to it in this round, and the round completes when they
// have all landed.  Every CTA pushes to every CTA in every round (rounds
// whose data goes to a subset add a 4-byte token to each of the others), so
// a completed round still means every CTA finished the phase before it.
__device__ __forceinline__ void finish_round(Smem& sm, Round& rd, uint32_t bytes_in) {
  __syncthreads();
  if (threadIdx.x == 0) mbar_expect_tx(&sm.xbar[rd.bar()], bytes_in);
  if (sm.err == 0 && !mbar_wait(&sm.xbar[rd.bar()], rd.parity())) sm.err = 1;
  ++rd.r;
  __syncthreads();
}

// 4-byte token from this CTA (rank c) to every CTA, for rounds whose data
// reaches only some of them.
__device__ __forceinline__ void push_tokens(Smem& sm, const Round& rd, int c) {
  if (threadIdx.x < kCS) {
    const int d = static_cast<int>(threadIdx.x);
    st_async_b32(cluster_addr(&sm.sink[c], d), 0u, cluster_addr(&sm.xbar[rd.bar()], d));
  }
}
constexpr uint32_t kTokenBytes = kCS * 4;

// ---------------------------------------------------------------------------
// weight stream
// ---------------------------------------------------------------------------

// Chunk kinds: 0 in-projection, 1 qkv, 2 o, 3 FFN1, 4 FFN2 (K slice), 5 head.
// They travel in groups that share a ring slot: per position [0] (at p = 0,
// or at every position without the folded tables), {1, 2}, {3, 4}, {5}.
// Group g lives in slot g & 1 and is issued as soon as group g - 2's last
// GEMM is done, so each group has the two phases before its use to arrive
// (the head, 64 KB, is in flight from the o-projection on).
constexpr int kGroupO = 3 * kHD * kD;  // element offset of o in group {1, 2}: 24 KB
constexpr int kGroupF2 = kFC * kD;     // element offset of FFN2 in group {3, 4}: 32 KB
static_assert(kGroupO + kDC * kD <= kSlotElems && kGroupF2 + kD * kFC <= kSlotElems, "group fits a slot");
static_assert((kGroupO * 2) % 1024 == 0 && (kGroupF2 * 2) % 1024 == 0, "swizzle-atom aligned chunks");

__device__ __forceinline__ int group_count(bool folded) { return folded ? 4 + 3 * (kPositions - 1) : 4 * kPositions; }

// Group index of (position p, group kind q: 0 in-projection, 1 {qkv, o},
// 2 {FFN1, FFN2}, 3 head), and back.
__device__ __forceinline__ int group_index(bool folded, int p, int q) {
  if (!folded) return 4 * p + q;
  return p == 0 ? q : 4 + 3 * (p - 1) + (q - 1);
}
__device__ __forceinline__ void group_of(bool folded, int g, int& p, int& q) {
  if (!folded || g < 4) {
    p = g / 4;
    q = g % 4;
  } else {
    p = 1 + (g - 4) / 3;
    q = 1 + (g - 4) % 3;
  }
}

__device__ __forceinline__ int chunk_rows(int k) {
  return k == 1 ? 3 * kHD : (k == 3 ? kFC : (k == 4 ? kD : (k == 5 ? kHeadCols : kDC)));
}

// Weight chunk (p, k) for CTA c into dst: one TMA tensor copy per 64-column
// panel, issued by the lanes of the calling warp; completes on bar.
__device__ __forceinline__ void issue_chunk(const WeightMaps& maps, bf16* dst, unsigned long long* bar, int p, int k,
                                            int c) {
  const int lane = threadIdx.x & 31;
  const int rows = chunk_rows(k);
  const CUtensorMap* map;
  int K, x0 = 0, row0 = 0;
  switch (k) {
    case 0: map = &maps.in_proj; K = kEmbed; row0 = kDC * c; break;
    case 1: map = &maps.qkv; K = kD; break;
    case 2: map = &maps.o; K = kD; row0 = kDC * c; break;
    case 3: map = &maps.ffn1; K = kD; row0 = kFC * c; break;
    case 4: map = &maps.ffn2; K = kFC; x0 = kFC * c; break;
    default: map = &maps.head; K = kD; row0 = p * kVocab + kHeadCols * c; break;
  }
  const int panels = K / kPanel;
  const int requests = k == 1 ? 3 * panels : panels;
  if (lane < requests) {
    if (k == 1) {  // q, k, v rows of head h = c / 4, dims [16(c%4), +16): three 16-row boxes per panel
      const int part = lane / panels, pp = lane % panels;
      const int y = part * kD + (c / kG) * kHeadDim + (c % kG) * kHD;
      tma_load_2d(dst + pp * (rows * kPanel) + part * (kHD * kPanel), map, pp * kPanel, y, bar);
    } else {
      tma_load_2d(dst + lane * (rows * kPanel), map, x0 + lane * kPanel, row0, bar);
    }
  }
}

// Issues weight group g (the calling warp, one lane announcing its bytes);
// nothing past the frame's last group.
__device__ __forceinline__ void issue_group(const WeightMaps& maps, Smem& sm, bool folded, int g, int c) {
  if (g >= group_count(folded)) return;
  int p, q;
  group_of(folded, g, p, q);
  bf16* slot = sm.ring[g & 1];
  unsigned long long* bar = &sm.mbar[g & 1];
  // (selected arithmetically: a table indexed at run time would be a memory load)
  const uint32_t bytes = q == 0   ? uint32_t(kDC * kEmbed * 2)
                         : q == 1 ? uint32_t((3 * kHD + kDC) * kD * 2)
                         : q == 2 ? uint32_t(2 * kFC * kD * 2)
                                  : uint32_t(kHeadCols * kD * 2);
  if ((threadIdx.x & 31) == 0) {
    fence_proxy_async();  // the slot's previous contents were read through the generic proxy
    mbar_expect_tx(bar, bytes);
  }
  __syncwarp();
  switch (q) {
    case 0: issue_chunk(maps, slot, bar, p, 0, c); break;
    case 1:
      issue_chunk(maps, slot, bar, p, 1, c);
      issue_chunk(maps, slot + kGroupO, bar, p, 2, c);
      break;
    case 2:
      issue_chunk(maps, slot, bar, p, 3, c);
      issue_chunk(maps, slot + kGroupF2, bar, p, 4, c);
      break;
    default: issue_chunk(maps, slot, bar, p, 5, c); break;
  }
}

// Waits for weight group g; returns its slot.
__device__ __forceinline__ const bf16* wait_group(Smem& sm, int g) {
  if (sm.err == 0 && !mbar_wait(&sm.mbar[g & 1], (g >> 1) & 1)) sm.err = 1;
  __syncthreads();
  return sm.ring[g & 1];
}

// After group g's last GEMM (whose closing barrier every thread has passed):
// its slot takes group g + 2.
__device__ __forceinline__ void release_group(const WeightMaps& maps, Smem& sm, bool folded, int g, int c) {
  if ((threadIdx.x >> 5) == 0) issue_group(maps, sm, folded, g + 2, c);
}

// Phase clock stamps (trace hook): CTA 0 of the first cluster writes its SM
// clock at 16 points of every position, then the clock and the global timer
// at the start and the end of the frame (to convert cycles to time).
__device__ __forceinline__ void stamp(const Frame& f, int p, int i) {
  if (f.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) f.trace[p * 16 + i] = clock64();
}
__device__ __forceinline__ void stamp_frame(const Frame& f, int at) {
  if (f.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) {
    uint64_t ns;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ns));
    f.trace[kPositions * 16 + 2 * at] = clock64();
    f.trace[kPositions * 16 + 2 * at + 1] = ns;
  }
}

__device__ __forceinline__ int64_t fused_input_token(const Frame& f, const Smem& sm, int s_local, int p) {
  if (f.forced) {
    const int64_t t = f.forced[static_cast<int64_t>(sm.sess[s_local]) * kPositions + p];
    return t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
  }
  return sm.tok[s_local][p];
}


__global__ void __cluster_dims__(kCS, 1, 1) __launch_bounds__(kThreads, 1)
    fused_frame_kernel(Frame f, const __grid_constant__ WeightMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // swizzled TMA destinations need 1024-byte alignment: align inside the
  // allocation (kSmemBytes = sizeof(Smem) + 1024); uniform across CTAs
  const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + pad);
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int tile = static_cast<int>(blockIdx.x) / kCS;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rp = f.rp;
  const int spt = kM / rp;  // sessions per tile
  const bool folded = f.emb_proj != nullptr;

  // ---- tile mapping: sessions [spt*tile, spt*tile + spt) of the active list
  if (warp == 0) {
    int seen = 0;
    const int first = spt * tile;
    for (int base = 0; base < f.n; base += 32) {
      const int s = base + lane;
      const bool act = s < f.n && (f.active == nullptr || f.active[s]);
      const unsigned m = __ballot_sync(0xffffffffu, act);
      const int rank = seen + __popc(m & ((1u << lane) - 1u));
      if (act && rank >= first && rank < first + spt) sm.sess[rank - first] = s;
      seen += __popc(m);
    }
    if (lane == 0) {
      const int left = seen - first;
      sm.n_sess = left <= 0 ? 0 : (left < spt ? left : spt);
      sm.err = 0;
    }
  }
  __syncthreads();
  const int n_sess = sm.n_sess;
  if (n_sess == 0) return;  // uniform across the cluster: no DSMEM traffic
  const int rows = n_sess * rp;

  if (threadIdx.x == 0) {
    mbar_init(&sm.mbar[0], 1);
    mbar_init(&sm.mbar[1], 1);
    mbar_init(&sm.xbar[0], 1);
    mbar_init(&sm.xbar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0 && lane < 6) {  // the six tensor maps into the TMA descriptor cache
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(reinterpret_cast<const CUtensorMap*>(&maps) + lane))
                 : "memory");
  }
  if (warp == 0) {
    issue_group(maps, sm, folded, 0, c);
    issue_group(maps, sm, folded, 1, c);
  }

  for (int i = threadIdx.x; i < kD / 8; i += blockDim.x) {
    reinterpret_cast<uint4*>(sm.lnw[0])[i] = reinterpret_cast<const uint4*>(f.ln1)[i];
    reinterpret_cast<uint4*>(sm.lnw[1])[i] = reinterpret_cast<const uint4*>(f.ln2)[i];
  }
  // ---- session state (every CTA scores every session's tokens)
  if (static_cast<int>(threadIdx.x) < n_sess) {
    const int sid = sm.sess[threadIdx.x];
    sm.seed[threadIdx.x] = f.seed[sid];
    sm.ctrs[threadIdx.x] = f.counter_io[sid];
    sm.flags[threadIdx.x] = (f.unfinished[sid] ? 1u : 0u) | (f.finished[sid] ? 2u : 0u) | (f.forbid[sid] ? 4u : 0u);
  }
  // ---- owner state
  const bool owner = c < n_sess;
  if (owner && threadIdx.x == 0) {
    const int sid = sm.sess[c];
    int32_t inv = 0;
    bool en = !f.unfinished[sid] && !f.finished[sid] && !f.forbid[sid];
    if (en && f.final_w == nullptr) {
      inv = 2;
      en = false;
    }
    sm.inv = inv;
    if (en) {
      const int slot = atomicAdd(f.eos_count, 1);
      f.eos_list[slot] = sid;
      f.eos_slot[sid] = slot;
    } else {
      f.eos_slot[sid] = -1;
    }
  }
  for (int i = threadIdx.x; i < kM * kLd256 / 8; i += blockDim.x) {
    reinterpret_cast<uint4*>(sm.x)[i] = make_uint4(0, 0, 0, 0);  // rows past the tile's sessions stay zero
  }
  cluster.sync();  // every CTA is running and its barriers initialised before any DSMEM access

  Round rd;
  const int hcols = c < kCS - 1 ? kHeadCols : kVocab - (kCS - 1) * kHeadCols;
  const bool bias_async = (reinterpret_cast<uintptr_t>(f.head_b) & 3u) == 0;
  const int head = c / kG, ds = c % kG;
  const uint32_t slice_bytes = static_cast<uint32_t>(rows) * kDC * 2;  // the live rows of a [16][16] bf16 slice
  stamp_frame(f, 0);
  for (int p = 0; p < kPositions; ++p) {
    stamp(f, p, 0);
    if (threadIdx.x < kM) sm.cnf[threadIdx.x] = 0;
    // the head bias slice of this position, in flight until the head phase
    if (bias_async && 2 * static_cast<int>(threadIdx.x) < hcols) {
      cp_async4(&sm.hbias[2 * threadIdx.x], f.head_b + static_cast<int64_t>(p) * kVocab + kHeadCols * c + 2 * threadIdx.x);
    }
    // ---------------- Ph0: in-projection + position embedding
    if (p > 0 && folded) {
      for (int i = threadIdx.x; i < kM * (kD / 8); i += blockDim.x) {
        const int r = i / (kD / 8), ch = i % (kD / 8);
        __align__(16) bf16 out[8];
        if (r < rows) {
          const int sl = r / rp;
          const uint4 pv = *reinterpret_cast<const uint4*>(
              f.emb_proj + (static_cast<int64_t>(p - 1) * kVocab + fused_input_token(f, sm, sl, p - 1)) * kD + ch * 8);
          const uint4 qv = *reinterpret_cast<const uint4*>(f.pos + static_cast<int64_t>(p) * kD + ch * 8);
          const bf16* pb = reinterpret_cast<const bf16*>(&pv);
          const bf16* qb = reinterpret_cast<const bf16*>(&qv);
#pragma unroll
          for (int j = 0; j < 8; ++j) out[j] = f2bf(__fadd_rn(bf2f(pb[j]), bf2f(qb[j])));
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) out[j] = f2bf(0.f);
        }
        *reinterpret_cast<uint4*>(sm.x + r * kLd256 + ch * 8) = *reinterpret_cast<const uint4*>(out);
      }
      __syncthreads();
    } else {
      for (int i = threadIdx.x; i < kM * (kEmbed / 8); i += blockDim.x) {
        const int r = i / (kEmbed / 8), ch = i % (kEmbed / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < rows) {
          const int sl = r / rp, sub = r % rp;
          const bf16* src;
          if (p == 0) {
            src = f.hidden + (static_cast<int64_t>(sm.sess[sl]) * rp + sub) * kEmbed;
          } else {
            src = f.emb + (static_cast<int64_t>(p - 1) * kVocab + fused_input_token(f, sm, sl, p - 1)) * kEmbed;
          }
          v = *reinterpret_cast<const uint4*>(src + ch * 8);
        }
        *reinterpret_cast<uint4*>(sm.big.src + r * kLd768 + ch * 8) = v;
      }
      const int g = group_index(folded, p, 0);
      const bf16* w = wait_group(sm, g);
      gemm16<2, 48>(sm.big.src, kLd768, w, kDC, &sm.u.red[0][0], [&](int r, int j, float v0, float v1) {
        const int n = kDC * c + j;
        const float y0 = round_bf16(__fadd_rn(v0, bf2f(f.in_b[n])));
        const float y1 = round_bf16(__fadd_rn(v1, bf2f(f.in_b[n + 1])));
        const bf16* pos = f.pos + static_cast<int64_t>(p) * kD + n;
        *reinterpret_cast<uint32_t*>(sm.stage + r * kDC + j) =
            pack_bf16x2(__fadd_rn(y0, bf2f(pos[0])), __fadd_rn(y1, bf2f(pos[1])));
      });
      release_group(maps, sm, folded, g, c);
      push_all16(sm, rd, rows, kDC, sm.x, kLd256, kDC * c);
      finish_round(sm, rd, kCS * slice_bytes);
    }
    stamp(f, p, 1);

    // ---------------- Ph1: LN1, qkv slice, partial scores to the head group
    layer_norm16(sm.x, sm.xa, sm.lnw[0]);
    const int g1 = group_index(folded, p, 1), g2 = g1 + 1, g3 = g1 + 2;
    const bf16* wg1 = wait_group(sm, g1);
    {
      const bf16* w = wg1;
      gemm16<6, 16>(sm.xa, kLd256, w, 3 * kHD, &sm.u.red[0][0], [&](int r, int j, float v0, float v1) {
        const int part = j / kHD, i = j % kHD;  // j even: the pair stays inside one part
        const uint32_t y = pack_bf16x2(v0, v1);
        if (part == 0) {
          *reinterpret_cast<uint32_t*>(&sm.qs[r][i]) = y;
        } else {
          *reinterpret_cast<uint32_t*>(&sm.kv[part - 1][r][p][i]) = y;
        }
      });
    }
    {
      float* scores = reinterpret_cast<float*>(sm.stage);  // [16][16] f32
      const int r = threadIdx.x >> 4, jk = threadIdx.x & 15;
      float s = 0.f;
      if (jk <= p) {
#pragma unroll
        for (int i = 0; i < kHD; ++i) s = fmaf(bf2f(sm.qs[r][i]), bf2f(sm.kv[0][r][jk][i]), s);
      }
      scores[r * kPositions + jk] = s;
      __syncthreads();
      // the live rows (64 bytes each) to each of the 4 CTAs of head h
      const int g = threadIdx.x >> 6, ch = threadIdx.x & 63;
      const int dst = head * kG + g;
      if (ch < rows * 4) {
        const uint4 v = *reinterpret_cast<const uint4*>(scores + ch * 4);
        st_async_v4(cluster_addr(reinterpret_cast<const float*>(&sm.part[ds][0][0]) + ch * 4, dst), v,
                    cluster_addr(&sm.xbar[rd.bar()], dst));
      }
    }
    stamp(f, p, 2);
    push_tokens(sm, rd, c);
    // the position's Gumbel noise depends only on (seed, counter, token):
    // drawn here, while the scores round is in flight, and added to the
    // values once the head's logits exist
    if (!f.prm.argmax) {
      for (int i = threadIdx.x; i < n_sess * hcols; i += blockDim.x) {
        const int sl = i / hcols, j = i % hcols;
        sm.gum[sl][j] = fast_gumbel(philox_uniform(
            call_seed32(sm.seed[sl]), call_offset(sm.ctrs[sl]) + static_cast<uint64_t>(kHeadCols * c + j)));
      }
    }
    finish_round(sm, rd, kG * uint32_t(rows * kPositions * 4) + kTokenBytes);
    stamp(f, p, 3);

    // ---------------- Ph2: attention (head, dims slice), all-gathered
    {
      const int r = threadIdx.x >> 4, jk = threadIdx.x & 15;
      float s = -CUDART_INF_F;
      if (jk <= p) {
        float acc = 0.f;
#pragma unroll
        for (int g = 0; g < kG; ++g) acc += sm.part[g][r][jk];
        s = round_bf16(__fmul_rn(round_bf16(acc), 0.125f));
      }
      float mx = s;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float e = jk <= p ? expf(s - mx) : 0.f;
      float sum = e;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float prob = round_bf16(e / sum);
      float o_acc = 0.f;
      const int gbase = lane & 16;
      for (int j = 0; j <= p; ++j) {
        const float pj = __shfl_sync(0xffffffffu, prob, gbase + j);
        o_acc = fmaf(pj, bf2f(sm.kv[1][r][j][jk]), o_acc);
      }
      sm.stage[r * kHD + jk] = f2bf(o_acc);
    }
    __syncthreads();
    stamp(f, p, 4);
    push_all16(sm, rd, rows, kHD, sm.xa, kLd256, head * kHeadDim + ds * kHD);
    finish_round(sm, rd, kCS * slice_bytes);
    stamp(f, p, 5);

    // ---------------- Ph3: o-projection + residual, all-gathered
    {
      const bf16* w = wg1 + kGroupO;
      gemm16<2, 16>(sm.xa, kLd256, w, kDC, &sm.u.red[0][0], [&](int r, int j, float v0, float v1) {
        const int n = kDC * c + j;
        const float x0 = bf2f(sm.x[r * kLd256 + n]), x1 = bf2f(sm.x[r * kLd256 + n + 1]);
        *reinterpret_cast<uint32_t*>(sm.stage + r * kDC + j) =
            pack_bf16x2(__fadd_rn(x0, round_bf16(v0)), __fadd_rn(x1, round_bf16(v1)));
      });
    }
    release_group(maps, sm, folded, g1, c);
    stamp(f, p, 6);
    push_all16(sm, rd, rows, kDC, sm.x, kLd256, kDC * c);
    finish_round(sm, rd, kCS * slice_bytes);
    stamp(f, p, 7);

    // ---------------- Ph4: LN2, FFN1 slice + GELU, FFN2 partials to the owners
    layer_norm16(sm.x, sm.xa, sm.lnw[1]);
    const bf16* wg2 = wait_group(sm, g2);
    {
      const bf16* w = wg2;
      gemm16<8, 16>(sm.xa, kLd256, w, kFC, &sm.u.red[0][0], [&](int r, int j, float v0, float v1) {
        *reinterpret_cast<uint32_t*>(sm.hc + r * kLdH + j) =
            pack_bf16x2(gelu_tanh_f(round_bf16(v0)), gelu_tanh_f(round_bf16(v1)));
      });
    }
    stamp(f, p, 8);
    {
      const bf16* w = wg2 + kGroupF2;
      gemm16<32, 4>(sm.hc, kLdH, w, kD, &sm.u.red[0][0], [&](int r, int j, float v0, float v1) {
        const int dst = j / kDC;
        if (r < rows) {
          st_async_v2f(cluster_addr(&sm.big.recv[c][r][j % kDC], dst), v0, v1, cluster_addr(&sm.xbar[rd.bar()], dst));
        }
      });
    }
    release_group(maps, sm, folded, g2, c);
    stamp(f, p, 9);
    finish_round(sm, rd, kCS * uint32_t(rows * kDC * 4));
    stamp(f, p, 10);

    // ---------------- Ph5: FFN2 output features (16 partials in CTA order) + residual
    {
      const int r = threadIdx.x >> 4, j = threadIdx.x & 15;
      float acc = 0.f;
#pragma unroll
      for (int s = 0; s < kCS; ++s) acc += sm.big.recv[s][r][j];
      const int n = kDC * c + j;
      sm.stage[r * kDC + j] = f2bf(__fadd_rn(bf2f(sm.x[r * kLd256 + n]), round_bf16(acc)));
    }
    __syncthreads();
    push_all16(sm, rd, rows, kDC, sm.x, kLd256, kDC * c);
    finish_round(sm, rd, kCS * slice_bytes);
    stamp(f, p, 11);

    // ---------------- Ph6: head p; logits rows to the owners
    if (bias_async) cp_async_wait_all();  // published by wait_group's barrier
    {
      const bf16* w = wait_group(sm, g3);
      gemm16<16, 16>(sm.x, kLd256, w, kHeadCols, &sm.u.red[0][0], [&](int r, int j, float v0, float v1) {
        if (j < hcols) {  // hcols is even: pairs never straddle it
          const int n = kHeadCols * c + j;
          const bf16* hb = bias_async ? &sm.hbias[j] : f.head_b + static_cast<int64_t>(p) * kVocab + n;
          const bf16 y0 = f2bf(__fadd_rn(v0, bf2f(hb[0])));
          const bf16 y1 = f2bf(__fadd_rn(v1, bf2f(hb[1])));
          sm.stage[r * kHeadCols + j] = y0;
          sm.stage[r * kHeadCols + j + 1] = y1;
          if (f.logits_out && r < rows) {
            const int sl = r / rp, sub = r % rp;
            bf16* lo = f.logits_out + ((static_cast<int64_t>(sm.sess[sl]) * kPositions + p) * rp + sub) * kVocab + n;
            lo[0] = y0;
            lo[1] = y1;
          }
        }
      });
    }
    release_group(maps, sm, folded, g3, c);
    stamp(f, p, 12);
    {
      // every live session's row (pair) in candidate form: the constrained
      // value's order key and its fast Philox-Gumbel score, for this CTA's
      // columns (the argmax mode sends no scores: -inf)
      const float cfg = f.prm.cfg_scale, temp = f.prm.temperature;
      for (int i = threadIdx.x; i < n_sess * hcols; i += blockDim.x) {
        const int sl = i / hcols, j = i % hcols, t = kHeadCols * c + j;
        const float cond = bf2f(sm.stage[(sl * rp) * kHeadCols + j]);
        const float raw = rp == 2 ? guided_logit(cond, bf2f(sm.stage[(sl * rp + 1) * kHeadCols + j]), cfg) : cond;
        const uint32_t fl = sm.flags[sl];
        bool nf = false;
        const float v = constrain_token(t, raw, fl & 1u, fl & 2u, fl & 4u, &nf);
        if (nf) atomicOr(&sm.cnf[sl], 1u);
        sm.big.cand_out.key[sl][j] = static_cast<uint16_t>(value_key16(v));
        // token_score_fast with the noise drawn in Ph1
        sm.big.cand_out.score[sl][j] =
            f.prm.argmax || v == -CUDART_INF_F ? -CUDART_INF_F : __fadd_rn(__fdiv_rn(v, temp), sm.gum[sl][j]);
      }
      __syncthreads();
      const int kch = hcols / 8, sch = hcols / 4, per = kch + sch;  // 16-byte chunks per session
      for (int i = threadIdx.x; i < n_sess * per; i += blockDim.x) {
        const int sl = i / per, q = i % per;
        const uint32_t bar = cluster_addr(&sm.xbar[rd.bar()], sl);
        if (q < kch) {
          const uint4 v = reinterpret_cast<const uint4*>(&sm.big.cand_out.key[sl][0])[q];
          st_async_v4(cluster_addr(&sm.u.cand.key[kHeadCols * c + 8 * q], sl), v, bar);
        } else {
          const uint4 v = reinterpret_cast<const uint4*>(&sm.big.cand_out.score[sl][0])[q - kch];
          st_async_v4(cluster_addr(&sm.u.cand.score[kHeadCols * c + 4 * (q - kch)], sl), v, bar);
        }
      }
      if (static_cast<int>(threadIdx.x) < n_sess) {
        const int d = static_cast<int>(threadIdx.x);
        st_async_b32(cluster_addr(&sm.u.cand.nf[c], d), sm.cnf[d], cluster_addr(&sm.xbar[rd.bar()], d));
      }
    }
    push_tokens(sm, rd, c);
    finish_round(sm, rd, (c < n_sess ? uint32_t(kVocab * 6 + kCS * 4) : 0u) + kTokenBytes);
    stamp(f, p, 13);

    // ---------------- Ph7: owner selects the token, broadcasts it
    if (owner) {
      SampleCall call{};
      call.kind = kLogitsBf16;
      const uint32_t fl = sm.flags[c];
      call.unfinished = fl & 1u;
      call.finished = fl & 2u;
      call.forbid_eos = fl & 4u;
      call.seed = sm.seed[c];
      call.counter = sm.ctrs[c];
      uint32_t any_nf = 0;
#pragma unroll
      for (int k = 0; k < kCS; ++k) any_nf |= sm.u.cand.nf[k];
      int invalid = 0;
      const int token =
          sample_block_scored(sm.u.cand.key, sm.u.cand.score, any_nf != 0, call, f.prm, sm.samp, sm.big.sample_scratch,
                              &invalid);
      if (threadIdx.x < kCS) {
        const int d = static_cast<int>(threadIdx.x);
        st_async_b32(cluster_addr(&sm.tok[c][p], d), static_cast<uint32_t>(token), cluster_addr(&sm.xbar[rd.bar()], d));
      }
      if (threadIdx.x == 0) sm.inv |= invalid;
    }
    stamp(f, p, 14);
    if (!owner) push_tokens(sm, rd, c);  // the owners' tokens are their 4 bytes
    finish_round(sm, rd, kTokenBytes);
    // every CTA advances the tile's counters as the owners do (sampling only)
    if (threadIdx.x == 0 && !f.prm.argmax) {
      for (int sl = 0; sl < n_sess; ++sl) {
        const int64_t k = sm.ctrs[sl];
        if (k >= 0 && k <= kMaxCounter) sm.ctrs[sl] = k + 1;
      }
    }
    stamp(f, p, 15);
  }
  stamp_frame(f, 1);

  // ---- commit (owner): tokens, counter, flags, next-frame embedding
  if (owner) {
    const int sid = sm.sess[c];
    if (threadIdx.x < kPositions) {
      const int pp = threadIdx.x;
      const int32_t t = sm.tok[c][pp];
      f.codec_tokens[codec_index(f, sid, pp)] = t;
      f.tokens[static_cast<int64_t>(sid) * kPositions + pp] = t;
    }
    if (threadIdx.x == 0) {
      f.counter_io[sid] = sm.ctrs[c];
      f.invalid_rows[sid] = sm.inv | (sm.err ? 4 : 0);
      if (f.eos_slot[sid] < 0) commit_end(f, sid, f.finished[sid] ? 0 : -1);
    }
    // sum_p table_p[token_p], each add rounded to bf16, in position order; / 16
    for (int k = threadIdx.x; k < kEmbed; k += blockDim.x) {
      float acc = 0.f;
#pragma unroll
      for (int pp = 0; pp < kPositions; ++pp) {
        const float v = bf2f(f.emb[(static_cast<int64_t>(pp) * kVocab + sm.tok[c][pp]) * kEmbed + k]);
        acc = pp == 0 ? v : round_bf16(__fadd_rn(acc, v));
      }
      f.next_emb[static_cast<int64_t>(sid) * kEmbed + k] = f2bf(__fdiv_rn(acc, 16.0f));
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still address its shared memory
}

// EOS decision for the sessions the frame kernel registered (projection from
// launch_eos_projection); resets the count.  A projection whose bounded waits
// gave up marks the sessions invalid (bit 4).
__global__ void __launch_bounds__(256) fused_eos_finish_kernel(Frame f) {
  wait_prior_grid();  // launched after the EOS projection with programmatic serialization
  const int count = *f.eos_count;
  const bool failed = f.eos_pre == nullptr && f.eos_count[1] != 0;
  for (int e = threadIdx.x; e < count; e += blockDim.x) {
    const int s = f.eos_list[e];
    const int32_t end = eos_decide_proj(eos_keys(f, s, e), eos_logits(f, s, e), f.tokens + s * kPositions, true, false);
    commit_end(f, s, end);
    if (failed) f.invalid_rows[s] |= 16;
  }
  __syncthreads();
  if (threadIdx.x == 0) *f.eos_count = 0;
}

}  // namespace

// ---------------------------------------------------------------------------
// host: TMA descriptors
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    cudaGetLastError();
  });
  return fn;
}

bool make_weight_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr || base == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * sizeof(bf16)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kPanel), box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


int fused_frame_clusters() {
  static PerDeviceInt cache;  // the opt-in below is per device context
  return cache.get([] {
    int clusters = 0;
    if (encode_tiled() != nullptr &&
        cudaFuncSetAttribute(fused_frame_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) == cudaSuccess &&
        cudaFuncSetAttribute(fused_frame_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(kCS);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmemBytes;
      if (cudaOccupancyMaxActiveClusters(&clusters, fused_frame_kernel, &cfg) != cudaSuccess) clusters = 0;
    }
    cudaGetLastError();
    return clusters;
  });
}

bool fused_frame_supported(const Frame& f) {
  if (f.d != kD || f.H != kHeads || f.F != kF || f.L != 1 || !f.in_proj || (f.rp != 1 && f.rp != 2)) return false;
  return fused_frame_clusters() > 0;
}

cudaError_t launch_fused_frame(const Frame& f, cudaStream_t stream) {
  WeightMaps maps;
  if (!make_weight_map(&maps.in_proj, f.in_w, kEmbed, kD, kDC) || !make_weight_map(&maps.qkv, f.qkv, kD, 3 * kD, kHD) ||
      !make_weight_map(&maps.o, f.o, kD, kD, kDC) || !make_weight_map(&maps.ffn1, f.w1, kD, kF, kFC) ||
      !make_weight_map(&maps.ffn2, f.w2, kF, kD, kD) ||
      !make_weight_map(&maps.head, f.head_w, kD, static_cast<uint64_t>(kPositions) * kVocab, kHeadCols)) {
    return cudaErrorInvalidValue;
  }
  const int spt = kM / f.rp;
  const int tiles = (f.n + spt - 1) / spt;
  cudaError_t e = cudaMemsetAsync(f.eos_count, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  fused_frame_kernel<<<tiles * kCS, kThreads, kSmemBytes, stream>>>(f, maps);
  return launch_frame_eos(f, stream);
}

cudaError_t launch_frame_eos(const Frame& f, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  // without the final projection no session was registered; with the Main
  // Decoder's projection (eos_pre) there is nothing to compute here
  if (f.final_w != nullptr && f.eos_pre == nullptr) {
    e = launch_eos_projection(frame_eos_args(f), stream);
    if (e != cudaSuccess) return e;
  }
  e = launch_serialized(fused_eos_finish_kernel, dim3(1), dim3(256), 0, stream, f);
  if (e != cudaSuccess) return e;
  return cudaPeekAtLastError();
}

EosProjArgs frame_eos_args(const Frame& f) {
  EosProjArgs a;
  a.hidden = f.hidden;
  a.hidden_stream_stride = static_cast<int64_t>(f.rp) * kEmbed;
  a.uncond_offset = f.rp == 2 ? kEmbed : 0;
  a.list = f.eos_list;
  a.count = f.eos_count;
  a.n_max = f.n;
  a.weight = f.final_w;
  a.bias = f.final_b;
  a.cfg_scale = f.rp == 2 ? f.prm.cfg_scale : 1.0f;
  a.rows = f.logits;  // the phase kernels' logits scratch is free once the frame's positions are done
  a.max_key = reinterpret_cast<uint32_t*>(f.eos_partial);
  a.eos_logit = f.eos_logit;
  a.proj_stride = kPositions;
  a.status = f.eos_count + 1;
  return a;
}

}  // namespace mtt
