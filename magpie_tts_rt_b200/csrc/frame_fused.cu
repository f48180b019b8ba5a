// Fused Local AR frame: one kernel launch runs all 16 positions of a frame
// for every active session, one 16-CTA thread-block cluster per tile of
// 8 sessions (16 CFG rows).  Clusters never wait on each other, so the only
// synchronisation is the hardware cluster barrier.
//
// Per position and per tile (reference ops: tools/export/local_ar_wrapper.py:
// 609-751; transformer_2501.py:405-442,761-851,1153-1232; sampling
// plugins/local_ar_plugins.cu:1211-1370; embedding sum
// main_decoder_wrapper.py:796-810), CTA c of the cluster:
//
//   Ph0 in-projection: features [16c, 16c+16) of bf16(bf16(W_in src + b) +
//       pos[p]) for the 16 rows (src = decoder hidden at p = 0, else the
//       sampled token's embedding row); all-gathered into every CTA's x.
//       With the folded tables (fold.cu), positions 1..15 instead gather
//       bf16(emb_proj[p-1][token] + pos[p]) for all features locally.
//   Ph1 LN1(x) (every CTA, all rows); qkv features of head h = c / 4,
//       head-dims [16(c%4), +16): q kept, k/v appended to this CTA's K/V
//       slice; partial q.k over those 16 dims sent to the 4 CTAs of head h.
//   Ph2 attention for head h, dims slice: scores = sum of the 4 partials,
//       bf16 rounding, x 1/8, softmax, probability-weighted V slice;
//       all-gathered into every CTA's attention buffer.
//   Ph3 o-projection features [16c, +16) + residual, all-gathered into x.
//   Ph4 LN2(x); FFN1 features [64c, +64) + GELU-tanh, all-gathered (FFN hidden).
//   Ph5 FFN2 features [16c, +16) + residual, all-gathered into x.
//   Ph6 head_p features [128c, +128) (+bias); each session's two logits rows
//       are sent to the CTA that owns the session (CTA s owns session s).
//   Ph7 the owner samples (sampling.cuh) and broadcasts the token; it keeps
//       the RNG counter and the invalid flag, and at the end of the frame
//       forms the next-frame embedding sum from the 16 sampled rows.
//
// Each exchange ends with barrier.cluster (8 per position, 7 when the
// in-projection is folded into the embedding tables: positions 1..15 then
// gather their input rows locally).  Every CTA streams its slice of each
// layer's weights from global memory (L2-resident across frames) through a
// two-slot shared-memory ring: one TMA tensor copy (cp.async.bulk.tensor.2d,
// 128-byte swizzle, no multicast) per 64-column panel, completing on an
// mbarrier, issued one phase ahead of use; the swizzle makes the ldmatrix
// reads bank-conflict free.  The 16-row tiles run on mma.sync m16n8k16 (bf16
// in, f32 accumulate): at 16 rows the contraction is a weight-streaming GEMV,
// below tcgen05's 64-row minimum.
//
// Supported shape: d_model 256, 4 heads, FFN 1024, 1 layer, in-projection
// (the benchmark shape); others use the phase kernels in frame.cu.
#include <cooperative_groups.h>
#include <cuda.h>

#include <mutex>

#include "frame_common.cuh"
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
constexpr int kLd1024 = kF + 8;
constexpr int kHeadCols = 128;  // head features per CTA (the last CTA: 2024 - 15*128 = 104)
constexpr int kPanel = 64;      // TMA box inner extent: 64 bf16 = one 128-byte swizzle row
constexpr int kSlotElems = kHeadCols * kD;  // 64 KB: the largest chunk (head slice)
constexpr uint32_t kWaitLimit = 1u << 22;   // bounded mbarrier wait (try_wait suspends per call)

static_assert(kHeadDim % kG == 0 && kHD == 16, "head split");
static_assert(16 * kEmbed <= kSlotElems && 48 * kD <= kSlotElems && 64 * kD <= kSlotElems && 16 * kF <= kSlotElems,
              "ring slot");
static_assert(kSampleScratchBytes <= kM * kLd1024 * 2, "sampler scratch aliases the FFN buffer");

// TMA descriptors of the weight matrices (2D, bf16, 128-byte swizzle).
struct WeightMaps {
  CUtensorMap in_proj;  // [256][768]   box 64 x 16
  CUtensorMap qkv;      // [768][256]   box 64 x 16
  CUtensorMap o;        // [256][256]   box 64 x 16
  CUtensorMap ffn1;     // [1024][256]  box 64 x 64
  CUtensorMap ffn2;     // [256][1024]  box 64 x 16
  CUtensorMap head;     // [16*2024][256] box 64 x 128
};

struct __align__(1024) Smem;
struct __align__(1024) Smem {
  bf16 ring[2][kSlotElems];  // 1024-byte aligned panels (128-byte swizzle atoms)
  bf16 x[kM * kLd256];      // residual stream, all rows, all features
  bf16 xa[kM * kLd256];     // LN output / attention output
  bf16 big[kM * kLd1024];   // in-projection source rows (ld 776) / FFN hidden (ld 1032) / sampler scratch
  bf16 kv[2][kM][kPositions][kHD];
  bf16 qs[kM][kHD];
  float part[kG][kM][kPositions];
  union {
    bf16 lg[2 * kVocab];      // this CTA's session logits (owner), written by all CTAs
    float red[8][kM * 8 * 2];  // cross-warp K-split partials
  } u;
  bf16 stage[kM * kHeadCols];  // local slice before an all-gather
  SampleShared samp;
  int32_t tok[kM][kPositions];  // tokens of the tile's sessions (every CTA)
  int32_t lead_token[kM];       // tokens feeding the next position (owner broadcast)
  int32_t sess[kM];             // stream ids of the tile's sessions
  int64_t ctr;                  // owner: working RNG counter
  int32_t inv;                  // owner: invalid flag
  int32_t n_sess;
  int32_t err;
  unsigned long long mbar[2];
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// Returns false when the phase did not complete within the bounded wait.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_addr(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// ---------------------------------------------------------------------------
// 16-row GEMM on the tile: C[16][8*NT] = A[16][16*KS] * B[8*NT][16*KS]^T.
// Warps split N (WN warps) and, when N is narrow, K (KW chunks reduced in a
// fixed order through shared memory).  Calls epi(row, col, value) once per
// output element from the thread that holds it.
// ---------------------------------------------------------------------------

template <int NT, int KS, typename Epi>
__device__ __forceinline__ void gemm16(const bf16* A, int lda, const bf16* B, int b_rows, float* red, Epi epi) {
  // B: b_rows x (16*KS) weight slice stored as 64-column panels of b_rows x 128 B,
  // 128-byte swizzled (16-byte chunk j of row n at chunk j ^ (n & 7)).
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
#pragma unroll
      for (int e = 0; e < 4; ++e) epi((lane >> 2) + 8 * (e >> 1), col0 + (e & 1), acc[j][e]);
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

// Copies a [16][cols] bf16 staging slice (row stride cols) into every CTA's
// buffer at (dst_ld, dst_col).  cols * 2 and dst_col * 2 are multiples of 16.
__device__ __forceinline__ void all_gather16(cg::cluster_group& cluster, const bf16* stage, int cols, bf16* dst,
                                             int dst_ld, int dst_col) {
  const int chunks_per_row = cols / 8;
  const int chunks = kM * chunks_per_row;
  for (int i = threadIdx.x; i < chunks * kCS; i += blockDim.x) {
    const int rank = i / chunks, k = i % chunks;
    const int r = k / chunks_per_row, cc = k % chunks_per_row;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * cols + cc * 8);
    bf16* remote = cluster.map_shared_rank(dst, rank);
    *reinterpret_cast<uint4*>(remote + r * dst_ld + dst_col + cc * 8) = v;
  }
}

// Order of the weight chunks a CTA streams: chunk kinds 0 in-projection,
// 1 qkv, 2 o, 3 FFN1, 4 FFN2, 5 head.  With the folded in-projection the
// in-projection chunk exists only at position 0.
__device__ __forceinline__ int chunk_index(bool folded, int p, int k) {
  return folded ? (k == 0 ? 0 : 1 + 5 * p + (k - 1)) : 6 * p + k;
}

// Rows of chunk kind k for CTA c (slot layout: 64-column panels of rows x 128 B).
__device__ __forceinline__ int chunk_rows(int k) {
  return k == 1 ? 3 * kHD : (k == 3 ? kFC : (k == 5 ? kHeadCols : kDC));
}

// Weight chunk (p, k) for CTA c: one TMA tensor copy per 64-column panel,
// issued by the lanes of the calling warp; completes on the slot's mbarrier.
__device__ __forceinline__ void issue_chunk(const WeightMaps& maps, Smem& sm, bool folded, int p, int k, int c) {
  const int slot = chunk_index(folded, p, k) & 1;
  bf16* dst = sm.ring[slot];
  const int lane = threadIdx.x & 31;
  const int rows = chunk_rows(k);
  const CUtensorMap* map;
  int K, row0 = 0, requests;
  switch (k) {
    case 0: map = &maps.in_proj; K = kEmbed; row0 = kDC * c; break;
    case 1: map = &maps.qkv; K = kD; break;
    case 2: map = &maps.o; K = kD; row0 = kDC * c; break;
    case 3: map = &maps.ffn1; K = kD; row0 = kFC * c; break;
    case 4: map = &maps.ffn2; K = kF; row0 = kDC * c; break;
    default: map = &maps.head; K = kD; row0 = p * kVocab + kHeadCols * c; break;
  }
  const int panels = K / kPanel;
  requests = k == 1 ? 3 * panels : panels;
  if (lane == 0) {
    fence_proxy_async();
    mbar_expect_tx(&sm.mbar[slot], static_cast<uint32_t>(rows * K * 2));
  }
  __syncwarp();
  if (lane < requests) {
    if (k == 1) {  // q, k, v rows of head h = c / 4, dims [16(c%4), +16): three 16-row boxes per panel
      const int part = lane / panels, pp = lane % panels;
      const int y = part * kD + (c / kG) * kHeadDim + (c % kG) * kHD;
      tma_load_2d(dst + pp * (rows * kPanel) + part * (kHD * kPanel), map, pp * kPanel, y, &sm.mbar[slot]);
    } else {
      tma_load_2d(dst + lane * (rows * kPanel), map, lane * kPanel, row0, &sm.mbar[slot]);
    }
  }
}

__device__ __forceinline__ int64_t fused_input_token(const Frame& f, const Smem& sm, int s_local, int p) {
  if (f.forced) {
    const int64_t t = f.forced[static_cast<int64_t>(sm.sess[s_local]) * kPositions + p];
    return t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
  }
  return sm.tok[s_local][p];
}

// Waits for weight chunk (p, k) and issues the next chunk of the stream into
// the other slot (freed by the previous weight phase).  Returns the slot.
__device__ __forceinline__ const bf16* next_weights(const WeightMaps& maps, Smem& sm, bool folded, int p, int k,
                                                    int c) {
  const int idx = chunk_index(folded, p, k);
  int np = p, nk = k + 1;
  if (nk == 6) {
    np = p + 1;
    nk = folded ? 1 : 0;
  }
  if ((threadIdx.x >> 5) == 0 && np < kPositions) issue_chunk(maps, sm, folded, np, nk, c);
  if (!mbar_wait(&sm.mbar[idx & 1], (idx >> 1) & 1)) sm.err = 1;
  __syncthreads();
  return sm.ring[idx & 1];
}

__global__ void __cluster_dims__(kCS, 1, 1) __launch_bounds__(kThreads, 1)
    fused_frame_kernel(Frame f, const __grid_constant__ WeightMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // swizzled TMA destinations need 1024-byte alignment: align inside the
  // allocation (sized kSmemBytes = sizeof(Smem) + 1024); uniform across CTAs
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
  if (n_sess == 0) return;  // uniform across the cluster: no DSMEM traffic, no barrier
  const int rows = n_sess * rp;

  if (threadIdx.x == 0) {
    mbar_init(&sm.mbar[0], 1);
    mbar_init(&sm.mbar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0) issue_chunk(maps, sm, folded, 0, 0, c);

  // ---- owner state
  const bool owner = c < n_sess;
  if (owner && threadIdx.x == 0) {
    const int sid = sm.sess[c];
    sm.ctr = f.counter_io[sid];
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
  cluster.sync();  // every CTA of the cluster is running before any DSMEM access

  const int head = c / kG, ds = c % kG;
  for (int p = 0; p < kPositions; ++p) {
    // ---------------- Ph0: in-projection + position embedding
    if (p > 0 && folded) {
      // x = bf16(emb_proj[p-1][token] + pos[p]), every CTA, all features, locally
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
        *reinterpret_cast<uint4*>(sm.big + r * kLd768 + ch * 8) = v;
      }
      const bf16* w = next_weights(maps, sm, folded, p, 0, c);
      gemm16<2, 48>(sm.big, kLd768, w, kDC, &sm.u.red[0][0], [&](int r, int j, float v) {
        const int n = kDC * c + j;
        const float y = round_bf16(__fadd_rn(v, bf2f(f.in_b[n])));
        sm.stage[r * kDC + j] = f2bf(__fadd_rn(y, bf2f(f.pos[static_cast<int64_t>(p) * kD + n])));
      });
      all_gather16(cluster, sm.stage, kDC, sm.x, kLd256, kDC * c);
      cluster.sync();  // B1
    }

    // ---------------- Ph1: LN1, qkv slice, partial scores
    layer_norm16(sm.x, sm.xa, f.ln1);
    {
      const bf16* w = next_weights(maps, sm, folded, p, 1, c);
      gemm16<6, 16>(sm.xa, kLd256, w, 3 * kHD, &sm.u.red[0][0], [&](int r, int j, float v) {
        const bf16 y = f2bf(v);
        const int part = j / kHD, i = j % kHD;
        if (part == 0) {
          sm.qs[r][i] = y;
        } else {
          sm.kv[part - 1][r][p][i] = y;
        }
      });
    }
    {
      const int r = threadIdx.x >> 4, jk = threadIdx.x & 15;
      float s = 0.f;
      if (jk <= p) {
#pragma unroll
        for (int i = 0; i < kHD; ++i) s = fmaf(bf2f(sm.qs[r][i]), bf2f(sm.kv[0][r][jk][i]), s);
      }
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        float* remote = cluster.map_shared_rank(&sm.part[0][0][0], head * kG + g);
        remote[(ds * kM + r) * kPositions + jk] = s;
      }
    }
    cluster.sync();  // B2

    // ---------------- Ph2: attention (head, dims slice)
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
    all_gather16(cluster, sm.stage, kHD, sm.xa, kLd256, head * kHeadDim + ds * kHD);
    cluster.sync();  // B3

    // ---------------- Ph3: o-projection + residual
    {
      const bf16* w = next_weights(maps, sm, folded, p, 2, c);
      gemm16<2, 16>(sm.xa, kLd256, w, kDC, &sm.u.red[0][0], [&](int r, int j, float v) {
        const int n = kDC * c + j;
        sm.stage[r * kDC + j] = f2bf(__fadd_rn(bf2f(sm.x[r * kLd256 + n]), round_bf16(v)));
      });
    }
    all_gather16(cluster, sm.stage, kDC, sm.x, kLd256, kDC * c);
    cluster.sync();  // B4

    // ---------------- Ph4: LN2, FFN1 + GELU
    layer_norm16(sm.x, sm.xa, f.ln2);
    {
      const bf16* w = next_weights(maps, sm, folded, p, 3, c);
      gemm16<8, 16>(sm.xa, kLd256, w, kFC, &sm.u.red[0][0], [&](int r, int j, float v) {
        sm.stage[r * kFC + j] = f2bf(gelu_tanh_f(round_bf16(v)));
      });
    }
    all_gather16(cluster, sm.stage, kFC, sm.big, kLd1024, kFC * c);
    cluster.sync();  // B5

    // ---------------- Ph5: FFN2 + residual
    {
      const bf16* w = next_weights(maps, sm, folded, p, 4, c);
      gemm16<2, 64>(sm.big, kLd1024, w, kDC, &sm.u.red[0][0], [&](int r, int j, float v) {
        const int n = kDC * c + j;
        sm.stage[r * kDC + j] = f2bf(__fadd_rn(bf2f(sm.x[r * kLd256 + n]), round_bf16(v)));
      });
    }
    all_gather16(cluster, sm.stage, kDC, sm.x, kLd256, kDC * c);
    cluster.sync();  // B6

    // ---------------- Ph6: head p; logits rows to the owners
    const int hcols = c < kCS - 1 ? kHeadCols : kVocab - (kCS - 1) * kHeadCols;
    {
      const bf16* w = next_weights(maps, sm, folded, p, 5, c);
      gemm16<16, 16>(sm.x, kLd256, w, kHeadCols, &sm.u.red[0][0], [&](int r, int j, float v) {
        if (j < hcols) {
          const int n = kHeadCols * c + j;
          const bf16 y = f2bf(__fadd_rn(v, bf2f(f.head_b[static_cast<int64_t>(p) * kVocab + n])));
          sm.stage[r * kHeadCols + j] = y;
          if (f.logits_out && r < rows) {
            const int sl = r / rp, sub = r % rp;
            f.logits_out[((static_cast<int64_t>(sm.sess[sl]) * kPositions + p) * rp + sub) * kVocab + n] = y;
          }
        }
      });
    }
    {
      const int chunks_per_row = hcols / 8;
      const int total = rows * chunks_per_row;
      for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int r = i / chunks_per_row, cc = i % chunks_per_row;
        const int sl = r / rp, sub = r % rp;
        const uint4 v = *reinterpret_cast<const uint4*>(sm.stage + r * kHeadCols + cc * 8);
        bf16* remote = cluster.map_shared_rank(&sm.u.lg[0], sl);
        *reinterpret_cast<uint4*>(remote + sub * kVocab + kHeadCols * c + cc * 8) = v;
      }
    }
    cluster.sync();  // B7

    // ---------------- Ph7: owner samples, broadcasts the token
    if (owner) {
      const int sid = sm.sess[c];
      SampleCall call;
      call.logits = &sm.u.lg[0];
      call.uncond_offset = kVocab;
      call.kind = rp == 2 ? kLogitsBf16Cfg : kLogitsBf16;
      call.unfinished = f.unfinished[sid];
      call.finished = f.finished[sid];
      call.forbid_eos = f.forbid[sid];
      call.seed = f.seed[sid];
      call.counter = sm.ctr;
      int invalid = 0;
      const int token = sample_block(call, f.prm, sm.samp, sm.big, &invalid);
      if (threadIdx.x < kCS) {
        int32_t* remote = cluster.map_shared_rank(&sm.tok[0][0], static_cast<int>(threadIdx.x));
        remote[c * kPositions + p] = token;
      }
      if (threadIdx.x == 0) {
        sm.inv |= invalid;
        const bool counter_valid = call.counter >= 0 && call.counter <= kMaxCounter;
        if (!f.prm.argmax && counter_valid) sm.ctr = call.counter + 1;
      }
    }
    cluster.sync();  // B8
  }

  // ---- commit (owner): tokens, counter, flags, next-frame embedding
  if (owner) {
    const int sid = sm.sess[c];
    if (threadIdx.x < kPositions) {
      const int pp = threadIdx.x;
      const int32_t t = sm.tok[c][pp];
      f.codec_tokens[static_cast<int64_t>(sid) * kPositions + (pp % kCodebooks) * kFrames + pp / kCodebooks] = t;
      f.tokens[static_cast<int64_t>(sid) * kPositions + pp] = t;
    }
    if (threadIdx.x == 0) {
      f.counter_io[sid] = sm.ctr;
      f.invalid_rows[sid] = sm.inv | (sm.err ? 4 : 0);
      if (f.eos_slot[sid] < 0) f.end_frame[sid] = f.finished[sid] ? 0 : -1;
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
}

// EOS decision for the sessions the fused kernel registered; resets the count.
__global__ void __launch_bounds__(256) fused_eos_finish_kernel(Frame f) {
  const int count = *f.eos_count;
  for (int e = threadIdx.x; e < count; e += blockDim.x) {
    const int s = f.eos_list[e];
    f.end_frame[s] = eos_decide(f.eos_partial + static_cast<int64_t>(e) * kPositions * kEosChunks,
                                f.eos_logit + static_cast<int64_t>(e) * kPositions, f.tokens + s * kPositions,
                                true, false);
  }
  __syncthreads();
  if (threadIdx.x == 0) *f.eos_count = 0;
}

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

bool make_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
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

}  // namespace

bool fused_frame_supported(const Frame& f) {
  if (f.d != kD || f.H != kHeads || f.F != kF || f.L != 1 || !f.in_proj || (f.rp != 1 && f.rp != 2)) return false;
  static int cached = -1;  // per process: the cluster shape is a property of the device model
  static std::mutex mu;
  const std::lock_guard<std::mutex> lock(mu);
  if (cached < 0) {
    int ok = 0;
    if (encode_tiled() != nullptr &&
        cudaFuncSetAttribute(fused_frame_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) == cudaSuccess &&
        cudaFuncSetAttribute(fused_frame_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(kCS);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmemBytes;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, fused_frame_kernel, &cfg) == cudaSuccess && clusters > 0) ok = 1;
    }
    cudaGetLastError();
    cached = ok;
  }
  return cached == 1;
}

cudaError_t launch_fused_frame(const Frame& f, cudaStream_t stream) {
  WeightMaps maps;
  if (!make_map(&maps.in_proj, f.in_w, kEmbed, kD, kDC) || !make_map(&maps.qkv, f.qkv, kD, 3 * kD, kHD) ||
      !make_map(&maps.o, f.o, kD, kD, kDC) || !make_map(&maps.ffn1, f.w1, kD, kF, kFC) ||
      !make_map(&maps.ffn2, f.w2, kF, kD, kDC) ||
      !make_map(&maps.head, f.head_w, kD, static_cast<uint64_t>(kPositions) * kVocab, kHeadCols)) {
    return cudaErrorInvalidValue;
  }
  const int spt = kM / f.rp;
  const int tiles = (f.n + spt - 1) / spt;
  cudaError_t e = cudaMemsetAsync(f.eos_count, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  fused_frame_kernel<<<tiles * kCS, kThreads, kSmemBytes, stream>>>(f, maps);
  EosArgs ea;
  ea.hidden = f.hidden;
  ea.hidden_stream_stride = static_cast<int64_t>(f.rp) * kEmbed;
  ea.uncond_offset = f.rp == 2 ? kEmbed : 0;
  ea.weight = f.final_w;
  ea.bias = f.final_b;
  ea.cfg_scale = f.rp == 2 ? f.prm.cfg_scale : 1.0f;
  ea.eos_list = f.eos_list;
  ea.eos_count = f.eos_count;
  ea.partial_max = f.eos_partial;
  ea.eos_logit = f.eos_logit;
  eos_project_kernel<<<dim3(kEosChunks, kPositions), kEosThreads, 0, stream>>>(ea);
  fused_eos_finish_kernel<<<1, 256, 0, stream>>>(f);
  return cudaPeekAtLastError();
}

}  // namespace mtt
