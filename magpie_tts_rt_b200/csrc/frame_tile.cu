// Tile frame kernel: one CTA runs all 16 positions of a Local AR frame for a
// tile of up to 8 sessions (16 rows with CFG), with no communication between
// CTAs.  This is the throughput path: at a few hundred sessions per GPU every
// SM holds its own tile, and the per-position critical path is the weight
// stream through the SM, not a cluster exchange.
//
// Per position (reference ops as in frame_fused.cu: local_ar_wrapper.py:609-751,
// transformer_2501.py:405-442,761-851,1153-1232, sampling
// local_ar_plugins.cu:1211-1370, embedding sum main_decoder_wrapper.py:796-810):
//
//   input rows: the in-projection (p = 0, or every p without the folded
//   tables), else x = bf16(emb_proj[p-1][token] + pos[p]) written by the
//   sampling warp as soon as it has the token; LN1; qkv; k/v appended to the
//   KV cache in tensor memory; causal attention over positions 0..p;
//   o-projection + residual; LN2; FFN1 + GELU-tanh; FFN2 + residual; head p
//   (+bias, CFG combine, constraints, order keys and each session's maximum
//   in the epilogue); one warp per session finds the exact top-k threshold,
//   scores the eligible tokens with Philox-Gumbel and picks the token.
//
// Data layout:
//   * Weights stream from global memory (L2-resident across frames) through a
//     five-slot ring of 32 KB chunks (64 weight rows x 256 K columns, four
//     TMA boxes of 64 x 64 with 128-byte swizzle, no multicast), filled by a
//     dedicated producer warp that runs ahead of the eight consumer warps;
//     full/empty mbarriers per slot.  Every GEMM is C[16][N] = A[16][K] W^T on
//     mma.sync m16n8k16 (bf16 in, f32 accumulate): at 16 rows this is a
//     weight-streaming GEMV, below tcgen05's 64-row minimum.  A (the 16 rows)
//     is held in registers for a whole GEMM; each warp reads its 8 weight rows
//     of a chunk with ldmatrix exactly once, in four independent accumulator
//     chains, and finishes a chunk's epilogue while the next chunk's MMAs run.
//   * The KV cache (16 rows x 16 positions x (256 k + 256 v) bf16 = 256 KB)
//     lives in tensor memory: TMEM lane 32h + 2r + half holds, for row r and
//     head h, dims [32 half, +32) of k_j at columns [16j, +16) and of v_j at
//     columns [256 + 16j, +16) (bf16 pairs).  Warps h and h + 4 own TMEM lanes
//     [32h, +32); warp h takes positions 0..7 of head h, warp h + 4 positions
//     8..15, and they exchange scores and partial outputs in shared memory.
//   * Rows: session slot s (s < 8) owns row s (conditional) and, with CFG,
//     row s + 8 (unconditional); one mma.sync thread holds both rows of a
//     session for the same columns, so the CFG combine needs no exchange.
//     Without CFG rows 8..15 are idle.
// Every wait is bounded; a timeout sets invalid bit 4 for the tile's sessions.
#include <cuda.h>

#include <mutex>

#include "frame_common.cuh"
#include "ptx.cuh"
#include "tile_common.cuh"

namespace mtt {
namespace {

constexpr int kTRows = 16;
constexpr int kTSess = 8;                    // session slots per tile
constexpr int kTWarps = 8;                   // consumer warps
constexpr int kTConsumers = kTWarps * 32;    // 256
constexpr int kTThreads = kTConsumers + 128;  // + the producer warpgroup (one warp issues TMA)
// Register split (setmaxnreg): launched at 168 per thread (65536 / 384, rounded
// down to 8); the producer warpgroup drops to 40 and the consumers rise to 232:
// 128 x 40 + 256 x 232 = 64512 = 384 x 168, so the increase never waits.
constexpr int kProducerRegs = 40;
constexpr int kConsumerRegs = 232;
static_assert(128 * kProducerRegs + kTConsumers * kConsumerRegs <= kTThreads * 168, "register split");
constexpr int kTD = 256;
constexpr int kTF = 1024;
constexpr int kTHeads = 4;
constexpr int kCRows = 64;                 // weight rows per chunk
constexpr int kCK = 256;                   // K columns per chunk
constexpr int kCPanel = 64;                // columns per TMA box (128 bytes)
constexpr int kCElems = kCRows * kCK;      // 16384 bf16
constexpr uint32_t kCBytes = kCElems * 2;  // 32 KB
constexpr int kSlots = 5;
constexpr int kLdX = kTD + 8;        // 264
constexpr int kLdSrc = kEmbed + 8;   // 776
constexpr int kLdQkv = 3 * kTD + 8;  // 776
constexpr int kLdHid = kTF + 8;      // 1032
constexpr int kTmemCols = 512;

static_assert(kVocab % 8 == 0, "vocab chunks");
static_assert(kTHeads * kHeadDim == kTD, "heads");

struct TileMaps {
  CUtensorMap in_proj;  // [256][768]
  CUtensorMap qkv;      // [768][256]
  CUtensorMap o;        // [256][256]
  CUtensorMap ffn1;     // [1024][256]
  CUtensorMap ffn2;     // [256][1024]
  CUtensorMap head;     // [16*2024][256]
};

// Attention exchange between the two warps of a head (inside TileU, after
// q/k/v have been consumed).
struct AttnExchange {
  float s[2][kTHeads][32][8];  // scores of positions [8 part, +8)
  float o[kTHeads][32][32];    // part-1 partial outputs
};

// Buffers of phases that never overlap within a position.
union TileU {
  bf16 src[kTRows * kLdSrc];      // in-projection input rows
  bf16 qkv[kTRows * kLdQkv];      // q | k | v of the current position
  AttnExchange att;               // after q/k/v are consumed
  bf16 hid[kTRows * kLdHid];      // FFN1 output
  uint16_t val[kTSess * kVocab];  // constrained (guided) logits, bf16 bits
};
static_assert(sizeof(AttnExchange) <= sizeof(bf16) * kTRows * kLdQkv, "attention exchange");

struct __align__(1024) TileSmem {
  bf16 ring[kSlots][kCElems];  // 1024-byte aligned panels (128-byte swizzle atoms)
  bf16 x[kTRows * kLdX];       // residual stream
  bf16 xa[kTRows * kLdX];      // LN output / attention output
  TileU u;
  uint32_t hist[kTSess][256];  // per session: the eligible-token list (u16)
  __align__(16) bf16 hb[kVocab];  // bias of head p
  int32_t tok[kTSess][kPositions];
  int32_t sess[kTSess];
  int64_t ctr[kTSess];
  int64_t seed[kTSess];
  uint32_t flags[kTSess];  // bit 0 unfinished, bit 1 finished, bit 2 forbid_eos
  int32_t inv[kTSess];
  uint32_t nonfinite[kTSess];
  int32_t last_issued[kSlots];
  int32_t n_sess;
  int32_t err;
  uint32_t tmem;
  unsigned long long full[kSlots];
  unsigned long long empty[kSlots];
};
constexpr size_t kTSmemBytes = sizeof(TileSmem) + 1024;
static_assert(kTSmemBytes <= 232448, "tile kernel shared memory");

__device__ __forceinline__ int err_flag(const TileSmem& sm) { return *reinterpret_cast<const volatile int*>(&sm.err); }

// Named barrier over the eight consumer warps (the producer warp never joins).
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// ---------------------------------------------------------------------------
// weight stream: the chunk schedule of one position (producer and consumers
// walk it in the same order)
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool has_in_projection(bool folded, int p) { return p == 0 || !folded; }

__device__ __forceinline__ int chunks_in_position(bool folded, int p) {
  return (has_in_projection(folded, p) ? 12 : 0) + 12 + 4 + 16 + 16 + 32;
}

// Chunk c of position p: tensor map and box origin (x = K column, y = row).
__device__ __forceinline__ const CUtensorMap* chunk_origin(const TileMaps& m, bool folded, int p, int c, int* x,
                                                           int* y) {
  if (has_in_projection(folded, p)) {
    if (c < 12) {  // in-projection, K-block major: (kb, nb)
      *x = kCK * (c / 4);
      *y = kCRows * (c % 4);
      return &m.in_proj;
    }
    c -= 12;
  }
  *x = 0;
  if (c < 12) {
    *y = kCRows * c;
    return &m.qkv;
  }
  c -= 12;
  if (c < 4) {
    *y = kCRows * c;
    return &m.o;
  }
  c -= 4;
  if (c < 16) {
    *y = kCRows * c;
    return &m.ffn1;
  }
  c -= 16;
  if (c < 16) {  // FFN2, K-block major
    *x = kCK * (c / 4);
    *y = kCRows * (c % 4);
    return &m.ffn2;
  }
  c -= 16;
  *y = p * kVocab + kCRows * c;  // the last chunk overhangs into head p+1 (or zero fill): ignored
  return &m.head;
}

__device__ void producer(TileSmem& sm, const TileMaps& maps, bool folded) {
  int it = 0;
  for (int p = 0; p < kPositions; ++p) {
    const int n = chunks_in_position(folded, p);
    for (int c = 0; c < n; ++c, ++it) {
      const int slot = it % kSlots;
      if (it >= kSlots && !mbar_wait(&sm.empty[slot], ((it / kSlots) - 1) & 1)) sm.err = 1;
      if (err_flag(sm)) return;
      int x, y;
      const CUtensorMap* map = chunk_origin(maps, folded, p, c, &x, &y);
      fence_proxy_async();
      mbar_expect_tx(&sm.full[slot], kCBytes);
#pragma unroll
      for (int b = 0; b < kCK / kCPanel; ++b) {
        tma_load_2d(sm.ring[slot] + b * (kCRows * kCPanel), map, x + b * kCPanel, y, &sm.full[slot]);
      }
      sm.last_issued[slot] = it;
    }
  }
}

__device__ __forceinline__ const bf16* acquire(TileSmem& sm, int it) {
  const int slot = it % kSlots;
  if (err_flag(sm) == 0 && !mbar_wait(&sm.full[slot], (it / kSlots) & 1)) sm.err = 1;
  return sm.ring[slot];
}

__device__ __forceinline__ void release(TileSmem& sm, int it) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.empty[it % kSlots]);
}

// A fragments of the 16 x 256 operand at A (row stride lda) for 16 k-steps.
__device__ __forceinline__ void load_a(uint32_t (&a)[16][4], const bf16* A, int lda) {
  const int lane = threadIdx.x & 31;
  const bf16* p = A + ((lane & 7) + 8 * ((lane >> 3) & 1)) * lda + 8 * (lane >> 4);
#pragma unroll
  for (int ks = 0; ks < 16; ++ks) ldsm_x4(a[ks], p + 16 * ks);
}

// c[j] += A[16][256] x chunk rows [8w, 8w+8)^T for warp w, k-steps j mod CH in
// chain j.  The chunk is four 64-column panels of 64 rows x 128 bytes;
// 16-byte unit j of row n sits at unit j ^ (n & 7) (128-byte swizzle).
template <int CH>
__device__ __forceinline__ void mma_chunk(float (&c)[CH][4], const uint32_t (&a)[16][4], const bf16* chunk) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = 8 * warp + (lane & 7);
  const int q = lane >> 3;
  const bf16* row = chunk + n * kCPanel;
  const int swz = n & 7;
#pragma unroll
  for (int ks2 = 0; ks2 < 8; ++ks2) {
    uint32_t b[4];
    ldsm_x4(b, row + (ks2 >> 1) * (kCRows * kCPanel) + (((4 * (ks2 & 1) + q) ^ swz) << 3));
    mma16816(c[(2 * ks2) % CH], a[2 * ks2], b[0], b[1]);
    mma16816(c[(2 * ks2 + 1) % CH], a[2 * ks2 + 1], b[2], b[3]);
  }
}

// C[16][64 nb_count] = A[16][256] W^T over nb_count chunks; epi(nb, acc) per
// chunk, one chunk behind the MMAs.
template <typename Epi>
__device__ __forceinline__ void gemm_n(TileSmem& sm, int& it, const uint32_t (&a)[16][4], int nb_count, Epi epi) {
  float prev[4][4];
  for (int nb = 0; nb < nb_count; ++nb, ++it) {
    const bf16* chunk = acquire(sm, it);
    float cur[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) cur[j][0] = cur[j][1] = cur[j][2] = cur[j][3] = 0.f;
    mma_chunk<4>(cur, a, chunk);
    release(sm, it);
    if (nb > 0) {
      float acc[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = (prev[0][e] + prev[1][e]) + (prev[2][e] + prev[3][e]);
      epi(nb - 1, acc);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) prev[j][e] = cur[j][e];
  }
  float acc[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) acc[e] = (prev[0][e] + prev[1][e]) + (prev[2][e] + prev[3][e]);
  epi(nb_count - 1, acc);
}

// C[16][256] = A[16][256 KB] W^T, chunks in K-block-major order; epi(nb, acc) at the end.
template <int KB, typename Epi>
__device__ __forceinline__ void gemm_k(TileSmem& sm, int& it, const bf16* A, int lda, Epi epi) {
  float c[4][2][4];
#pragma unroll
  for (int nb = 0; nb < 4; ++nb)
#pragma unroll
    for (int j = 0; j < 2; ++j) c[nb][j][0] = c[nb][j][1] = c[nb][j][2] = c[nb][j][3] = 0.f;
  for (int kb = 0; kb < KB; ++kb) {
    uint32_t a[16][4];
    load_a(a, A + kCK * kb, lda);
#pragma unroll
    for (int nb = 0; nb < 4; ++nb, ++it) {
      const bf16* chunk = acquire(sm, it);
      mma_chunk<2>(c[nb], a, chunk);
      release(sm, it);
    }
  }
#pragma unroll
  for (int nb = 0; nb < 4; ++nb) {
    float acc[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = c[nb][0][e] + c[nb][1][e];
    epi(nb, acc);
  }
}

// LayerNorm (no bias, eps 1e-5) of the 16 rows of x into xa with this lane's
// 8 weights g (columns 8 lane ..); warp w: rows 2w, 2w+1.
__device__ __forceinline__ void layer_norm_rows(const bf16* x, bf16* xa, const float (&g)[8]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = 2 * warp + rr;
    float v[8];
    unpack8(*reinterpret_cast<const uint4*>(x + r * kLdX + lane * 8), v);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += v[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(kTD);
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) var += (v[j] - mean) * (v[j] - mean);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    const float rstd = 1.0f / sqrtf(var / static_cast<float>(kTD) + 1.0e-5f);
    float out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = ((v[j] - mean) * rstd) * g[j];
    *reinterpret_cast<uint4*>(xa + r * kLdX + lane * 8) = pack8(out);
  }
}

// ---------------------------------------------------------------------------
// attention over the TMEM KV cache: warp w, head h = w % 4, part = w / 4
// (positions j = part, part + 2, ..); thread t: row t / 2, dims [32 (t % 2), +32)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void attention(TileSmem& sm, int p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = warp & 3, part = warp >> 2;
  const int r = lane >> 1, half = lane & 1;
  const uint32_t tl = sm.tmem + (static_cast<uint32_t>(32 * h) << 16);
  const bf16* qrow = sm.u.qkv + r * kLdQkv + kHeadDim * h + 32 * half;
  {  // append k (part 0) or v (part 1) of position p
    uint32_t kv[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 t = *reinterpret_cast<const uint4*>(qrow + (1 + part) * kTD + 8 * j);
      kv[4 * j] = t.x;
      kv[4 * j + 1] = t.y;
      kv[4 * j + 2] = t.z;
      kv[4 * j + 3] = t.w;
    }
    tmem_st16(tl + 256 * part + 16 * tmem_block(p), kv);
    tmem_wait_st();
  }
  float q[32];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float f8[8];
    unpack8(*reinterpret_cast<const uint4*>(qrow + 8 * j), f8);
#pragma unroll
    for (int e = 0; e < 8; ++e) q[8 * j + e] = f8[e];
  }
  tmem_fence_before_sync();
  cbar();  // k_p and v_p in TMEM; q/k/v staging free for the exchange
  tmem_fence_after_sync();

  // scores of this part's positions j = 2m + part (m = 0..7), four per TMEM load
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
          dot = fmaf(q[2 * e], t.x, dot);
          dot = fmaf(q[2 * e + 1], t.y, dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        if (2 * (4 * g4 + jj) + part <= p) s[4 * g4 + jj] = round_bf16(__fmul_rn(round_bf16(dot), 0.125f));
      }
    }
  }
  float* my_s = sm.u.att.s[part][h][lane];
#pragma unroll
  for (int m = 0; m < 8; ++m) my_s[m] = s[m];
  cbar();
  // the full softmax over positions 0..p (both parts compute it)
  float all[kPositions];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    all[2 * m] = sm.u.att.s[0][h][lane][m];
    all[2 * m + 1] = sm.u.att.s[1][h][lane][m];
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
    float* dst = sm.u.att.o[h][lane];
#pragma unroll
    for (int d = 0; d < 32; ++d) dst[d] = o[d];
  }
  cbar();
  if (part == 0) {
    const float* src = sm.u.att.o[h][lane];
#pragma unroll
    for (int d = 0; d < 32; ++d) o[d] += src[d];
    bf16* out = sm.xa + r * kLdX + kHeadDim * h + 32 * half;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float f8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f8[e] = o[8 * j + e];
      *reinterpret_cast<uint4*>(out + 8 * j) = pack8(f8);
    }
  }
}

constexpr int kListStride = (kTRows * kLdX) / kTSess;  // 528 u16 per session slot in xa
static_assert(kListStride >= kListCap + 1, "candidate list");

__device__ __forceinline__ int sample_slot(TileSmem& sm, const Frame& f, int slot, int* invalid_out) {
  RowSample rs;
  rs.vals = sm.u.val + slot * kVocab;
  rs.flags = sm.flags[slot];
  rs.nonfinite = sm.nonfinite[slot] != 0;
  rs.seed = sm.seed[slot];
  rs.counter = sm.ctr[slot];
  return sample_row(rs, f.prm, reinterpret_cast<uint16_t*>(sm.xa) + slot * kListStride,
                    reinterpret_cast<uint16_t*>(sm.hist[slot]), invalid_out);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

__device__ __forceinline__ int64_t tile_input_token(const Frame& f, const TileSmem& sm, int slot, int p) {
  if (f.forced) {
    const int64_t t = f.forced[static_cast<int64_t>(sm.sess[slot]) * kPositions + p];
    return t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
  }
  return sm.tok[slot][p];
}

__global__ void __launch_bounds__(kTThreads, 1) tile_frame_kernel(Frame f, const __grid_constant__ TileMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t pad = (1024u - (smem_addr(smem_raw) & 1023u)) & 1023u;
  TileSmem& sm = *reinterpret_cast<TileSmem*>(smem_raw + pad);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rp = f.rp;
  const bool folded = f.emb_proj != nullptr;

  // ---- sessions [8 tile, +8) of the active list
  if (warp == 0) {
    int seen = 0;
    const int first = kTSess * static_cast<int>(blockIdx.x);
    for (int base = 0; base < f.n; base += 32) {
      const int s = base + lane;
      const bool act = s < f.n && (f.active == nullptr || f.active[s]);
      const unsigned m = __ballot_sync(0xffffffffu, act);
      const int rank = seen + __popc(m & ((1u << lane) - 1u));
      if (act && rank >= first && rank < first + kTSess) sm.sess[rank - first] = s;
      seen += __popc(m);
    }
    if (lane == 0) {
      const int left = seen - first;
      sm.n_sess = left <= 0 ? 0 : (left < kTSess ? left : kTSess);
      sm.err = 0;
    }
  }
  __syncthreads();
  const int n_sess = sm.n_sess;
  if (n_sess == 0) return;
  // row r belongs to session slot r % 8 (sub-row r / 8); live iff that slot is and r / 8 < rp
  auto live = [&](int r) { return (r & 7) < n_sess && (r >> 3) < rp; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kTWarps);
      sm.last_issued[s] = -1;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(&sm.tmem, kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x < n_sess) {  // per-session state and EOS registration
    const int s = threadIdx.x;
    const int sid = sm.sess[s];
    sm.ctr[s] = f.counter_io[sid];
    sm.seed[s] = f.seed[sid];
    sm.flags[s] = (f.unfinished[sid] ? 1u : 0u) | (f.finished[sid] ? 2u : 0u) | (f.forbid[sid] ? 4u : 0u);
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

  if (warp >= kTWarps) {  // producer warpgroup
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == kTWarps && lane == 0) producer(sm, maps, folded);
    return;  // its copies complete on the full barriers, which the consumers wait for
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
  {
    // per-thread constants: LN weights of columns [8 lane, +8); the session
    // whose rows this thread holds in mma.sync fragments (slot lane / 4)
    float g1[8], g2[8];
    unpack8(*reinterpret_cast<const uint4*>(f.ln1 + lane * 8), g1);
    unpack8(*reinterpret_cast<const uint4*>(f.ln2 + lane * 8), g2);
    const int my_slot = lane >> 2;
    const bool my_live = my_slot < n_sess;
    int it = 0;
    for (int p = 0; p < kPositions; ++p) {
      // ---------------- input rows (folded p >= 1: written by the sampling warps)
      if (has_in_projection(folded, p)) {
        for (int i = threadIdx.x; i < kTRows * (kEmbed / 8); i += kTConsumers) {
          const int r = i / (kEmbed / 8), ch = i % (kEmbed / 8);
          uint4 v = make_uint4(0, 0, 0, 0);
          if (live(r)) {
            const int slot = r & 7, sub = r >> 3;
            const bf16* src;
            if (p == 0) {
              src = f.hidden + (static_cast<int64_t>(sm.sess[slot]) * rp + sub) * kEmbed;
            } else {
              src = f.emb + (static_cast<int64_t>(p - 1) * kVocab + tile_input_token(f, sm, slot, p - 1)) * kEmbed;
            }
            v = *reinterpret_cast<const uint4*>(src + ch * 8);
          }
          *reinterpret_cast<uint4*>(sm.u.src + r * kLdSrc + ch * 8) = v;
        }
        cbar();
        const bf16* pos = f.pos + static_cast<int64_t>(p) * kTD;
        gemm_k<3>(sm, it, sm.u.src, kLdSrc, [&](int nb, const float (&acc)[4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
          const float b0 = bf2f(f.in_b[n]), b1 = bf2f(f.in_b[n + 1]);
          const float q0 = bf2f(pos[n]), q1 = bf2f(pos[n + 1]);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int r = (lane >> 2) + 8 * hh;
            const float y0 = round_bf16(__fadd_rn(acc[2 * hh], b0));
            const float y1 = round_bf16(__fadd_rn(acc[2 * hh + 1], b1));
            *reinterpret_cast<uint32_t*>(sm.x + r * kLdX + n) = pack_bf16x2(__fadd_rn(y0, q0), __fadd_rn(y1, q1));
          }
        });
      }
      // head p bias; per-position sampling state (the histograms are zeroed per use)
      {
        const bf16* hb = f.head_b + static_cast<int64_t>(p) * kVocab;
        if (threadIdx.x < kVocabChunks) {
          *reinterpret_cast<uint4*>(sm.hb + 8 * threadIdx.x) = *reinterpret_cast<const uint4*>(hb + 8 * threadIdx.x);
        }
        if (threadIdx.x < kTSess) sm.nonfinite[threadIdx.x] = 0;
      }
      cbar();

      // ---------------- LN1, qkv
      layer_norm_rows(sm.x, sm.xa, g1);
      cbar();
      {
        uint32_t a[16][4];
        load_a(a, sm.xa, kLdX);
        gemm_n(sm, it, a, 12, [&](int nb, const float (&acc)[4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
          const int r = lane >> 2;
          *reinterpret_cast<uint32_t*>(sm.u.qkv + r * kLdQkv + n) = pack_bf16x2(acc[0], acc[1]);
          *reinterpret_cast<uint32_t*>(sm.u.qkv + (r + 8) * kLdQkv + n) = pack_bf16x2(acc[2], acc[3]);
        });
      }
      cbar();

      // ---------------- KV append + attention
      attention(sm, p);
      cbar();

      // ---------------- o-projection + residual
      {
        uint32_t a[16][4];
        load_a(a, sm.xa, kLdX);
        gemm_n(sm, it, a, 4, [&](int nb, const float (&acc)[4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            bf16* xr = sm.x + ((lane >> 2) + 8 * hh) * kLdX + n;
            *reinterpret_cast<uint32_t*>(xr) = pack_bf16x2(__fadd_rn(bf2f(xr[0]), round_bf16(acc[2 * hh])),
                                                           __fadd_rn(bf2f(xr[1]), round_bf16(acc[2 * hh + 1])));
          }
        });
      }
      cbar();

      // ---------------- LN2, FFN1 + GELU
      layer_norm_rows(sm.x, sm.xa, g2);
      cbar();
      {
        uint32_t a[16][4];
        load_a(a, sm.xa, kLdX);
        gemm_n(sm, it, a, 16, [&](int nb, const float (&acc)[4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            *reinterpret_cast<uint32_t*>(sm.u.hid + ((lane >> 2) + 8 * hh) * kLdHid + n) =
                pack_bf16x2(gelu_tanh(round_bf16(acc[2 * hh])), gelu_tanh(round_bf16(acc[2 * hh + 1])));
          }
        });
      }
      cbar();

      // ---------------- FFN2 + residual
      gemm_k<4>(sm, it, sm.u.hid, kLdHid, [&](int nb, const float (&acc)[4]) {
        const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          bf16* xr = sm.x + ((lane >> 2) + 8 * hh) * kLdX + n;
          *reinterpret_cast<uint32_t*>(xr) = pack_bf16x2(__fadd_rn(bf2f(xr[0]), round_bf16(acc[2 * hh])),
                                                         __fadd_rn(bf2f(xr[1]), round_bf16(acc[2 * hh + 1])));
        }
      });
      cbar();

      // ---------------- head p: bias, CFG combine and constraints in the epilogue
      {
        uint32_t a[16][4];
        load_a(a, sm.x, kLdX);
        bool nf = false;
        uint16_t* vals = sm.u.val + my_slot * kVocab;
        const bool cfg = rp == 2;
        const float cfg_scale = f.prm.cfg_scale, uncond_scale = __fsub_rn(1.0f, f.prm.cfg_scale);
        const uint32_t my_flags = my_live ? sm.flags[my_slot] : 0u;
        bf16* lo_row = (f.logits_out && my_live)
                           ? f.logits_out + (static_cast<int64_t>(sm.sess[my_slot]) * kPositions + p) * rp * kVocab
                           : nullptr;
        gemm_n(sm, it, a, 32, [&](int nb, const float (&acc)[4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
          if (n < kVocab && my_live) {  // n is even and kVocab is even: the pair stays inside
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sm.hb + n));
            const uint32_t c2 = pack2_rn(__fadd_rn(acc[0], b.x), __fadd_rn(acc[1], b.y));
            const uint32_t u2 = pack2_rn(__fadd_rn(acc[2], b.x), __fadd_rn(acc[3], b.y));
            if (lo_row) {
              *reinterpret_cast<uint32_t*>(lo_row + n) = c2;
              if (cfg) *reinterpret_cast<uint32_t*>(lo_row + kVocab + n) = u2;
            }
            const uint32_t g = cfg ? guided_value2(c2, u2, cfg_scale, uncond_scale) : c2;
            *reinterpret_cast<uint32_t*>(vals + n) = constrain2(g, n, my_flags, nf);
          }
        });
        if (nf) atomicOr(&sm.nonfinite[my_slot], 1u);
      }
      cbar();

      // ---------------- sampling: warp w takes session slot w, then writes the
      // session's next input rows (folded tables)
      if (warp < n_sess) {
        const int slot = warp;
        int invalid = 0;
        const int token = sample_slot(sm, f, slot, &invalid);
        const int64_t counter = sm.ctr[slot];
        __syncwarp();
        if (lane == 0) {
          sm.tok[slot][p] = token;
          sm.inv[slot] |= invalid;
          const bool counter_valid = counter >= 0 && counter <= kMaxCounter;
          if (!f.prm.argmax && counter_valid) sm.ctr[slot] = counter + 1;
        }
        if (folded && p + 1 < kPositions) {
          int64_t tin = token;
          if (f.forced) {
            const int64_t t = f.forced[static_cast<int64_t>(sm.sess[slot]) * kPositions + p];
            tin = t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
          }
          float e8[8], p8[8];
          unpack8(*reinterpret_cast<const uint4*>(f.emb_proj + (static_cast<int64_t>(p) * kVocab + tin) * kTD + lane * 8),
                  e8);
          unpack8(*reinterpret_cast<const uint4*>(f.pos + static_cast<int64_t>(p + 1) * kTD + lane * 8), p8);
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = __fadd_rn(e8[e], p8[e]);
          const uint4 row = pack8(y);
          *reinterpret_cast<uint4*>(sm.x + slot * kLdX + lane * 8) = row;
          if (rp == 2) *reinterpret_cast<uint4*>(sm.x + (slot + 8) * kLdX + lane * 8) = row;
        }
      }
      cbar();
    }
  }

  // ---- drain: no TMA copy may still be writing when the CTA leaves
  cbar();
  if (threadIdx.x == 0 && sm.err) {
    for (int s = 0; s < kSlots; ++s) {
      const int last = sm.last_issued[s];
      if (last >= 0) mbar_wait(&sm.full[s], (last / kSlots) & 1);
    }
  }

  // ---- commit: tokens, counters, flags, next-frame embedding
  for (int i = threadIdx.x; i < n_sess * kPositions; i += kTConsumers) {
    const int slot = i / kPositions, pp = i % kPositions;
    const int sid = sm.sess[slot];
    const int32_t t = sm.tok[slot][pp];
    f.codec_tokens[codec_index(f, sid, pp)] = t;
    f.tokens[static_cast<int64_t>(sid) * kPositions + pp] = t;
  }
  if (threadIdx.x < n_sess) {
    const int slot = threadIdx.x;
    const int sid = sm.sess[slot];
    f.counter_io[sid] = sm.ctr[slot];
    f.invalid_rows[sid] = sm.inv[slot] | (sm.err ? 4 : 0);
    if (f.eos_slot[sid] < 0) commit_end(f, sid, f.finished[sid] ? 0 : -1);
  }
  // sum_p table_p[token_p], each add rounded to bf16, in position order; / 16
  for (int i = threadIdx.x; i < n_sess * (kEmbed / 8); i += kTConsumers) {
    const int slot = i / (kEmbed / 8), k8 = 8 * (i % (kEmbed / 8));
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

  tmem_fence_before_sync();
  cbar();
  if (warp == 0) {
    tmem_fence_after_sync();
    tmem_dealloc(sm.tmem, kTmemCols);
  }
}

}  // namespace

bool tile_frame_supported(const Frame& f) {
  if (f.d != kTD || f.H != kTHeads || f.F != kTF || f.L != 1 || !f.in_proj || (f.rp != 1 && f.rp != 2)) return false;
  static PerDeviceInt cache;  // the opt-in below is per device context
  return cache.get([] {
    int ok = 0;
    if (cudaFuncSetAttribute(tile_frame_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kTSmemBytes)) == cudaSuccess) {
      int blocks = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, tile_frame_kernel, kTThreads, kTSmemBytes) ==
              cudaSuccess &&
          blocks == 1) {
        ok = 1;
      }
    }
    cudaGetLastError();
    return ok;
  }) == 1;
}

int tile_frame_clusters() {
  Frame probe{};
  probe.d = kTD;
  probe.H = kTHeads;
  probe.F = kTF;
  probe.L = 1;
  probe.in_proj = 1;
  probe.rp = 2;
  if (!tile_frame_supported(probe)) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return sms;  // one CTA per SM
}

cudaError_t launch_tile_frame(const Frame& f, cudaStream_t stream) {
  TileMaps maps;
  if (!make_weight_map(&maps.in_proj, f.in_w, kEmbed, kTD, kCRows) ||
      !make_weight_map(&maps.qkv, f.qkv, kTD, 3 * kTD, kCRows) || !make_weight_map(&maps.o, f.o, kTD, kTD, kCRows) ||
      !make_weight_map(&maps.ffn1, f.w1, kTD, kTF, kCRows) || !make_weight_map(&maps.ffn2, f.w2, kTF, kTD, kCRows) ||
      !make_weight_map(&maps.head, f.head_w, kTD, static_cast<uint64_t>(kPositions) * kVocab, kCRows)) {
    return cudaErrorInvalidValue;
  }
  const int tiles = (f.n + kTSess - 1) / kTSess;
  cudaError_t e = cudaMemsetAsync(f.eos_count, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  tile_frame_kernel<<<tiles, kTThreads, kTSmemBytes, stream>>>(f, maps);
  return launch_frame_eos(f, stream);
}

}  // namespace mtt
