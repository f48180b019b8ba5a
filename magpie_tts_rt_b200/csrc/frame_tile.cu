// Tile frame kernel: one CTA runs all 16 positions of a Local AR frame for a
// tile of 16 rows (8 sessions x CFG pair, or 16 sessions without CFG), with
// no communication between CTAs.  This is the throughput path: at a few
// hundred sessions per GPU every SM holds its own tile, and the per-position
// critical path is the weight stream through the SM, not a cluster exchange.
//
// Per position (reference ops as in frame_fused.cu: local_ar_wrapper.py:609-751,
// transformer_2501.py:405-442,761-851,1153-1232, sampling
// local_ar_plugins.cu:1211-1370, embedding sum main_decoder_wrapper.py:796-810):
//
//   in-projection (p = 0, or every p without the folded tables) or the folded
//   gather x = bf16(emb_proj[p-1][token] + pos[p]); LN1; qkv; k/v appended
//   to the KV cache in tensor memory; causal attention over positions 0..p;
//   o-projection + residual; LN2; FFN1 + GELU-tanh; FFN2 + residual; head p
//   (+bias, CFG combine in the epilogue); one warp samples each session.
//
// Data layout:
//   * Weights stream from global memory (L2-resident across frames) through a
//     four-slot ring of 32 KB chunks (64 weight rows x 256 K columns, four
//     TMA boxes of 64 x 64 with 128-byte swizzle, no multicast), filled by a
//     dedicated producer warp that runs ahead of the eight consumer warps;
//     full/empty mbarriers per slot.  Every GEMM is C[16][N] = A[16][K] W^T on
//     mma.sync m16n8k16 (bf16 in, f32 accumulate): at 16 rows this is a
//     weight-streaming GEMV, below tcgen05's 64-row minimum.  A (the 16 rows)
//     is held in registers for a whole GEMM; each warp reads its 8 weight rows
//     of a chunk with ldmatrix exactly once.
//   * The KV cache (16 rows x 16 positions x (256 k + 256 v) bf16 = 256 KB)
//     lives in tensor memory: TMEM lane 32h + 2r + half holds, for row r and
//     head h, dims [32 half, +32) of k_j at columns [16j, +16) and of v_j at
//     columns [256 + 16j, +16) (bf16 pairs).  Warp h (h < 4) owns TMEM lanes
//     [32h, +32) and computes head h's attention for all 16 rows.
//   * Rows: row r is slot r % S, sub-row r / S (S = 16 / rows per session),
//     so with CFG the conditional and unconditional rows of a session are rows
//     s and s + 8, which one mma.sync thread holds together in the head
//     epilogue (the CFG combine needs no exchange).
// Every wait is bounded; a timeout sets invalid bit 4 for the tile's sessions.
#include <cuda.h>

#include <mutex>

#include "frame_common.cuh"
#include "ptx.cuh"

namespace mtt {
namespace {

constexpr int kTRows = 16;
constexpr int kTWarps = 8;                   // consumer warps
constexpr int kTConsumers = kTWarps * 32;    // 256
constexpr int kTThreads = kTConsumers + 32;  // + the TMA producer warp
constexpr int kTD = 256;
constexpr int kTF = 1024;
constexpr int kTHeads = 4;
constexpr int kCRows = 64;                      // weight rows per chunk
constexpr int kCK = 256;                        // K columns per chunk
constexpr int kCPanel = 64;                     // columns per TMA box (128 bytes)
constexpr int kCElems = kCRows * kCK;           // 16384 bf16
constexpr uint32_t kCBytes = kCElems * 2;       // 32 KB
constexpr int kSlots = 4;
constexpr int kLdX = kTD + 8;       // 264
constexpr int kLdSrc = kEmbed + 8;  // 776
constexpr int kLdQkv = 3 * kTD + 8; // 776
constexpr int kLdHid = kTF + 8;     // 1032
constexpr int kElig = 256;          // per-warp eligible-token list
constexpr int kTmemCols = 512;
constexpr int kVocabChunks = kVocab / 8;  // 253 chunks of 8 logits per session row

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

// Buffers of phases that never overlap within a position.
union TileU {
  bf16 src[kTRows * kLdSrc];  // in-projection input rows
  bf16 qkv[kTRows * kLdQkv];  // q | k | v of the current position
  bf16 hid[kTRows * kLdHid];  // FFN1 output
  bf16 g[kTRows * kVocab];    // guided (or plain) logits, one row per session slot
};

struct __align__(1024) TileSmem {
  bf16 ring[kSlots][kCElems];  // 1024-byte aligned panels (128-byte swizzle atoms)
  bf16 x[kTRows * kLdX];       // residual stream
  bf16 xa[kTRows * kLdX];      // LN output / attention output
  TileU u;
  uint32_t hist[kTWarps][256];
  uint16_t elig[kTWarps][kElig];
  int32_t tok[kTRows][kPositions];
  int32_t sess[kTRows];
  int64_t ctr[kTRows];
  int32_t inv[kTRows];
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

// acc += A[16][256] x chunk rows [8w, 8w+8)^T for warp w.  The chunk is four
// 64-column panels of 64 rows x 128 bytes; 16-byte unit j of row n sits at
// unit j ^ (n & 7) (128-byte swizzle).
__device__ __forceinline__ void mma_chunk(float (&acc)[4], const uint32_t (&a)[16][4], const bf16* chunk) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = 8 * warp + (lane & 7);
  const int q = lane >> 3;
  const bf16* row = chunk + n * kCPanel;
  const int swz = n & 7;
  float odd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ks2 = 0; ks2 < 8; ++ks2) {
    uint32_t b[4];
    ldsm_x4(b, row + (ks2 >> 1) * (kCRows * kCPanel) + (((4 * (ks2 & 1) + q) ^ swz) << 3));
    mma16816(acc, a[2 * ks2], b[0], b[1]);
    mma16816(odd, a[2 * ks2 + 1], b[2], b[3]);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) acc[e] += odd[e];
}

// C[16][64 nb_count] = A[16][256] W^T over nb_count chunks; epi(nb, acc) per chunk.
template <typename Epi>
__device__ __forceinline__ void gemm_n(TileSmem& sm, int& it, const bf16* A, int lda, int nb_count, Epi epi) {
  uint32_t a[16][4];
  load_a(a, A, lda);
  for (int nb = 0; nb < nb_count; ++nb, ++it) {
    const bf16* chunk = acquire(sm, it);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    mma_chunk(acc, a, chunk);
    release(sm, it);
    epi(nb, acc);
  }
}

// C[16][256] = A[16][256 KB] W^T, chunks in K-block-major order; epi(nb, acc) at the end.
template <int KB, typename Epi>
__device__ __forceinline__ void gemm_k(TileSmem& sm, int& it, const bf16* A, int lda, Epi epi) {
  float acc[4][4];
#pragma unroll
  for (int nb = 0; nb < 4; ++nb) acc[nb][0] = acc[nb][1] = acc[nb][2] = acc[nb][3] = 0.f;
  for (int kb = 0; kb < KB; ++kb) {
    uint32_t a[16][4];
    load_a(a, A + kCK * kb, lda);
#pragma unroll
    for (int nb = 0; nb < 4; ++nb, ++it) {
      const bf16* chunk = acquire(sm, it);
      mma_chunk(acc[nb], a, chunk);
      release(sm, it);
    }
  }
#pragma unroll
  for (int nb = 0; nb < 4; ++nb) epi(nb, acc[nb]);
}

// LayerNorm (no bias, eps 1e-5) of the 16 rows of x into xa; warp w: rows 2w, 2w+1.
__device__ __forceinline__ void layer_norm_rows(const bf16* x, bf16* xa, const bf16* w) {
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
    const uint4 xv = *reinterpret_cast<const uint4*>(x + r * kLdX + lane * 8);
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
    const float mean = sum / static_cast<float>(kTD);
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) var += (v[j] - mean) * (v[j] - mean);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    const float rstd = 1.0f / sqrtf(var / static_cast<float>(kTD) + 1.0e-5f);
    __align__(16) bf16 out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = f2bf(((v[j] - mean) * rstd) * g[j]);
    *reinterpret_cast<uint4*>(xa + r * kLdX + lane * 8) = *reinterpret_cast<const uint4*>(out);
  }
}

__device__ __forceinline__ float gelu_tanh(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

// ---------------------------------------------------------------------------
// attention over the TMEM KV cache (warp h < 4: head h, thread t: row t / 2,
// dims [32 (t % 2), +32) of the head)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void attention_warp(TileSmem& sm, int p) {
  const int lane = threadIdx.x & 31, h = threadIdx.x >> 5;
  const int r = lane >> 1, half = lane & 1;
  const uint32_t tl = sm.tmem + (static_cast<uint32_t>(32 * h) << 16);
  const bf16* qrow = sm.u.qkv + r * kLdQkv + kHeadDim * h + 32 * half;
  {
    uint32_t kv[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 t = *reinterpret_cast<const uint4*>(qrow + kTD + 8 * j);
      kv[4 * j] = t.x;
      kv[4 * j + 1] = t.y;
      kv[4 * j + 2] = t.z;
      kv[4 * j + 3] = t.w;
    }
    tmem_st16(tl + 16 * p, kv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 t = *reinterpret_cast<const uint4*>(qrow + 2 * kTD + 8 * j);
      kv[4 * j] = t.x;
      kv[4 * j + 1] = t.y;
      kv[4 * j + 2] = t.z;
      kv[4 * j + 3] = t.w;
    }
    tmem_st16(tl + 256 + 16 * p, kv);
    tmem_wait_st();
  }
  float q[32];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(qrow + 8 * j), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) q[8 * j + e] = f[e];
  }
  float s[kPositions];
#pragma unroll
  for (int j = 0; j < kPositions; ++j) {
    s[j] = -CUDART_INF_F;
    if (j <= p) {
      uint32_t k[16];
      tmem_ld16(k, tl + 16 * j);
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&k[e]));
        dot = fmaf(q[2 * e], t.x, dot);
        dot = fmaf(q[2 * e + 1], t.y, dot);
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      s[j] = round_bf16(__fmul_rn(round_bf16(dot), 0.125f));
    }
  }
  float mx = s[0];
#pragma unroll
  for (int j = 1; j < kPositions; ++j) mx = fmaxf(mx, s[j]);
  float e[kPositions];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPositions; ++j) {
    e[j] = j <= p ? expf(s[j] - mx) : 0.f;
    sum += e[j];
  }
  float o[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) o[d] = 0.f;
#pragma unroll
  for (int j = 0; j < kPositions; ++j) {
    if (j <= p) {
      const float prob = round_bf16(e[j] / sum);
      uint32_t v[16];
      tmem_ld16(v, tl + 256 + 16 * j);
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v[d]));
        o[2 * d] = fmaf(prob, t.x, o[2 * d]);
        o[2 * d + 1] = fmaf(prob, t.y, o[2 * d + 1]);
      }
    }
  }
  bf16* out = sm.xa + r * kLdX + kHeadDim * h + 32 * half;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(o[8 * j], o[8 * j + 1]);
    u.y = pack_bf16x2(o[8 * j + 2], o[8 * j + 3]);
    u.z = pack_bf16x2(o[8 * j + 4], o[8 * j + 5]);
    u.w = pack_bf16x2(o[8 * j + 6], o[8 * j + 7]);
    *reinterpret_cast<uint4*>(out + 8 * j) = u;
  }
}

// ---------------------------------------------------------------------------
// warp sampler: one (session, position) call on a row of 2024 bf16 logits
// (CFG already combined) in shared memory.  Same contract as sample_block in
// sampling.cuh; lane l holds tokens [8c, 8c+8) for c = l + 32i.
// ---------------------------------------------------------------------------

constexpr uint32_t kKeyNegInf = 0x007fu;  // 16-bit order key of bf16 -inf

// Order key of a bf16 bit pattern with -0 folded onto +0 (key order == float order).
__device__ __forceinline__ uint32_t sample_key(uint32_t b) {
  b = (b == 0x8000u) ? 0u : b;
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

struct WarpSample {
  const bf16* g;
  bool unfinished, finished, forbid_eos;
  int64_t seed, counter;
};

__device__ __forceinline__ uint32_t warp_count_ge(const uint32_t (&kp)[8][4], uint32_t t) {
  const int lane = threadIdx.x & 31;
  uint32_t c = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (lane + 32 * i < kVocabChunks) {
#pragma unroll
      for (int e = 0; e < 4; ++e) c += ((kp[i][e] & 0xffffu) >= t) + ((kp[i][e] >> 16) >= t);
    }
  }
  return __reduce_add_sync(0xffffffffu, c);
}

__device__ int warp_sample(const WarpSample& a, const SamplingParams& prm, uint32_t* hist, uint16_t* elig,
                           int* invalid_out) {
  const int lane = threadIdx.x & 31;
  uint32_t kp[8][4];
  bool nonfinite = false;
  uint32_t mx = 0, finite = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = lane + 32 * i;
    if (c < kVocabChunks) {
      const uint4 v = *reinterpret_cast<const uint4*>(a.g + 8 * c);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint32_t key2[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int t = 8 * c + 2 * e + hh;
          uint32_t b = hh ? (w[e] >> 16) : (w[e] & 0xffffu);
          if ((b & 0x7f80u) == 0x7f80u) {
            nonfinite = true;
            b = 0xff80u;
          }
          if (t >= kCodebook && (t != kEosId || a.unfinished || a.forbid_eos)) b = 0xff80u;
          if (a.finished) b = (t == kEosId) ? 0u : 0xff80u;
          key2[hh] = sample_key(b);
          mx = key2[hh] > mx ? key2[hh] : mx;
          finite += key2[hh] != kKeyNegInf ? 1u : 0u;
        }
        kp[i][e] = key2[0] | (key2[1] << 16);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) kp[i][e] = 0;
    }
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  finite = __reduce_add_sync(0xffffffffu, finite);
  nonfinite = __any_sync(0xffffffffu, nonfinite);

  int token;
  int invalid;
  if (prm.argmax) {
    // left-most token holding the largest value
    int first = kVocab;
#pragma unroll
    for (int i = 7; i >= 0; --i) {
      const int c = lane + 32 * i;
      if (c < kVocabChunks) {
#pragma unroll
        for (int e = 3; e >= 0; --e) {
          if ((kp[i][e] >> 16) == mx) first = 8 * c + 2 * e + 1;
          if ((kp[i][e] & 0xffffu) == mx) first = 8 * c + 2 * e;
        }
      }
    }
    first = __reduce_min_sync(0xffffffffu, first);
    invalid = (nonfinite || finite == 0) ? 1 : 0;
    token = (mx == kKeyNegInf || first >= kVocab) ? 0 : first;
    if (mx == kKeyNegInf) invalid = 1;
    *invalid_out = invalid;
    return token;
  }

  // ---- k-th largest key: histogram of mx - key over the 256 keys below mx
  const uint32_t kk = static_cast<uint32_t>(prm.top_k);
#pragma unroll
  for (int i = 0; i < 8; ++i) hist[lane * 8 + i] = 0;
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (lane + 32 * i < kVocabChunks) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t d0 = mx - (kp[i][e] & 0xffffu), d1 = mx - (kp[i][e] >> 16);
        if (d0 < 256u) atomicAdd(&hist[d0], 1u);
        if (d1 < 256u) atomicAdd(&hist[d1], 1u);
      }
    }
  }
  __syncwarp();
  uint32_t cnt[8];
  uint32_t sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    cnt[j] = hist[lane * 8 + j];
    sum += cnt[j];
  }
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - sum;
  const uint32_t window_total = __shfl_sync(0xffffffffu, incl, 31);
  uint32_t thr;
  if (window_total >= kk) {
    uint32_t cand = 0;
    const bool here = excl < kk && kk <= incl;
    if (here) {
      uint32_t acc = excl;
      int j = 0;
      for (; j < 7; ++j) {
        if (kk <= acc + cnt[j]) break;
        acc += cnt[j];
      }
      cand = mx - static_cast<uint32_t>(lane * 8 + j);
    }
    const unsigned who = __ballot_sync(0xffffffffu, here);
    thr = __shfl_sync(0xffffffffu, cand, __ffs(who) - 1);
  } else {
    // exact binary search: count(key >= lo) >= k > count(key >= hi)
    uint32_t lo = kKeyNegInf, hi = mx + 1;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (warp_count_ge(kp, mid) >= kk) {
        lo = mid;
      } else {
        hi = mid;
      }
    }
    thr = lo;
  }
  __syncwarp();  // hist is reused by the next call

  invalid = (nonfinite || finite == 0) ? 1 : 0;
  if (a.unfinished && a.finished) invalid = 1;
  if (a.finished && a.forbid_eos) invalid = 1;
  const bool seed_valid = a.seed >= 0 && static_cast<uint64_t>(a.seed) < (1ull << 32);
  const bool counter_valid = a.counter >= 0 && a.counter <= kMaxCounter;
  if (!seed_valid || !counter_valid) invalid = 1;
  const uint32_t seed32 = seed_valid ? static_cast<uint32_t>(a.seed) : 0u;
  const uint64_t off64 = counter_valid ? static_cast<uint64_t>(a.counter) * kPhiloxStride : 0ull;

  // ---- finite eligible tokens (key >= thr) in token order, scored by Philox-Gumbel
  uint32_t mine = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (lane + 32 * i < kVocabChunks) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t k0 = kp[i][e] & 0xffffu, k1 = kp[i][e] >> 16;
        mine += (k0 >= thr && k0 != kKeyNegInf) + (k1 >= thr && k1 != kKeyNegInf);
      }
    }
  }
  uint32_t pos = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, pos, o);
    if (lane >= o) pos += y;
  }
  const uint32_t total = __shfl_sync(0xffffffffu, pos, 31);
  pos -= mine;

  float best = -CUDART_INF_F;
  int best_id = kVocab;
  auto score = [&](int t) {
    const float value = a.finished ? 0.0f : bf2f(a.g[t]);
    const float gm = clamped_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t)));
    const float sc = __fadd_rn(__fdiv_rn(value, prm.temperature), gm);
    if (sc > best || (sc == best && t < best_id)) {
      best = sc;
      best_id = t;
    }
  };
  if (total <= static_cast<uint32_t>(kElig)) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = lane + 32 * i;
      if (c < kVocabChunks) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t k0 = kp[i][e] & 0xffffu, k1 = kp[i][e] >> 16;
          if (k0 >= thr && k0 != kKeyNegInf) elig[pos++] = static_cast<uint16_t>(8 * c + 2 * e);
          if (k1 >= thr && k1 != kKeyNegInf) elig[pos++] = static_cast<uint16_t>(8 * c + 2 * e + 1);
        }
      }
    }
    __syncwarp();
    for (uint32_t e = lane; e < total; e += 32) score(elig[e]);
    __syncwarp();
  } else {  // many ties: every lane scores its own eligible tokens
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = lane + 32 * i;
      if (c < kVocabChunks) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t k0 = kp[i][e] & 0xffffu, k1 = kp[i][e] >> 16;
          if (k0 >= thr && k0 != kKeyNegInf) score(8 * c + 2 * e);
          if (k1 >= thr && k1 != kKeyNegInf) score(8 * c + 2 * e + 1);
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_id, o);
    if (ob > best || (ob == best && oi < best_id)) {
      best = ob;
      best_id = oi;
    }
  }
  token = best_id;
  if (token >= kVocab || best == -CUDART_INF_F) {
    invalid = 1;
    token = 0;
  }
  *invalid_out = invalid;
  return token;
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
  const int spt = kTRows / rp;  // sessions (slots) per tile
  const bool folded = f.emb_proj != nullptr;

  // ---- sessions [spt * tile, +spt) of the active list
  if (warp == 0) {
    int seen = 0;
    const int first = spt * static_cast<int>(blockIdx.x);
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
  if (n_sess == 0) return;
  // row r belongs to session slot r % spt (sub-row r / spt); it is live iff that slot is
  auto live = [&](int r) { return r % spt < n_sess; };

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

  if (warp == kTWarps) {
    if (lane == 0) producer(sm, maps, folded);
  } else {
    int it = 0;
    for (int p = 0; p < kPositions; ++p) {
      // ---------------- input rows
      if (has_in_projection(folded, p)) {
        for (int i = threadIdx.x; i < kTRows * (kEmbed / 8); i += kTConsumers) {
          const int r = i / (kEmbed / 8), ch = i % (kEmbed / 8);
          uint4 v = make_uint4(0, 0, 0, 0);
          if (live(r)) {
            const int slot = r % spt, sub = r / spt;
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
      } else {
        for (int i = threadIdx.x; i < kTRows * (kTD / 8); i += kTConsumers) {
          const int r = i / (kTD / 8), ch = i % (kTD / 8);
          uint4 out = make_uint4(0, 0, 0, 0);
          if (live(r)) {
            const int slot = r % spt;
            float e8[8], p8[8];
            unpack8(*reinterpret_cast<const uint4*>(
                        f.emb_proj + (static_cast<int64_t>(p - 1) * kVocab + tile_input_token(f, sm, slot, p - 1)) * kTD +
                        ch * 8),
                    e8);
            unpack8(*reinterpret_cast<const uint4*>(f.pos + static_cast<int64_t>(p) * kTD + ch * 8), p8);
            out.x = pack_bf16x2(__fadd_rn(e8[0], p8[0]), __fadd_rn(e8[1], p8[1]));
            out.y = pack_bf16x2(__fadd_rn(e8[2], p8[2]), __fadd_rn(e8[3], p8[3]));
            out.z = pack_bf16x2(__fadd_rn(e8[4], p8[4]), __fadd_rn(e8[5], p8[5]));
            out.w = pack_bf16x2(__fadd_rn(e8[6], p8[6]), __fadd_rn(e8[7], p8[7]));
          }
          *reinterpret_cast<uint4*>(sm.x + r * kLdX + ch * 8) = out;
        }
      }
      cbar();

      // ---------------- LN1, qkv
      layer_norm_rows(sm.x, sm.xa, f.ln1);
      cbar();
      gemm_n(sm, it, sm.xa, kLdX, 12, [&](int nb, const float (&acc)[4]) {
        const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
        const int r = lane >> 2;
        *reinterpret_cast<uint32_t*>(sm.u.qkv + r * kLdQkv + n) = pack_bf16x2(acc[0], acc[1]);
        *reinterpret_cast<uint32_t*>(sm.u.qkv + (r + 8) * kLdQkv + n) = pack_bf16x2(acc[2], acc[3]);
      });
      cbar();

      // ---------------- KV append + attention (warps 0-3, one head each)
      if (warp < kTHeads) attention_warp(sm, p);
      cbar();

      // ---------------- o-projection + residual
      gemm_n(sm, it, sm.xa, kLdX, 4, [&](int nb, const float (&acc)[4]) {
        const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          bf16* xr = sm.x + ((lane >> 2) + 8 * hh) * kLdX + n;
          *reinterpret_cast<uint32_t*>(xr) = pack_bf16x2(__fadd_rn(bf2f(xr[0]), round_bf16(acc[2 * hh])),
                                                         __fadd_rn(bf2f(xr[1]), round_bf16(acc[2 * hh + 1])));
        }
      });
      cbar();

      // ---------------- LN2, FFN1 + GELU
      layer_norm_rows(sm.x, sm.xa, f.ln2);
      cbar();
      gemm_n(sm, it, sm.xa, kLdX, 16, [&](int nb, const float (&acc)[4]) {
        const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          *reinterpret_cast<uint32_t*>(sm.u.hid + ((lane >> 2) + 8 * hh) * kLdHid + n) =
              pack_bf16x2(gelu_tanh(round_bf16(acc[2 * hh])), gelu_tanh(round_bf16(acc[2 * hh + 1])));
        }
      });
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

      // ---------------- head p (+bias), CFG combine, raw logits to the test hook
      {
        const bf16* hb = f.head_b + static_cast<int64_t>(p) * kVocab;
        gemm_n(sm, it, sm.x, kLdX, 32, [&](int nb, const float (&acc)[4]) {
          const int n = kCRows * nb + 8 * warp + 2 * (lane & 3);
          if (n < kVocab) {  // n is even and kVocab is even: the pair stays inside
            const float b0 = bf2f(hb[n]), b1 = bf2f(hb[n + 1]);
            const int r = lane >> 2;
            const bf16 c0 = f2bf(__fadd_rn(acc[0], b0)), c1 = f2bf(__fadd_rn(acc[1], b1));
            const bf16 u0 = f2bf(__fadd_rn(acc[2], b0)), u1 = f2bf(__fadd_rn(acc[3], b1));
            if (rp == 2) {
              *reinterpret_cast<uint32_t*>(sm.u.g + r * kVocab + n) =
                  pack_bf16x2(guided_logit(bf2f(c0), bf2f(u0), f.prm.cfg_scale),
                              guided_logit(bf2f(c1), bf2f(u1), f.prm.cfg_scale));
            } else {
              *reinterpret_cast<uint32_t*>(sm.u.g + r * kVocab + n) = pack_bf16x2(bf2f(c0), bf2f(c1));
              *reinterpret_cast<uint32_t*>(sm.u.g + (r + 8) * kVocab + n) = pack_bf16x2(bf2f(u0), bf2f(u1));
            }
            if (f.logits_out) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int row = r + 8 * hh;
                if (live(row)) {
                  const int slot = row % spt, sub = row / spt;
                  bf16* lo = f.logits_out +
                             ((static_cast<int64_t>(sm.sess[slot]) * kPositions + p) * rp + sub) * kVocab + n;
                  lo[0] = hh ? u0 : c0;
                  lo[1] = hh ? u1 : c1;
                }
              }
            }
          }
        });
      }
      cbar();

      // ---------------- sampling: warp w takes slots w (and w + 8 without CFG)
      for (int slot = warp; slot < n_sess; slot += kTWarps) {
        const int sid = sm.sess[slot];
        WarpSample ws;
        ws.g = sm.u.g + slot * kVocab;
        ws.unfinished = f.unfinished[sid];
        ws.finished = f.finished[sid];
        ws.forbid_eos = f.forbid[sid];
        ws.seed = f.seed[sid];
        ws.counter = sm.ctr[slot];
        int invalid = 0;
        const int token = warp_sample(ws, f.prm, sm.hist[warp], sm.elig[warp], &invalid);
        if (lane == 0) {
          sm.tok[slot][p] = token;
          sm.inv[slot] |= invalid;
          const bool counter_valid = ws.counter >= 0 && ws.counter <= kMaxCounter;
          if (!f.prm.argmax && counter_valid) sm.ctr[slot] = ws.counter + 1;
        }
      }
      cbar();
    }
  }

  // ---- drain: no TMA copy may still be writing when the CTA leaves
  __syncthreads();
  if (threadIdx.x == 0 && sm.err) {
    for (int s = 0; s < kSlots; ++s) {
      const int last = sm.last_issued[s];
      if (last >= 0) mbar_wait(&sm.full[s], (last / kSlots) & 1);
    }
  }

  // ---- commit: tokens, counters, flags, next-frame embedding
  for (int i = threadIdx.x; i < n_sess * kPositions; i += blockDim.x) {
    const int slot = i / kPositions, pp = i % kPositions;
    const int sid = sm.sess[slot];
    const int32_t t = sm.tok[slot][pp];
    f.codec_tokens[static_cast<int64_t>(sid) * kPositions + (pp % kCodebooks) * kFrames + pp / kCodebooks] = t;
    f.tokens[static_cast<int64_t>(sid) * kPositions + pp] = t;
  }
  if (threadIdx.x < n_sess) {
    const int slot = threadIdx.x;
    const int sid = sm.sess[slot];
    f.counter_io[sid] = sm.ctr[slot];
    f.invalid_rows[sid] = sm.inv[slot] | (sm.err ? 4 : 0);
    if (f.eos_slot[sid] < 0) f.end_frame[sid] = f.finished[sid] ? 0 : -1;
  }
  // sum_p table_p[token_p], each add rounded to bf16, in position order; / 16
  for (int i = threadIdx.x; i < n_sess * (kEmbed / 8); i += blockDim.x) {
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
    uint4 out;
    out.x = pack_bf16x2(__fdiv_rn(acc[0], 16.0f), __fdiv_rn(acc[1], 16.0f));
    out.y = pack_bf16x2(__fdiv_rn(acc[2], 16.0f), __fdiv_rn(acc[3], 16.0f));
    out.z = pack_bf16x2(__fdiv_rn(acc[4], 16.0f), __fdiv_rn(acc[5], 16.0f));
    out.w = pack_bf16x2(__fdiv_rn(acc[6], 16.0f), __fdiv_rn(acc[7], 16.0f));
    *reinterpret_cast<uint4*>(f.next_emb + static_cast<int64_t>(sm.sess[slot]) * kEmbed + k8) = out;
  }

  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tmem_fence_after_sync();
    tmem_dealloc(sm.tmem, kTmemCols);
  }
}

}  // namespace

bool tile_frame_supported(const Frame& f) {
  if (f.d != kTD || f.H != kTHeads || f.F != kTF || f.L != 1 || !f.in_proj || (f.rp != 1 && f.rp != 2)) return false;
  static int cached = -1;  // per process
  static std::mutex mu;
  const std::lock_guard<std::mutex> lock(mu);
  if (cached < 0) {
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
    cached = ok;
  }
  return cached == 1;
}

cudaError_t launch_tile_frame(const Frame& f, cudaStream_t stream) {
  TileMaps maps;
  if (!make_weight_map(&maps.in_proj, f.in_w, kEmbed, kTD, kCRows) ||
      !make_weight_map(&maps.qkv, f.qkv, kTD, 3 * kTD, kCRows) || !make_weight_map(&maps.o, f.o, kTD, kTD, kCRows) ||
      !make_weight_map(&maps.ffn1, f.w1, kTD, kTF, kCRows) || !make_weight_map(&maps.ffn2, f.w2, kTF, kTD, kCRows) ||
      !make_weight_map(&maps.head, f.head_w, kTD, static_cast<uint64_t>(kPositions) * kVocab, kCRows)) {
    return cudaErrorInvalidValue;
  }
  const int spt = kTRows / f.rp;
  const int tiles = (f.n + spt - 1) / spt;
  cudaError_t e = cudaMemsetAsync(f.eos_count, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  tile_frame_kernel<<<tiles, kTThreads, kTSmemBytes, stream>>>(f, maps);
  return launch_frame_eos(f, stream);
}

}  // namespace mtt
