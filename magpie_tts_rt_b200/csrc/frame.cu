// Batched Local AR frame: 16 positions of the causal Local Transformer, the
// per-position heads, sampling, EOS and the next-frame embedding sum for N
// independent sessions ("streams"), stream-ordered on one CUDA stream.
//
// Reference path being replaced (per session): the TensorRT Local AR plan
// (tools/export/local_ar_wrapper.py:609-751 is its tensor statement; NeMo
// forward: transformer_2501.py:405-442,761-851,1153-1232, ffn_modules.py:
// 268-290), its MagpieLocalARSampling / MagpieLocalAREos plugins
// (plugins/local_ar_plugins.cu:1149-1495), the Main Decoder's embedding sum
// (tools/export/main_decoder_wrapper.py:796-810) and finalize_local_step
// (src/runtime/synthesis_kernels.cu:53-86).
//
// bf16 storage, f32 accumulation, and a bf16 rounding at every point where the
// PyTorch oracle rounds (each linear/conv output, the position add, every
// residual add, LN output, GELU output, attention scores, probabilities and
// context).
//
// Phase kernels (one launch each, per position):
//   embed   : x = bf16(bf16(W_in src + b_in) + pos[p])   (src = decoder hidden
//             at p = 0, else table_{p-1}[token_{p-1}]); identity in-projection
//             shapes use a plain add
//   per layer: LN1 -> qkv (K/V appended to the per-frame cache)
//              -> attention over p + 1 keys -> o + residual
//              -> LN2 -> FFN1 + GELU -> FFN2 + residual
//   head    : logits = bf16(W_p x + b_p)
//   sample  : one block per stream (sampling.cuh), token, counter, invalid,
//             running bf16 embedding sum
// then the EOS projection (eos.cuh) and the commit of tokens / counter /
// invalid / end_frame / next embedding.
//
// Streams flagged inactive are compacted away on the device at the start of
// the frame: every kernel is sized for n streams and its blocks beyond the
// active count exit at once.
#include <cstddef>

#include <atomic>

#include "../../include/magpie_tts_rt_b200.h"
#include "eos.cuh"
#include "frame_common.cuh"
#include "gemm_tc.cuh"
#include "sampling.cuh"

namespace mtt {
namespace {

constexpr int kLinThreads = 256;
constexpr int kBM = 8;   // rows per linear tile (one warp per row in the prologue)
constexpr int kBN = 32;  // output features per linear tile
constexpr int kBeginThreads = 1024;

// ---------------------------------------------------------------------------
// frame begin: compact the active streams, choose EOS-enabled ones, init state
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kBeginThreads) frame_begin_kernel(Frame f) {
  __shared__ int warp_act[kBeginThreads / 32], warp_en[kBeginThreads / 32];
  __shared__ int base_act, base_en;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    base_act = 0;
    base_en = 0;
  }
  __syncthreads();
  for (int start = 0; start < f.n; start += kBeginThreads) {
    const int s = start + threadIdx.x;
    const bool in = s < f.n;
    const bool act = in && (f.active == nullptr || f.active[s]);
    bool en = act && !f.unfinished[s] && !f.finished[s] && !f.forbid[s];
    int32_t init_inv = 0;
    if (en && f.final_w == nullptr) {
      init_inv = 2;  // EOS evaluation required but no final projection supplied
      en = false;
    }
    if (in) {
      f.ctr[s] = f.counter_io[s];
      f.inv[s] = init_inv;
    }
    const unsigned ba = __ballot_sync(0xffffffffu, act);
    const unsigned be = __ballot_sync(0xffffffffu, en);
    if (lane == 0) {
      warp_act[warp] = __popc(ba);
      warp_en[warp] = __popc(be);
    }
    __syncthreads();
    int pa = base_act, pe = base_en;
    for (int w = 0; w < warp; ++w) {
      pa += warp_act[w];
      pe += warp_en[w];
    }
    const unsigned below = (1u << lane) - 1u;
    if (act) f.list[pa + __popc(ba & below)] = s;
    if (in) f.eos_slot[s] = en ? pe + __popc(be & below) : -1;
    if (en) f.eos_list[pe + __popc(be & below)] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 0; w < kBeginThreads / 32; ++w) {
        base_act += warp_act[w];
        base_en += warp_en[w];
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *f.count = base_act;
    *f.eos_count = base_en;
  }
}

// ---------------------------------------------------------------------------
// linear layers
// ---------------------------------------------------------------------------

enum Pro { kProHidden, kProGather, kProLn1, kProLn2, kProAtt, kProH, kProX };
enum Epi { kEpiInProj, kEpiQkv, kEpiResid, kEpiGelu, kEpiHead };

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(h2[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ float gelu_tanh(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

// Token that feeds position p + 1: the sampled one, or the caller's forced
// token (clamped into the vocabulary so a bad value cannot index outside the
// table).
__device__ __forceinline__ int64_t input_token(const Frame& f, int s, int p) {
  if (f.forced) {
    const int64_t t = f.forced[static_cast<int64_t>(s) * kPositions + p];
    return t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
  }
  return f.tokens[static_cast<int64_t>(s) * kPositions + p];
}

// Fills xs[m][0..K) (bf16) for row r of the tile; one warp per row.
template <int PRO>
__device__ __forceinline__ void load_row(const Frame& f, int p, int l, int r, int K, bf16* xs_row) {
  const int lane = threadIdx.x & 31;
  const int i = r / f.rp, sub = r % f.rp;
  const bf16* src = nullptr;
  if constexpr (PRO == kProHidden) {
    const int s = f.list[i];
    src = f.hidden + (static_cast<int64_t>(s) * f.rp + sub) * kEmbed;
  } else if constexpr (PRO == kProGather) {
    const int s = f.list[i];
    const int64_t tok = input_token(f, s, p - 1);
    src = f.emb + (static_cast<int64_t>(p - 1) * kVocab + tok) * kEmbed;
  } else if constexpr (PRO == kProAtt) {
    src = f.att + static_cast<int64_t>(r) * f.d;
  } else if constexpr (PRO == kProH) {
    src = f.h + static_cast<int64_t>(r) * f.F;
  } else if constexpr (PRO == kProX) {
    src = f.x + static_cast<int64_t>(r) * f.d;
  }
  if constexpr (PRO == kProLn1 || PRO == kProLn2) {
    const bf16* xr = f.x + static_cast<int64_t>(r) * f.d;
    const bf16* w = (PRO == kProLn1 ? f.ln1 : f.ln2) + static_cast<int64_t>(l) * f.d;
    float sum = 0.f;
    for (int k = lane * 8; k < K; k += 256) {
      float v[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + k), v);
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(K);
    float var = 0.f;
    for (int k = lane * 8; k < K; k += 256) {
      float v[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + k), v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float dlt = v[j] - mean;
        var += dlt * dlt;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    const float rstd = 1.0f / sqrtf(var / static_cast<float>(K) + 1.0e-5f);
    for (int k = lane * 8; k < K; k += 256) {
      float v[8], g[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + k), v);
      unpack8(*reinterpret_cast<const uint4*>(w + k), g);
      __align__(16) bf16 out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = f2bf(((v[j] - mean) * rstd) * g[j]);
      *reinterpret_cast<uint4*>(xs_row + k) = *reinterpret_cast<const uint4*>(out);
    }
  } else {
    for (int k = lane * 8; k < K; k += 256) {
      *reinterpret_cast<uint4*>(xs_row + k) = *reinterpret_cast<const uint4*>(src + k);
    }
  }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(kLinThreads) linear_kernel(Frame f, int p, int l, int N, int K, const bf16* W,
                                                             const bf16* bias) {
  extern __shared__ __align__(16) unsigned char lin_smem[];
  bf16* xs = reinterpret_cast<bf16*>(lin_smem);
  const int rows = *f.count * f.rp;
  const int r0 = blockIdx.y * kBM;
  if (r0 >= rows) return;
  const int n0 = blockIdx.x * kBN;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  {
    const int r = r0 + warp;
    bf16* xr = xs + warp * K;
    if (r < rows) {
      load_row<PRO>(f, p, l, r, K, xr);
    } else {
      for (int k = lane * 8; k < K; k += 256) *reinterpret_cast<uint4*>(xr + k) = make_uint4(0, 0, 0, 0);
    }
  }
  __syncthreads();
  constexpr int kCols = kBN / (kLinThreads / 32);
  for (int c = 0; c < kCols; ++c) {
    const int n = n0 + warp * kCols + c;
    if (n >= N) break;
    float acc[kBM];
#pragma unroll
    for (int m = 0; m < kBM; ++m) acc[m] = 0.f;
    const bf16* wr = W + static_cast<int64_t>(n) * K;
    for (int k = lane * 8; k < K; k += 256) {
      float wf[8];
      unpack8(*reinterpret_cast<const uint4*>(wr + k), wf);
#pragma unroll
      for (int m = 0; m < kBM; ++m) {
        float xf[8];
        unpack8(*reinterpret_cast<const uint4*>(xs + m * K + k), xf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[m] = fmaf(wf[j], xf[j], acc[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < kBM; ++m) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    }
    float v = acc[0];
#pragma unroll
    for (int m = 1; m < kBM; ++m) v = (lane == m) ? acc[m] : v;
    const int r = r0 + lane;
    if (lane < kBM && r < rows) {
      if constexpr (EPI == kEpiInProj) {
        const float y = round_bf16(__fadd_rn(v, bf2f(bias[n])));
        f.x[static_cast<int64_t>(r) * f.d + n] = f2bf(__fadd_rn(y, bf2f(f.pos[static_cast<int64_t>(p) * f.d + n])));
      } else if constexpr (EPI == kEpiQkv) {
        const bf16 y = f2bf(v);
        if (n < f.d) {
          f.q[static_cast<int64_t>(r) * f.d + n] = y;
        } else {
          const int which = n < 2 * f.d ? 0 : 1;
          const int col = n - (which + 1) * f.d;
          bf16* cache = which == 0 ? f.kc : f.vc;
          const int64_t R = static_cast<int64_t>(f.n) * f.rp;
          cache[((static_cast<int64_t>(l) * R + r) * kPositions + p) * f.d + col] = y;
        }
      } else if constexpr (EPI == kEpiResid) {
        bf16* xp = f.x + static_cast<int64_t>(r) * f.d + n;
        *xp = f2bf(__fadd_rn(bf2f(*xp), round_bf16(v)));
      } else if constexpr (EPI == kEpiGelu) {
        f.h[static_cast<int64_t>(r) * f.F + n] = f2bf(gelu_tanh(round_bf16(v)));
      } else if constexpr (EPI == kEpiHead) {
        const bf16 y = f2bf(__fadd_rn(v, bf2f(bias[n])));
        f.logits[static_cast<int64_t>(r) * kVocab + n] = y;
        if (f.logits_out) {
          const int i = r / f.rp, sub = r % f.rp;
          const int s = f.list[i];
          f.logits_out[((static_cast<int64_t>(s) * kPositions + p) * f.rp + sub) * kVocab + n] = y;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// tensor-core linear layers (shapes with K a multiple of 64): the
// activations are materialised as bf16 rows (LayerNorm rows first go to
// `att`, which is free at both LayerNorms), then gemm_tc.cuh runs them with
// the active rows on the MMA's M side (count on the device) and the layer's
// output features on its N side (256 per tile); the epilogue does what
// linear_kernel's does, 32 consecutive features of one row per lane.
// ---------------------------------------------------------------------------

constexpr int kRowChunks = 4;  // 8-column chunks per lane: rows of up to 1024 features in registers

// LayerNorm (no bias, eps 1e-5) of one row held in registers, v[8c + j] =
// feature 8 (lane + 32c) + j, written to out; the same arithmetic and order
// as load_row's LayerNorm prologue.
__device__ __forceinline__ void ln_row_regs(const float (&v)[8 * kRowChunks], int K, const bf16* w, bf16* out) {
  const int lane = threadIdx.x & 31;
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    if (lane * 8 + 256 * c < K) {
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[8 * c + j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / static_cast<float>(K);
  float var = 0.f;
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    if (lane * 8 + 256 * c < K) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float dlt = v[8 * c + j] - mean;
        var += dlt * dlt;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float rstd = 1.0f / sqrtf(var / static_cast<float>(K) + 1.0e-5f);
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int k = lane * 8 + 256 * c;
    if (k < K) {
      float g[8];
      unpack8(*reinterpret_cast<const uint4*>(w + k), g);
      __align__(16) bf16 o8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o8[j] = f2bf(((v[8 * c + j] - mean) * rstd) * g[j]);
      *reinterpret_cast<uint4*>(out + k) = *reinterpret_cast<const uint4*>(o8);
    }
  }
}

// att = LayerNorm(x) with weights w, one warp per row.
__global__ void __launch_bounds__(256) ln_rows_kernel(Frame f, const bf16* w) {
  const int rows = *f.count * f.rp;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const bf16* xr = f.x + static_cast<int64_t>(r) * f.d;
  float v[8 * kRowChunks];
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int k = lane * 8 + 256 * c;
    float t[8];
    if (k < f.d) unpack8(*reinterpret_cast<const uint4*>(xr + k), t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[8 * c + j] = k < f.d ? t[j] : 0.f;
  }
  ln_row_regs(v, f.d, w, f.att + static_cast<int64_t>(r) * f.d);
}

// x = bf16(x + bf16(sum of the split GEMM's partials, in split order)), one
// warp per row (large batches); with LN, att = LayerNorm(x) with weights lnw (the next
// sub-layer's pre-norm).
template <bool LN>
__global__ void __launch_bounds__(256) resid_sum_rows_kernel(Frame f, int splits, const bf16* lnw) {
  const int rows = *f.count * f.rp;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t rows_max = static_cast<int64_t>(f.n) * f.rp;
  bf16* xr = f.x + static_cast<int64_t>(r) * f.d;
  // each split's slice of the row is loaded whole before it is added, two
  // splits at a time (the sums still run split by split, in order)
  uint4 xv[kRowChunks];
  float acc[8 * kRowChunks];
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int k = lane * 8 + 256 * c;
    if (k < f.d) xv[c] = *reinterpret_cast<const uint4*>(xr + k);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[8 * c + j] = 0.f;
  }
#pragma unroll 2
  for (int sp = 0; sp < splits; ++sp) {
    float4 pv[2 * kRowChunks];
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
      const int k = lane * 8 + 256 * c;
      if (k < f.d) {
        const float4* pp = reinterpret_cast<const float4*>(f.part + (sp * rows_max + r) * f.d + k);
        pv[2 * c] = pp[0];
        pv[2 * c + 1] = pp[1];
      }
    }
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
      if (lane * 8 + 256 * c < f.d) {
        float* a = acc + 8 * c;
        a[0] += pv[2 * c].x; a[1] += pv[2 * c].y; a[2] += pv[2 * c].z; a[3] += pv[2 * c].w;
        a[4] += pv[2 * c + 1].x; a[5] += pv[2 * c + 1].y; a[6] += pv[2 * c + 1].z; a[7] += pv[2 * c + 1].w;
      }
    }
  }
  float v[8 * kRowChunks];
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int k = lane * 8 + 256 * c;
    if (k < f.d) {
      float a[8];
      unpack8(xv[c], a);
      __align__(16) bf16 o8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o8[j] = f2bf(__fadd_rn(a[j], round_bf16(acc[8 * c + j])));
        v[8 * c + j] = bf2f(o8[j]);
      }
      *reinterpret_cast<uint4*>(xr + k) = *reinterpret_cast<const uint4*>(o8);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * c + j] = 0.f;
    }
  }
  if constexpr (LN) ln_row_regs(v, f.d, lnw, f.att + static_cast<int64_t>(r) * f.d);
}

// The same for small batches (x = bf16(x + bf16(sum of the partials))); with
// LN, att = LayerNorm(x) with weights lnw (the next sub-layer's pre-norm).
// A row is spread over d / 256 warps (8 features a lane) and a CTA holds two
// rows, so that every split's slice of the row is loaded before the first
// add (the sums still run split by split, in order); the LayerNorm's row sums
// cross the row's warps through shared memory.
template <bool LN>
__global__ void __launch_bounds__(256) resid_sum_wide_kernel(Frame f, int splits, const bf16* lnw) {
  __shared__ float red[2][4][2];  // [row of the CTA][warp of the row][sum, squared deviations]
  const int wpr = (f.d + 255) / 256;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rl = warp / wpr, part = warp % wpr;
  const int rows = *f.count * f.rp;
  const int r = 2 * static_cast<int>(blockIdx.x) + rl;
  const int k = 256 * part + 8 * lane;
  const bool has = r < rows && k < f.d;
  const int64_t rows_max = static_cast<int64_t>(f.n) * f.rp;
  bf16* xr = f.x + static_cast<int64_t>(r) * f.d;
  uint4 xv = make_uint4(0, 0, 0, 0);
  float4 pv[kMaxPhaseSplits][2];
  if (has) {
    xv = *reinterpret_cast<const uint4*>(xr + k);
#pragma unroll
    for (int sp = 0; sp < kMaxPhaseSplits; ++sp) {
      if (sp < splits) {
        const float4* pp = reinterpret_cast<const float4*>(f.part + (sp * rows_max + r) * f.d + k);
        pv[sp][0] = pp[0];
        pv[sp][1] = pp[1];
      }
    }
  }
  float v[8];
  {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int sp = 0; sp < kMaxPhaseSplits; ++sp) {
      if (has && sp < splits) {
        acc[0] += pv[sp][0].x; acc[1] += pv[sp][0].y; acc[2] += pv[sp][0].z; acc[3] += pv[sp][0].w;
        acc[4] += pv[sp][1].x; acc[5] += pv[sp][1].y; acc[6] += pv[sp][1].z; acc[7] += pv[sp][1].w;
      }
    }
    float a[8];
    unpack8(xv, a);
    __align__(16) bf16 o8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o8[j] = f2bf(__fadd_rn(a[j], round_bf16(acc[j])));
      v[j] = has ? bf2f(o8[j]) : 0.f;
    }
    if (has) *reinterpret_cast<uint4*>(xr + k) = *reinterpret_cast<const uint4*>(o8);
  }
  if constexpr (LN) {
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += v[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0 && rl < 2) red[rl][part][0] = sum;
    __syncthreads();
    float tot = 0.f;
    for (int q = 0; q < wpr; ++q) tot += red[rl < 2 ? rl : 0][q][0];
    const float mean = tot / static_cast<float>(f.d);
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float dlt = v[j] - mean;
      sq += has ? dlt * dlt : 0.f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0 && rl < 2) red[rl][part][1] = sq;
    __syncthreads();
    float var = 0.f;
    for (int q = 0; q < wpr; ++q) var += red[rl < 2 ? rl : 0][q][1];
    const float rstd = 1.0f / sqrtf(var / static_cast<float>(f.d) + 1.0e-5f);
    if (has) {
      float g[8];
      unpack8(*reinterpret_cast<const uint4*>(lnw + k), g);
      __align__(16) bf16 o8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o8[j] = f2bf(((v[j] - mean) * rstd) * g[j]);
      *reinterpret_cast<uint4*>(f.att + static_cast<int64_t>(r) * f.d + k) = *reinterpret_cast<const uint4*>(o8);
    }
  }
}


// The residual sum of a split GEMM: rows over d / 256 warps each while one
// warp per row would leave SMs idle (fewer than 8 rows per SM), one warp per
// row above that (measured faster for large batches).
template <bool LN>
void launch_resid_sum(const Frame& f, int splits, const bf16* lnw, cudaStream_t st) {
  const int rows_max = f.n * f.rp;
  if ((rows_max + 7) / 8 < gemm_grid(1 << 30)) {
    resid_sum_wide_kernel<LN><<<(rows_max + 1) / 2, 64 * ((f.d + 255) / 256), 0, st>>>(f, splits, lnw);
  } else {
    resid_sum_rows_kernel<LN><<<(rows_max + 7) / 8, 256, 0, st>>>(f, splits, lnw);
  }
}

// Epilogues of the tensor-core linear layers.  A lane holds 32 consecutive
// output features of one row; the warp stages its 32 rows in shared memory
// (row stride 80 bytes: conflict-free 16-byte access) and writes them back
// four lanes per row, so a store instruction covers eight whole 64-byte row
// segments instead of 32 scattered 16-byte pieces.
constexpr int kPhaseStageRow = 40;  // bf16 per staged row (64 bytes + 16 of padding)

template <int EPI>
struct EpiPhase {
  Frame f;
  int p, l, N;
  const bf16* bias;

  // destination of 8 features [n, n + 8) of row r (q, the K/V cache, FFN hidden)
  __device__ __forceinline__ bf16* dst(int r, int n) const {
    if constexpr (EPI == kEpiQkv) {
      if (n < f.d) return f.q + static_cast<int64_t>(r) * f.d + n;
      const int which = n < 2 * f.d ? 0 : 1;
      const int col = n - (which + 1) * f.d;
      const int64_t R = static_cast<int64_t>(f.n) * f.rp;
      return (which == 0 ? f.kc : f.vc) + ((static_cast<int64_t>(l) * R + r) * kPositions + p) * f.d + col;
    } else if constexpr (EPI == kEpiGelu) {
      return f.h + static_cast<int64_t>(r) * f.F + n;
    } else {
      return f.x + static_cast<int64_t>(r) * f.d + n;
    }
  }

  __device__ __forceinline__ void chunk(int m, int n0, int /*ks*/, const uint32_t (&v)[32], int /*n_cols*/) const {
    __shared__ __align__(16) bf16 stage[kGemmEpiWarps][32][kPhaseStageRow];
    const int lane = threadIdx.x & 31, w = gemm_epi_warp();
    float bvals[32];
    if constexpr (EPI == kEpiHead) {
      // the chunk's bias (the same 64 bytes for every lane: a broadcast load)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float t[8];
        if (n0 + 8 * q < N) {
          unpack8(reinterpret_cast<const uint4*>(bias + n0)[q], t);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) t[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) bvals[8 * q + e] = t[e];
      }
    }
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float a = __uint_as_float(v[2 * j]), b = __uint_as_float(v[2 * j + 1]);
      if constexpr (EPI == kEpiHead) {
        a = __fadd_rn(a, bvals[2 * j]);
        b = __fadd_rn(b, bvals[2 * j + 1]);
      } else if constexpr (EPI == kEpiGelu) {
        a = gelu_tanh(round_bf16(a));
        b = gelu_tanh(round_bf16(b));
      }
      // q|k|v: bf16(v); residual: bf16(v) here, added to x below
      const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
      packed[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    uint4* mine = reinterpret_cast<uint4*>(stage[w][lane]);
#pragma unroll
    for (int q = 0; q < 4; ++q) mine[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    __syncwarp();
    const int m0 = m - lane;  // the warp's first row
    const int rows = *f.count * f.rp;  // rows past the active ones are padding
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int rl = 8 * it + (lane >> 2), q = lane & 3;
      const int r = m0 + rl, n = n0 + 8 * q;
      if (r < rows && n < N) {
        const uint4 y = reinterpret_cast<const uint4*>(stage[w][rl])[q];
        if constexpr (EPI == kEpiHead) {
          *reinterpret_cast<uint4*>(f.logits + static_cast<int64_t>(r) * kVocab + n) = y;
          if (f.logits_out != nullptr) {
            const int i = r / f.rp, sub = r % f.rp;
            bf16* out = f.logits_out + ((static_cast<int64_t>(f.list[i]) * kPositions + p) * f.rp + sub) * kVocab + n;
            *reinterpret_cast<uint4*>(out) = y;
          }
        } else if constexpr (EPI == kEpiResid) {
          bf16* xp = dst(r, n);
          float x8[8], y8[8];
          unpack8(*reinterpret_cast<const uint4*>(xp), x8);
          unpack8(y, y8);
          __align__(16) bf16 o8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) o8[e] = f2bf(__fadd_rn(x8[e], y8[e]));
          *reinterpret_cast<uint4*>(xp) = *reinterpret_cast<const uint4*>(o8);
        } else {
          *reinterpret_cast<uint4*>(dst(r, n)) = y;
        }
      }
    }
    __syncwarp();
  }
};

// Split-K partial sums of a residual GEMM: part[ks][r][n] (f32), summed by
// launch_resid_sum; staged like EpiPhase, 16 columns (64 bytes per row) at a
// time.
constexpr int kPhaseStageRowF = 20;  // f32 per staged row (64 bytes + 16 of padding)
struct EpiPhasePart {
  float* part;
  int rows_max, N;
  const int* count;
  int rp;
  __device__ __forceinline__ void chunk(int m, int n0, int ks, const uint32_t (&v)[32], int /*n_cols*/) const {
    __shared__ __align__(16) float stage[kGemmEpiWarps][32][kPhaseStageRowF];
    const int lane = threadIdx.x & 31, w = gemm_epi_warp();
    const int m0 = m - lane;
    const int rows = *count * rp;
    float* base = part + static_cast<int64_t>(ks) * rows_max * N;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4* mine = reinterpret_cast<float4*>(stage[w][lane]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        mine[q] = make_float4(__uint_as_float(v[16 * h + 4 * q]), __uint_as_float(v[16 * h + 4 * q + 1]),
                              __uint_as_float(v[16 * h + 4 * q + 2]), __uint_as_float(v[16 * h + 4 * q + 3]));
      }
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int rl = 8 * it + (lane >> 2), q = lane & 3;
        const int r = m0 + rl, n = n0 + 16 * h + 4 * q;
        if (r < rows && n < N) {
          *reinterpret_cast<float4*>(base + static_cast<int64_t>(r) * N + n) =
              reinterpret_cast<const float4*>(stage[w][rl])[q];
        }
      }
      __syncwarp();
    }
  }
};

// A operand of a tensor-core linear layer: the rows it reads.
template <int PRO>
const bf16* tc_rows(const Frame& f) {
  if constexpr (PRO == kProAtt || PRO == kProLn1 || PRO == kProLn2) return f.att;
  if constexpr (PRO == kProH) return f.h;
  return f.x;  // kProX
}

// K in whole 64-column chunks, q, k and v starting on 32-column chunk
// bounds, rows that fit ln_row_regs (the workspace's 256-byte alignment puts
// every row buffer on the 16-byte boundary a tensor map needs).
bool tc_linear_supported(int d, int F) { return d % 64 == 0 && F % 64 == 0 && d <= 256 * kRowChunks; }

// Weight-tile width (N side) of a phase GEMM: the narrowest of 256 / 128 / 64
// columns whose tiles (x K splits) still fit in one wave of the SMs.  Few
// activation rows give few 128-row tiles, and 64-wide weight tiles then put
// 4x the CTAs on the K loop (each MMA of N = 64 costs ~48 cycles against
// ~128 at N = 256); large batches keep 256-wide tiles.
int phase_weight_tile(int m_tiles, int N, int splits) {
  const int sms = gemm_grid(1 << 30);
  int bn = 256;
  for (const int cand : {128, 64}) {
    if (m_tiles * ((N + cand - 1) / cand) * splits <= sms) bn = cand;
  }
  return bn;
}

template <int BN, int PRO, int EPI>
cudaError_t launch_linear_tc_bn(const Frame& f, cudaStream_t st, int p, int l, int N, const bf16* bias,
                                const CUtensorMap& amap, const CUtensorMap& bmap, const GemmProblem& pr) {
  if constexpr (EPI < 0) {
    return launch_gemm_tc<BN>(amap, bmap, pr, EpiPhasePart{f.part, f.n * f.rp, N, f.count, f.rp}, st);
  } else {
    return launch_gemm_tc<BN>(amap, bmap, pr, EpiPhase<EPI>{f, p, l, N, bias}, st);
  }
}

// The GEMM of a tensor-core linear layer (its LayerNorm rows, where it has
// one, already in `att`); EPI < 0: split-K partial sums into f.part.
template <int PRO, int EPI>
cudaError_t launch_linear_tc(const Frame& f, cudaStream_t st, int p, int l, int N, int K, const bf16* W,
                             const bf16* bias, int splits = 1) {
  const int rows_max = f.n * f.rp;
  const int bn = phase_weight_tile((rows_max + 127) / 128, N, splits);
  CUtensorMap amap, bmap;
  if (!cached_map(&amap, tc_rows<PRO>(f), static_cast<uint64_t>(K), static_cast<uint64_t>(rows_max), 128) ||
      !cached_map(&bmap, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint32_t>(bn))) {
    return cudaErrorInvalidValue;
  }
  GemmProblem pr;
  pr.m_tiles = (rows_max + 127) / 128;
  pr.m_rows_dev = f.count;
  pr.m_rows_scale = f.rp;
  pr.n_rows = N;
  pr.n_rows_dev = nullptr;
  pr.n_rows_scale = 1;
  pr.k_chunks = K / kGemmKChunk / splits;
  pr.splits = splits;
  pr.status = nullptr;
  pr.b_constant = 0;
  return bn == 64    ? launch_linear_tc_bn<64, PRO, EPI>(f, st, p, l, N, bias, amap, bmap, pr)
         : bn == 128 ? launch_linear_tc_bn<128, PRO, EPI>(f, st, p, l, N, bias, amap, bmap, pr)
                     : launch_linear_tc_bn<256, PRO, EPI>(f, st, p, l, N, bias, amap, bmap, pr);
}

// Identity in-projection (d == 768): x = bf16(src + pos[p]).
// Identity in-projection: x = bf16(src + pos[p]), src the decoder hidden row
// (p = 0) or the embedding of the previous position's token; one warp per
// row.  With LN (tensor-core layers) it also writes att = LN1_0(x).
__device__ __forceinline__ void pos_row(const Frame& f, int r, const bf16* src, int p);

template <bool LN>
__global__ void __launch_bounds__(256) add_pos_kernel(Frame f, int p) {
  const int rows = *f.count * f.rp;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int i = r / f.rp, sub = r % f.rp;
  const int s = f.list[i];
  const bf16* src = p == 0 ? f.hidden + (static_cast<int64_t>(s) * f.rp + sub) * kEmbed
                           : f.emb + (static_cast<int64_t>(p - 1) * kVocab + input_token(f, s, p - 1)) * kEmbed;
  if constexpr (LN) {
    pos_row(f, r, src, p);
  } else {
    const int lane = threadIdx.x & 31;
    const bf16* pos = f.pos + static_cast<int64_t>(p) * f.d;
    bf16* xr = f.x + static_cast<int64_t>(r) * f.d;
    for (int k = lane * 8; k < f.d; k += 256) {
      float a[8], b[8];
      unpack8(*reinterpret_cast<const uint4*>(src + k), a);
      unpack8(*reinterpret_cast<const uint4*>(pos + k), b);
      __align__(16) bf16 o8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o8[j] = f2bf(__fadd_rn(a[j], b[j]));
      *reinterpret_cast<uint4*>(xr + k) = *reinterpret_cast<const uint4*>(o8);
    }
  }
}

// Row r of the identity in-projection at position p, one warp: x = bf16(src +
// pos[p]) and att = LN1_0(x).
__device__ __forceinline__ void pos_row(const Frame& f, int r, const bf16* src, int p) {
  const int lane = threadIdx.x & 31;
  const bf16* pos = f.pos + static_cast<int64_t>(p) * f.d;
  bf16* xr = f.x + static_cast<int64_t>(r) * f.d;
  float v[8 * kRowChunks];
#pragma unroll
  for (int j = 0; j < 8 * kRowChunks; ++j) v[j] = 0.f;
  for (int c = 0, k = lane * 8; k < f.d; ++c, k += 256) {
    float a[8], b[8];
    unpack8(*reinterpret_cast<const uint4*>(src + k), a);
    unpack8(*reinterpret_cast<const uint4*>(pos + k), b);
    __align__(16) bf16 o8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o8[j] = f2bf(__fadd_rn(a[j], b[j]));
    *reinterpret_cast<uint4*>(xr + k) = *reinterpret_cast<const uint4*>(o8);
#pragma unroll
    for (int cc = 0; cc < kRowChunks; ++cc) {
      if (cc == c) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * cc + j] = bf2f(o8[j]);
      }
    }
  }
  ln_row_regs(v, f.d, f.ln1, f.att + static_cast<int64_t>(r) * f.d);
}

// ---------------------------------------------------------------------------
// attention: one warp per (row, head), p + 1 keys
// ---------------------------------------------------------------------------

// Causal self-attention of position p for one (row, head) per warp: lane
// 8 g + c holds head dims [8c, +8) of the window's positions g, g + 4, g + 8,
// g + 12, so each lane issues at most four 16-byte key and four value loads,
// all before the first use.  A score is summed over the 8 lanes of its group,
// rounded as the reference rounds it (bf16, x 1/8, bf16) and gathered into
// every lane, which runs the softmax over the positions in order; each lane
// weights its own value rows and the four groups' sums are combined.
__global__ void __launch_bounds__(256) attention_kernel(Frame f, int p, int l) {
  const int rows = *f.count * f.rp;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows * f.H) return;
  const int r = gw / f.H, hd = gw % f.H;
  const int g = lane >> 3, cc = lane & 7;
  const int64_t R = static_cast<int64_t>(f.n) * f.rp;
  float q[8];
  unpack8(*reinterpret_cast<const uint4*>(f.q + static_cast<int64_t>(r) * f.d + hd * kHeadDim + 8 * cc), q);
  const int64_t base = ((static_cast<int64_t>(l) * R + r) * kPositions) * f.d + hd * kHeadDim + 8 * cc;
  uint4 kr[4], vr[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = g + 4 * i;
    if (j <= p) {
      kr[i] = *reinterpret_cast<const uint4*>(f.kc + base + static_cast<int64_t>(j) * f.d);
      vr[i] = *reinterpret_cast<const uint4*>(f.vc + base + static_cast<int64_t>(j) * f.d);
    }
  }
  float sc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float dot = 0.f;
    if (g + 4 * i <= p) {
      float k[8];
      unpack8(kr[i], k);
#pragma unroll
      for (int e = 0; e < 8; ++e) dot = fmaf(q[e], k[e], dot);
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    dot += __shfl_xor_sync(0xffffffffu, dot, 4);
    sc[i] = round_bf16(__fmul_rn(round_bf16(dot), 0.125f));
  }
  // position j's score lives in group j mod 4, slot j / 4
  float mx = -CUDART_INF_F;
  float s[kPositions];
#pragma unroll
  for (int j = 0; j < kPositions; ++j) {
    s[j] = __shfl_sync(0xffffffffu, sc[j >> 2], 8 * (j & 3));
    if (j <= p) mx = fmaxf(mx, s[j]);
  }
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPositions; ++j) {
    if (j <= p) sum += expf(s[j] - mx);
  }
  float o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (g + 4 * i <= p) {
      const float prob = round_bf16(expf(sc[i] - mx) / sum);
      float v[8];
      unpack8(vr[i], v);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = fmaf(prob, v[e], o[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    o[e] += __shfl_xor_sync(0xffffffffu, o[e], 8);
    o[e] += __shfl_xor_sync(0xffffffffu, o[e], 16);
  }
  if (g == 0) {
    __align__(16) bf16 o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = f2bf(o[e]);
    *reinterpret_cast<uint4*>(f.att + static_cast<int64_t>(r) * f.d + hd * kHeadDim + 8 * cc) =
        *reinterpret_cast<const uint4*>(o8);
  }
}

// ---------------------------------------------------------------------------
// sampling + running embedding sum
// ---------------------------------------------------------------------------

// NEXT (identity in-projection, tensor-core layers): the CTA also writes the
// next position's input rows of its session and their LN1 (what
// add_pos_kernel<true> would do), one warp per row.
template <bool NEXT>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(Frame f, int p) {
  __shared__ SampleShared sh;
  __shared__ __align__(16) unsigned char scratch[kSampleScratchBytes];
  const int i = blockIdx.x;
  if (i >= *f.count) return;
  const int s = f.list[i];
  SampleCall c;
  c.logits = f.logits + static_cast<int64_t>(i) * f.rp * kVocab;
  c.uncond_offset = kVocab;
  c.kind = f.rp == 2 ? kLogitsBf16Cfg : kLogitsBf16;
  c.unfinished = f.unfinished[s];
  c.finished = f.finished[s];
  c.forbid_eos = f.forbid[s];
  c.seed = f.seed[s];
  c.counter = f.ctr[s];
  int invalid = 0;
  const int token = sample_block(c, f.prm, sh, scratch, &invalid);
  if (threadIdx.x == 0) {
    f.tokens[s * kPositions + p] = token;
    f.inv[s] |= invalid;
    const bool counter_valid = c.counter >= 0 && c.counter <= kMaxCounter;
    if (!f.prm.argmax && counter_valid) f.ctr[s] = c.counter + 1;
  }
  const bf16* row = f.emb + (static_cast<int64_t>(p) * kVocab + token) * kEmbed;
  float* acc = f.emb_acc + static_cast<int64_t>(s) * kEmbed;
  for (int k = threadIdx.x; k < kEmbed; k += blockDim.x) {
    const float v = bf2f(row[k]);
    acc[k] = p == 0 ? v : round_bf16(__fadd_rn(acc[k], v));
  }
  if constexpr (NEXT) {
    const int warp = threadIdx.x >> 5;
    if (p + 1 < kPositions && warp < f.rp) {
      int64_t tin = token;
      if (f.forced) {
        const int64_t t = f.forced[static_cast<int64_t>(s) * kPositions + p];
        tin = t < 0 ? 0 : (t >= kVocab ? kVocab - 1 : t);
      }
      pos_row(f, i * f.rp + warp, f.emb + (static_cast<int64_t>(p) * kVocab + tin) * kEmbed, p + 1);
    }
  }
}

// ---------------------------------------------------------------------------
// frame end: EOS decision and commit
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) frame_end_kernel(Frame f) {
  const int i = blockIdx.x;
  if (i >= *f.count) return;
  const int s = f.list[i];
  if (threadIdx.x == 0) {
    const int32_t* tok = f.tokens + s * kPositions;
    for (int p = 0; p < kPositions; ++p) {
      f.codec_tokens[codec_index(f, s, p)] = tok[p];
    }
    const int slot = f.eos_slot[s];
    const int e = slot < 0 ? 0 : slot;
    commit_end(f, s, eos_decide_proj(eos_keys(f, s, e), eos_logits(f, s, e), tok, slot >= 0, f.finished[s]));
    f.counter_io[s] = f.ctr[s];
    // a projection whose bounded waits gave up marks its sessions invalid (bit 4)
    f.invalid_rows[s] = f.inv[s] | (slot >= 0 && f.eos_pre == nullptr && f.eos_count[1] != 0 ? 16 : 0);
  }
  const float* acc = f.emb_acc + static_cast<int64_t>(s) * kEmbed;
  for (int k = threadIdx.x; k < kEmbed; k += blockDim.x) {
    f.next_emb[static_cast<int64_t>(s) * kEmbed + k] = f2bf(__fdiv_rn(acc[k], 16.0f));
  }
}

template <int PRO, int EPI>
void launch_linear(const Frame& f, cudaStream_t st, int p, int l, int N, int K, const bf16* W, const bf16* bias) {
  const int rows_max = f.n * f.rp;
  const dim3 grid((N + kBN - 1) / kBN, (rows_max + kBM - 1) / kBM);
  const size_t smem = static_cast<size_t>(kBM) * K * sizeof(bf16);
  linear_kernel<PRO, EPI><<<grid, kLinThreads, smem, st>>>(f, p, l, N, K, W, bias);
}

bool shape_ok(const mtt_b200_local_ar_shape_t* s) {
  return s && s->d_model > 0 && s->n_heads > 0 && s->d_model == s->n_heads * kHeadDim && s->d_model % 256 == 0 &&
         s->d_ffn % 256 == 0 && s->d_ffn > 0 && s->n_layers > 0 && s->n_layers <= 8 && s->d_ffn <= 3072 &&
         s->d_model <= 3072;
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API size_t mtt_b200_local_ar_frame_workspace_size(const mtt_b200_local_ar_shape_t* shape,
                                                                      int32_t max_streams, int32_t cfg) {
  if (!mtt::shape_ok(shape) || max_streams <= 0) return 0;
  return mtt::make_layout(shape->d_model, shape->n_layers, shape->d_ffn, max_streams, cfg ? 2 : 1).total;
}

namespace {

// Trace hook: device buffer for the fused cluster kernel's phase stamps
// (mtt_b200_test_frame_trace); null in normal operation.
std::atomic<uint64_t*> g_frame_trace{nullptr};

// Resolves the path for a shape / configuration / batch size on the current
// device.  AUTO, benchmark shape, by the batch's 16-row tiles (8 sessions
// each): the fused 16-CTA cluster kernel while the tiles fit in one wave of
// its clusters (on B200 0.24 ms per frame, 7 clusters); then the split
// kernel with the widest cluster (8, 4, else 2 CTAs per tile) whose tiles
// still fit in one wave (0.35 / 0.42 / 0.55 ms per frame; 15 / 33 / 74
// clusters); above that the pair kernel while its 16-session tiles fit in one
// wave (0.73 ms per frame, 74 clusters of 2), then the tile kernel (0.75 ms
// per frame, one CTA per SM).
// So the frame time falls with the batch, and sessions sharded over more
// GPUs run shorter frames.  Other shapes: the phase kernels.
int split_of_path(int32_t path) {
  return path == MTT_B200_FRAME_PATH_SPLIT_8 ? 8
         : path == MTT_B200_FRAME_PATH_SPLIT_4 ? 4
         : (path == MTT_B200_FRAME_PATH_SPLIT_2 || path == MTT_B200_FRAME_PATH_SPLIT_2X32) ? 2
                                                                                          : 1;
}

int rows_of_path(int32_t path) { return path == MTT_B200_FRAME_PATH_SPLIT_2X32 ? 32 : 16; }

bool is_split_path(int32_t path) {
  return path == MTT_B200_FRAME_PATH_SPLIT_1 || path == MTT_B200_FRAME_PATH_SPLIT_2 ||
         path == MTT_B200_FRAME_PATH_SPLIT_4 || path == MTT_B200_FRAME_PATH_SPLIT_8 ||
         path == MTT_B200_FRAME_PATH_SPLIT_2X32;
}

int32_t resolve_path(const mtt_b200_local_ar_shape_t* shape, const mtt_b200_sampling_config_t* sampling,
                     int32_t n_streams) {
  mtt::Frame probe{};
  probe.d = shape->d_model;
  probe.L = shape->n_layers;
  probe.H = shape->n_heads;
  probe.F = shape->d_ffn;
  probe.rp = sampling->cfg ? 2 : 1;
  probe.in_proj = shape->d_model != mtt::kEmbed;
  const bool fused = mtt::fused_frame_supported(probe);
  const bool tile = mtt::tile_frame_supported(probe);
  const bool pair = mtt::pair_frame_supported(probe);
  switch (sampling->path) {
    case MTT_B200_FRAME_PATH_AUTO: {
      if (!fused && !tile && !pair) return MTT_B200_FRAME_PATH_PHASE_KERNELS;
      const int spt = 16 / probe.rp;  // sessions per tile of the fused cluster kernel
      if (fused && (n_streams + spt - 1) / spt <= mtt::fused_frame_clusters()) {
        return MTT_B200_FRAME_PATH_FUSED_CLUSTER;
      }
      const int tiles = (n_streams + 7) / 8;  // split kernel tiles
      if (tiles <= mtt::split_frame_clusters(8, 16) && mtt::split_frame_supported(probe, 8, 16)) {
        return MTT_B200_FRAME_PATH_SPLIT_8;
      }
      if (tiles <= mtt::split_frame_clusters(4, 16) && mtt::split_frame_supported(probe, 4, 16)) {
        return MTT_B200_FRAME_PATH_SPLIT_4;
      }
      // 16-session tiles on 4-CTA clusters while they fit in one wave
      if ((n_streams + 15) / 16 <= mtt::quad_frame_clusters() && mtt::quad_frame_supported(probe)) {
        return MTT_B200_FRAME_PATH_QUAD;
      }
      if (tiles <= mtt::split_frame_clusters(2, 16) && mtt::split_frame_supported(probe, 2, 16)) {
        return MTT_B200_FRAME_PATH_SPLIT_2;
      }
      if (pair && (n_streams + 15) / 16 <= mtt::pair_frame_clusters()) return MTT_B200_FRAME_PATH_FUSED_PAIR;
      if (tile) return MTT_B200_FRAME_PATH_FUSED_TILE;
      if (pair) return MTT_B200_FRAME_PATH_FUSED_PAIR;
      return MTT_B200_FRAME_PATH_FUSED_CLUSTER;
    }
    case MTT_B200_FRAME_PATH_PHASE_KERNELS:
      return MTT_B200_FRAME_PATH_PHASE_KERNELS;
    case MTT_B200_FRAME_PATH_FUSED_CLUSTER:
      return fused ? MTT_B200_FRAME_PATH_FUSED_CLUSTER : MTT_B200_STATUS_UNSUPPORTED;
    case MTT_B200_FRAME_PATH_FUSED_TILE:
      return tile ? MTT_B200_FRAME_PATH_FUSED_TILE : MTT_B200_STATUS_UNSUPPORTED;
    case MTT_B200_FRAME_PATH_FUSED_PAIR:
      return pair ? MTT_B200_FRAME_PATH_FUSED_PAIR : MTT_B200_STATUS_UNSUPPORTED;
    case MTT_B200_FRAME_PATH_SPLIT_1:
    case MTT_B200_FRAME_PATH_SPLIT_2:
    case MTT_B200_FRAME_PATH_SPLIT_4:
    case MTT_B200_FRAME_PATH_SPLIT_8:
    case MTT_B200_FRAME_PATH_SPLIT_2X32:
      return mtt::split_frame_supported(probe, split_of_path(sampling->path), rows_of_path(sampling->path))
                 ? sampling->path
                 : MTT_B200_STATUS_UNSUPPORTED;
    case MTT_B200_FRAME_PATH_QUAD:
      return mtt::quad_frame_supported(probe) ? MTT_B200_FRAME_PATH_QUAD : MTT_B200_STATUS_UNSUPPORTED;
    case MTT_B200_FRAME_PATH_OCTO:
      return mtt::octo_frame_supported(probe) ? MTT_B200_FRAME_PATH_OCTO : MTT_B200_STATUS_UNSUPPORTED;
    default:
      return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
}

}  // namespace

extern "C" MTT_B200_API int mtt_b200_test_frame_trace(uint64_t* stamps) {
  g_frame_trace.store(stamps);
  return MTT_B200_STATUS_OK;
}

extern "C" MTT_B200_API int32_t mtt_b200_local_ar_frame_path(const mtt_b200_local_ar_shape_t* shape,
                                                             const mtt_b200_sampling_config_t* sampling,
                                                             int32_t n_streams) {
  if (!mtt::shape_ok(shape) || sampling == nullptr || n_streams <= 0) return MTT_B200_STATUS_INVALID_ARGUMENT;
  return resolve_path(shape, sampling, n_streams);
}

extern "C" MTT_B200_API int32_t mtt_b200_local_ar_frame_path_clusters(int32_t path) {
  switch (path) {
    case MTT_B200_FRAME_PATH_FUSED_CLUSTER: return mtt::fused_frame_clusters();
    case MTT_B200_FRAME_PATH_FUSED_PAIR: return mtt::pair_frame_clusters();
    case MTT_B200_FRAME_PATH_FUSED_TILE: return mtt::tile_frame_clusters();
    case MTT_B200_FRAME_PATH_SPLIT_1:
    case MTT_B200_FRAME_PATH_SPLIT_2:
    case MTT_B200_FRAME_PATH_SPLIT_4:
    case MTT_B200_FRAME_PATH_SPLIT_8:
    case MTT_B200_FRAME_PATH_SPLIT_2X32: return mtt::split_frame_clusters(split_of_path(path), rows_of_path(path));
    case MTT_B200_FRAME_PATH_QUAD: return mtt::quad_frame_clusters();
    case MTT_B200_FRAME_PATH_OCTO: return mtt::octo_frame_clusters();
    default: return 0;
  }
}

extern "C" MTT_B200_API int32_t mtt_b200_local_ar_frame_launch_count(const mtt_b200_local_ar_shape_t* shape,
                                                                     const mtt_b200_sampling_config_t* sampling,
                                                                     int32_t n_streams) {
  if (!mtt::shape_ok(shape) || sampling == nullptr || n_streams <= 0) return 0;
  const int32_t path = resolve_path(shape, sampling, n_streams);
  if (path == MTT_B200_FRAME_PATH_FUSED_CLUSTER || path == MTT_B200_FRAME_PATH_FUSED_TILE ||
      path == MTT_B200_FRAME_PATH_FUSED_PAIR || path == MTT_B200_FRAME_PATH_QUAD || path == MTT_B200_FRAME_PATH_OCTO ||
      is_split_path(path)) {
    return 3;  // fused frame, EOS projection, EOS finish
  }
  if (path != MTT_B200_FRAME_PATH_PHASE_KERNELS) return 0;
  // begin + 16 x (embed + 5 per layer + head + sample) + eos projection + end
  // begin; per position: in-projection (+ LayerNorm rows on the tensor-core
  // layers) or position add, the layers, head, sampling; EOS rows and
  // projection GEMM; end
  if (mtt::tc_linear_supported(shape->d_model, shape->d_ffn)) {
    // 7 per layer; without the split, no LayerNorm launch after the last FFN2;
    // with the identity in-projection only position 0 has a position-add
    // launch (the sampling kernel writes the next position's rows)
    const int last = mtt::fused_frame_shape(shape->d_model, shape->n_layers, shape->d_ffn) ? 1 : 0;
    const int per_position = 7 * shape->n_layers - last + 2;
    if (shape->d_model != mtt::kEmbed) return 1 + mtt::kPositions * (2 + per_position) + 3;
    return 1 + 1 + mtt::kPositions * per_position + 3;
  }
  return 1 + mtt::kPositions * (1 + 5 * shape->n_layers + 2) + 3;
}

extern "C" MTT_B200_API int mtt_b200_launch_local_ar_frame(const mtt_b200_local_ar_shape_t* shape,
                                                          const mtt_b200_local_ar_weights_t* w,
                                                          const mtt_b200_sampling_config_t* sampling,
                                                          const mtt_b200_stream_batch_t* b, void* workspace,
                                                          size_t workspace_bytes, void* stream) {
  using namespace mtt;
  if (!shape_ok(shape) || !w || !sampling || !b || !workspace || b->n_streams <= 0) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  const bool in_proj = shape->d_model != kEmbed;
  if (!w->pos || !w->ln_self || !w->qkv || !w->o || !w->ln_ff || !w->ffn1 || !w->ffn2 || !w->head_w || !w->head_b ||
      !w->emb || (in_proj && (!w->in_proj_w || !w->in_proj_b)) || (w->final_w == nullptr) != (w->final_b == nullptr)) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  if (!b->decoder_hidden || !b->unfinished || !b->finished || !b->forbid_eos || !b->rng_seed || !b->rng_counter ||
      !b->codec_tokens || !b->invalid_rows || !b->end_frame_index || !b->next_embedding) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  // codec rows: [n][8][stride] with the frame's two frames at offset, offset
  // even (finalize_local_step's frame offsets 0, 2, 4, 6 for stride 8)
  if (b->codec_frames_stride < 0 || (b->codec_frames_stride != 0 && b->codec_frames_stride < kFrames) ||
      b->codec_frame_offset < 0 || b->codec_frame_offset % kFrames != 0 ||
      b->codec_frame_offset + kFrames > (b->codec_frames_stride == 0 ? kFrames : b->codec_frames_stride)) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  if (sampling->top_k < 1 || sampling->top_k > kVocab || !(sampling->temperature > 0.f) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  const int rp = sampling->cfg ? 2 : 1;
  const Layout lo = make_layout(shape->d_model, shape->n_layers, shape->d_ffn, b->n_streams, rp);
  if (workspace_bytes < lo.total) return MTT_B200_STATUS_INVALID_ARGUMENT;

  Frame f{};
  f.d = shape->d_model;
  f.L = shape->n_layers;
  f.H = shape->n_heads;
  f.F = shape->d_ffn;
  f.rp = rp;
  f.n = b->n_streams;
  f.in_proj = in_proj;
  f.prm = SamplingParams{sampling->top_k, sampling->temperature, sampling->cfg_scale, sampling->argmax};
  auto B = [](const void* p) { return static_cast<const bf16*>(p); };
  f.in_w = B(w->in_proj_w);
  f.in_b = B(w->in_proj_b);
  f.pos = B(w->pos);
  f.ln1 = B(w->ln_self);
  f.qkv = B(w->qkv);
  f.o = B(w->o);
  f.ln2 = B(w->ln_ff);
  f.w1 = B(w->ffn1);
  f.w2 = B(w->ffn2);
  f.head_w = B(w->head_w);
  f.head_b = B(w->head_b);
  f.emb = B(w->emb);
  f.final_w = B(w->final_w);
  f.final_b = B(w->final_b);
  f.emb_proj = in_proj ? B(w->emb_proj) : nullptr;
  f.hidden = B(b->decoder_hidden);
  f.unfinished = b->unfinished;
  f.finished = b->finished;
  f.forbid = b->forbid_eos;
  f.active = b->active;
  f.seed = b->rng_seed;
  f.counter_io = b->rng_counter;
  f.codec_tokens = b->codec_tokens;
  f.codec_stride = b->codec_frames_stride == 0 ? kFrames : b->codec_frames_stride;
  f.codec_offset = b->codec_frame_offset;
  f.finished_latch = b->finished_latch;
  f.codec_frames = b->codec_frames;
  f.invalid_rows = b->invalid_rows;
  f.end_frame = b->end_frame_index;
  f.next_emb = static_cast<bf16*>(b->next_embedding);
  f.forced = b->forced_tokens;
  f.logits_out = static_cast<bf16*>(b->logits_out);
  f.eos_pre = static_cast<const uint32_t*>(b->eos_projection);
  f.trace = g_frame_trace.load();
  char* ws = static_cast<char*>(workspace);
  f.list = reinterpret_cast<int32_t*>(ws + lo.list);
  f.count = reinterpret_cast<int32_t*>(ws + lo.count);
  f.eos_list = reinterpret_cast<int32_t*>(ws + lo.eos_list);
  f.eos_count = reinterpret_cast<int32_t*>(ws + lo.eos_count);
  f.eos_slot = reinterpret_cast<int32_t*>(ws + lo.eos_slot);
  f.x = reinterpret_cast<bf16*>(ws + lo.x);
  f.q = reinterpret_cast<bf16*>(ws + lo.q);
  f.kc = reinterpret_cast<bf16*>(ws + lo.kc);
  f.vc = reinterpret_cast<bf16*>(ws + lo.vc);
  f.att = reinterpret_cast<bf16*>(ws + lo.att);
  f.h = reinterpret_cast<bf16*>(ws + lo.h);
  f.logits = reinterpret_cast<bf16*>(ws + lo.logits);
  f.tokens = reinterpret_cast<int32_t*>(ws + lo.tokens);
  f.emb_acc = reinterpret_cast<float*>(ws + lo.emb_acc);
  f.ctr = reinterpret_cast<int64_t*>(ws + lo.ctr);
  f.inv = reinterpret_cast<int32_t*>(ws + lo.inv);
  f.eos_partial = reinterpret_cast<float*>(ws + lo.eos_partial);
  f.eos_logit = reinterpret_cast<float*>(ws + lo.eos_logit);
  f.part = reinterpret_cast<float*>(ws + lo.part);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int32_t path = resolve_path(shape, sampling, b->n_streams);
  if (path < 0) return path;
  if (path == MTT_B200_FRAME_PATH_FUSED_CLUSTER) {
    return launch_fused_frame(f, st) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
  }
  if (path == MTT_B200_FRAME_PATH_FUSED_TILE) {
    return launch_tile_frame(f, st) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
  }
  if (path == MTT_B200_FRAME_PATH_FUSED_PAIR) {
    return launch_pair_frame(f, st) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
  }
  if (path == MTT_B200_FRAME_PATH_QUAD) {
    return launch_quad_frame(f, st) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
  }
  if (path == MTT_B200_FRAME_PATH_OCTO) {
    return launch_octo_frame(f, st) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
  }
  if (is_split_path(path)) {
    return launch_split_frame(f, split_of_path(path), rows_of_path(path), st) == cudaSuccess
               ? MTT_B200_STATUS_OK
               : MTT_B200_STATUS_CUDA_ERROR;
  }
  const int d = f.d, F = f.F;
  // Tensor-core layers: LayerNorm rows come out of the kernel before each
  // GEMM (the in-projection / position add, the residual sum of the previous
  // split GEMM, or ln_rows_kernel); the o-projection and FFN2 split K and sum
  // their partials in launch_resid_sum (the benchmark shape: no split, the
  // residual added in the GEMM epilogue).
  const bool tc = tc_linear_supported(f.d, f.F);
  const bool split = !fused_frame_shape(f.d, f.L, f.F);
  const int rows_max = f.n * f.rp;
  const int row_blocks = (rows_max + 7) / 8;
  const int split_o = phase_splits(rows_max, d, d), split_f = phase_splits(rows_max, d, F);
  frame_begin_kernel<<<1, kBeginThreads, 0, st>>>(f);
  for (int p = 0; p < kPositions; ++p) {
    if (in_proj) {
      if (p == 0) {
        launch_linear<kProHidden, kEpiInProj>(f, st, p, 0, d, kEmbed, f.in_w, f.in_b);
      } else {
        launch_linear<kProGather, kEpiInProj>(f, st, p, 0, d, kEmbed, f.in_w, f.in_b);
      }
      if (tc) ln_rows_kernel<<<row_blocks, 256, 0, st>>>(f, f.ln1);
    } else if (tc) {
      // position p >= 1's rows come from the previous position's sampling kernel
      if (p == 0) add_pos_kernel<true><<<row_blocks, 256, 0, st>>>(f, p);
    } else {
      add_pos_kernel<false><<<row_blocks, 256, 0, st>>>(f, p);
    }
    for (int l = 0; l < f.L; ++l) {
      const int64_t dd = static_cast<int64_t>(d) * d;
      const bf16* w1 = f.w1 + static_cast<int64_t>(l) * F * d;
      const bf16* w2 = f.w2 + static_cast<int64_t>(l) * F * d;
      const int warps = f.n * f.rp * f.H;
      if (tc) {
        const bf16* ln2 = f.ln2 + static_cast<int64_t>(l) * d;
        const bf16* ln_next = l + 1 < f.L ? f.ln1 + static_cast<int64_t>(l + 1) * d : nullptr;
        if (launch_linear_tc<kProLn1, kEpiQkv>(f, st, p, l, 3 * d, d, f.qkv + l * 3 * dd, nullptr) != cudaSuccess) {
          return MTT_B200_STATUS_CUDA_ERROR;
        }
        attention_kernel<<<(warps + 7) / 8, 256, 0, st>>>(f, p, l);
        cudaError_t e;
        if (split) {
          e = launch_linear_tc<kProAtt, -1>(f, st, p, l, d, d, f.o + l * dd, nullptr, split_o);
          if (e == cudaSuccess) launch_resid_sum<true>(f, split_o, ln2, st);
        } else {
          e = launch_linear_tc<kProAtt, kEpiResid>(f, st, p, l, d, d, f.o + l * dd, nullptr);
          if (e == cudaSuccess) ln_rows_kernel<<<row_blocks, 256, 0, st>>>(f, ln2);
        }
        if (e == cudaSuccess) e = launch_linear_tc<kProLn2, kEpiGelu>(f, st, p, l, F, d, w1, nullptr);
        if (e == cudaSuccess && split) {
          e = launch_linear_tc<kProH, -1>(f, st, p, l, d, F, w2, nullptr, split_f);
          if (e == cudaSuccess && ln_next != nullptr) {
            launch_resid_sum<true>(f, split_f, ln_next, st);
          } else if (e == cudaSuccess) {
            launch_resid_sum<false>(f, split_f, nullptr, st);
          }
        } else if (e == cudaSuccess) {
          e = launch_linear_tc<kProH, kEpiResid>(f, st, p, l, d, F, w2, nullptr);
          if (e == cudaSuccess && ln_next != nullptr) ln_rows_kernel<<<row_blocks, 256, 0, st>>>(f, ln_next);
        }
        if (e != cudaSuccess) return MTT_B200_STATUS_CUDA_ERROR;
      } else {
        launch_linear<kProLn1, kEpiQkv>(f, st, p, l, 3 * d, d, f.qkv + l * 3 * dd, nullptr);
        attention_kernel<<<(warps + 7) / 8, 256, 0, st>>>(f, p, l);
        launch_linear<kProAtt, kEpiResid>(f, st, p, l, d, d, f.o + l * dd, nullptr);
        launch_linear<kProLn2, kEpiGelu>(f, st, p, l, F, d, w1, nullptr);
        launch_linear<kProH, kEpiResid>(f, st, p, l, d, F, w2, nullptr);
      }
    }
    const bf16* hw = f.head_w + static_cast<int64_t>(p) * kVocab * d;
    const bf16* hb = f.head_b + static_cast<int64_t>(p) * kVocab;
    if (tc && (reinterpret_cast<uintptr_t>(f.head_b) & 15u) == 0) {  // its epilogue reads the bias as 16-byte vectors
      if (launch_linear_tc<kProX, kEpiHead>(f, st, p, 0, kVocab, d, hw, hb) != cudaSuccess) {
        return MTT_B200_STATUS_CUDA_ERROR;
      }
    } else {
      launch_linear<kProX, kEpiHead>(f, st, p, 0, kVocab, d, hw, hb);
    }
    if (tc && !in_proj) {
      sample_kernel<true><<<f.n, kSampleThreads, 0, st>>>(f, p);
    } else {
      sample_kernel<false><<<f.n, kSampleThreads, 0, st>>>(f, p);
    }
  }
  if (f.final_w != nullptr && f.eos_pre == nullptr && launch_eos_projection(frame_eos_args(f), st) != cudaSuccess) {
    return MTT_B200_STATUS_CUDA_ERROR;
  }
  frame_end_kernel<<<f.n, 256, 0, st>>>(f);
  return cudaPeekAtLastError() == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}
