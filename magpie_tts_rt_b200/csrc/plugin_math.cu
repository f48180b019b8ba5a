// Drop-in kernels behind the reference's MagpieLayerNorm, MagpieGeluTanh and
// MagpieSoftmax (mode 0) plugins: launch_layer_norm / launch_gelu_tanh /
// launch_softmax (plugins/local_ar_plugins.hpp:57-76, launchers
// plugins/local_ar_plugins.cu:4218-4356).  They reproduce PyTorch 2.11's bf16
// results (docs/engine-contracts.md:231-246), which the reference pins with
// bit-level known-answer tests (tests/plugins/local_ar_plugin_tests.cu:280-408);
// so the reduction orders that decide the bits follow the same steps:
//   * LayerNorm (width 768, no bias, eps 1e-5): 128 threads per row; each
//     thread folds its 4-wide vectors v, v + 128, .. into a Welford
//     (mean, M2, count) in element order, the warp combines by shuffle-down
//     offsets 16..1, the 4 warps by a pairwise tree (warp i + offset into
//     warp i), and out = bf16(w * (rsqrt(M2/768 + eps) * (x - mean)));
//   * GELU-tanh: bf16(0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))));
//   * Softmax over rows of n <= 512 (PyTorch's persistent softmax): row
//     width padded to the next power of two P, min(P, 32) lanes per row, two
//     rows per warp when P <= 128, max and sum by xor-butterfly, expf(x - max),
//     bf16(e / sum) (NaN when the sum is 0).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include "magpie_tts_rt_b200.h"

namespace mtt {
namespace {

constexpr int kNormWidth = 768;
constexpr int kNormVectors = kNormWidth / 4;
constexpr int kNormThreads = 128;  // 32 x 4
constexpr float kNormEps = 1.0e-5f;
constexpr int kMaxNormRows = 2 * 512;
constexpr int kFfnWidth = 3072;
constexpr int kMaxText = 512;
constexpr int kGeluThreads = 256;

struct Welford {
  float mean, m2, count;
};

__device__ __forceinline__ Welford welford_add(Welford w, float x) {
  const float delta = x - w.mean;
  const float count = w.count + 1.0f;
  const float mean = w.mean + delta * (1.0f / count);
  return {mean, w.m2 + delta * (x - mean), count};
}

// Combines b into a (a holds the lower-indexed part).
__device__ __forceinline__ Welford welford_merge(Welford a, Welford b) {
  const float delta = a.mean - b.mean;
  const float count = b.count + a.count;
  if (count <= 0.0f) return {0.0f, 0.0f, 0.0f};
  const float inv = 1.0f / count;
  const float wb = b.count * inv, wa = a.count * inv;
  return {wb * b.mean + wa * a.mean, b.m2 + a.m2 + delta * delta * b.count * wa, count};
}

struct alignas(8) Bf16x4 {
  __nv_bfloat16 v[4];
};

__global__ void __launch_bounds__(kNormThreads) layer_norm_kernel(const __nv_bfloat16* __restrict__ in,
                                                                  const __nv_bfloat16* __restrict__ weight,
                                                                  __nv_bfloat16* __restrict__ out) {
  __shared__ float part[6];  // warps 2..3 (mean, M2) pairs and counts of the tree
  const int t = static_cast<int>(threadIdx.x + threadIdx.y * 32);
  const Bf16x4* row = reinterpret_cast<const Bf16x4*>(in + static_cast<int64_t>(blockIdx.x) * kNormWidth);
  Welford w{0.0f, 0.0f, 0.0f};
  for (int v = t; v < kNormVectors; v += kNormThreads) {
    const Bf16x4 q = row[v];
#pragma unroll
    for (int e = 0; e < 4; ++e) w = welford_add(w, __bfloat162float(q.v[e]));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const Welford o{__shfl_down_sync(0xffffffffu, w.mean, off), __shfl_down_sync(0xffffffffu, w.m2, off),
                    __shfl_down_sync(0xffffffffu, w.count, off)};
    w = welford_merge(w, o);
  }
  // warps: 2 -> 0 and 3 -> 1, then 1 -> 0
  float* mm = part;        // [2][2]
  float* cnt = part + 4;   // [2]
  for (int off = 2; off > 0; off >>= 1) {
    const int y = static_cast<int>(threadIdx.y);
    if (threadIdx.x == 0 && y >= off && y < 2 * off) {
      mm[2 * (y - off)] = w.mean;
      mm[2 * (y - off) + 1] = w.m2;
      cnt[y - off] = w.count;
    }
    __syncthreads();
    if (threadIdx.x == 0 && y < off) w = welford_merge(w, Welford{mm[2 * y], mm[2 * y + 1], cnt[y]});
    __syncthreads();
  }
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    mm[0] = w.mean;
    mm[1] = w.m2 / static_cast<float>(kNormWidth);
  }
  __syncthreads();
  const float mean = mm[0];
  const float rstd = rsqrtf(mm[1] + kNormEps);
  const Bf16x4* wr = reinterpret_cast<const Bf16x4*>(weight);
  Bf16x4* orow = reinterpret_cast<Bf16x4*>(out + static_cast<int64_t>(blockIdx.x) * kNormWidth);
  for (int v = t; v < kNormVectors; v += kNormThreads) {
    const Bf16x4 q = row[v], g = wr[v];
    Bf16x4 r;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float normalized = rstd * (__bfloat162float(q.v[e]) - mean);
      r.v[e] = __float2bfloat16_rn(__bfloat162float(g.v[e]) * normalized);
    }
    orow[v] = r;
  }
}

__global__ void __launch_bounds__(kGeluThreads) gelu_tanh_kernel(const __nv_bfloat16* __restrict__ in,
                                                                 __nv_bfloat16* __restrict__ out, size_t n) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = __bfloat162float(in[i]);
  const float cube = x * x * x;
  const float inner = 0.7978845608028654f * (x + 0.044715f * cube);
  out[i] = __float2bfloat16_rn(0.5f * x * (1.0f + tanhf(inner)));
}

template <int LOG2>
__global__ void softmax_kernel(__nv_bfloat16* out, const __nv_bfloat16* in, int rows, int n) {
  constexpr int P = 1 << LOG2;
  constexpr int LANES = P < 32 ? P : 32;
  constexpr int ITERS = P / LANES;
  constexpr int RPW = P <= 128 ? 2 : 1;  // rows per warp
  const int first = (static_cast<int>(blockDim.y) * static_cast<int>(blockIdx.x) + static_cast<int>(threadIdx.y)) * RPW;
  int local_rows = rows - first;
  if (local_rows > RPW) local_rows = RPW;
  const int lane = static_cast<int>(threadIdx.x);
  in += static_cast<int64_t>(first) * n + lane;
  out += static_cast<int64_t>(first) * n + lane;
  float x[RPW][ITERS];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int len = r >= local_rows ? 0 : n;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      x[r][it] = lane + it * LANES < len ? __bfloat162float(in[r * n + it * LANES]) : -CUDART_INF_F;
    }
  }
  float mx[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    mx[r] = x[r][0];
#pragma unroll
    for (int it = 0; it < ITERS; ++it) mx[r] = mx[r] > x[r][it] ? mx[r] : x[r][it];
  }
#pragma unroll
  for (int off = LANES / 2; off > 0; off /= 2)
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const float o = __shfl_xor_sync(0xffffffffu, mx[r], off, LANES);
      mx[r] = mx[r] < o ? o : mx[r];
    }
  float sum[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    sum[r] = 0.0f;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      x[r][it] = expf(x[r][it] - mx[r]);
      sum[r] += x[r][it];
    }
  }
#pragma unroll
  for (int off = LANES / 2; off > 0; off /= 2)
#pragma unroll
    for (int r = 0; r < RPW; ++r) sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], off, LANES);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    if (r >= local_rows) break;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      if (lane + it * LANES < n) {
        const float v = sum[r] == 0.0f ? CUDART_NAN_F : x[r][it] / sum[r];
        out[r * n + it * LANES] = __float2bfloat16_rn(v);
      }
    }
  }
}

template <int LOG2>
cudaError_t launch_softmax_log2(const __nv_bfloat16* in, __nv_bfloat16* out, int rows, int n, cudaStream_t st) {
  constexpr int P = 1 << LOG2;
  constexpr int LANES = P < 32 ? P : 32;
  constexpr int RPW = P <= 128 ? 2 : 1;
  constexpr int WARPS = 128 / LANES;  // 128 threads per block
  const int per_block = WARPS * RPW;
  softmax_kernel<LOG2><<<(rows + per_block - 1) / per_block, dim3(LANES, WARPS), 0, st>>>(out, in, rows, n);
  return cudaPeekAtLastError();
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API int mtt_b200_launch_layer_norm(const void* input, const void* weight, void* output,
                                                      int32_t row_count, void* stream) {
  if (input == nullptr || weight == nullptr || output == nullptr || row_count < 1 || row_count > mtt::kMaxNormRows) {
    return -1;
  }
  mtt::layer_norm_kernel<<<row_count, dim3(32, 4), 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(input), static_cast<const __nv_bfloat16*>(weight),
      static_cast<__nv_bfloat16*>(output));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

extern "C" MTT_B200_API int mtt_b200_launch_gelu_tanh(const void* input, void* output, size_t element_count,
                                                     void* stream) {
  const size_t max_elements = static_cast<size_t>(mtt::kFfnWidth) * mtt::kMaxText;
  if (input == nullptr || output == nullptr || element_count == 0 || element_count > max_elements) return -1;
  const size_t blocks = (element_count + mtt::kGeluThreads - 1) / mtt::kGeluThreads;
  mtt::gelu_tanh_kernel<<<static_cast<unsigned>(blocks), mtt::kGeluThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(input), static_cast<__nv_bfloat16*>(output), element_count);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

extern "C" MTT_B200_API int mtt_b200_launch_softmax(const void* input, void* output, int32_t batch_count,
                                                   int32_t element_count, void* stream) {
  if (input == nullptr || output == nullptr || batch_count < 1 || element_count < 1 ||
      element_count > mtt::kMaxText) {
    return -1;
  }
  int log2 = 0;
  while ((1 << log2) < element_count) ++log2;
  const auto* in = static_cast<const __nv_bfloat16*>(input);
  auto* out = static_cast<__nv_bfloat16*>(output);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (log2) {
    case 0: e = mtt::launch_softmax_log2<0>(in, out, batch_count, element_count, st); break;
    case 1: e = mtt::launch_softmax_log2<1>(in, out, batch_count, element_count, st); break;
    case 2: e = mtt::launch_softmax_log2<2>(in, out, batch_count, element_count, st); break;
    case 3: e = mtt::launch_softmax_log2<3>(in, out, batch_count, element_count, st); break;
    case 4: e = mtt::launch_softmax_log2<4>(in, out, batch_count, element_count, st); break;
    case 5: e = mtt::launch_softmax_log2<5>(in, out, batch_count, element_count, st); break;
    case 6: e = mtt::launch_softmax_log2<6>(in, out, batch_count, element_count, st); break;
    case 7: e = mtt::launch_softmax_log2<7>(in, out, batch_count, element_count, st); break;
    case 8: e = mtt::launch_softmax_log2<8>(in, out, batch_count, element_count, st); break;
    case 9: e = mtt::launch_softmax_log2<9>(in, out, batch_count, element_count, st); break;
    default: return -1;
  }
  return e == cudaSuccess ? 0 : -1;
}
