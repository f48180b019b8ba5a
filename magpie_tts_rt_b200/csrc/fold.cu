// One-time weight transform: the Local AR in-projection folded into the
// audio embedding tables.  Position p >= 1 of a frame feeds the Local
// Transformer with in_proj(table_{p-1}[token]) (magpietts_modules.py:666-667,
// local_ar_wrapper.py:744-746); both factors are weights, so
//   emb_proj[q][v][n] = bf16(sum_k table_q[v][k] * W_in[n][k] + b_in[n])
// is computed once, with the same f32 accumulation and single bf16 rounding
// the per-position product has, and the frame gathers one d-wide row.
#include "../../include/magpie_tts_rt_b200.h"
#include "common.cuh"

namespace mtt {
namespace {

constexpr int kFoldRows = 16;  // vocabulary rows per block
constexpr int kFoldThreads = 256;

// grid (ceil(2024 / 16), 16 tables); each thread: one output feature n for 16 rows.
__global__ void __launch_bounds__(kFoldThreads) fold_kernel(const __nv_bfloat16* emb, const __nv_bfloat16* w,
                                                            const __nv_bfloat16* b, __nv_bfloat16* out, int d) {
  __shared__ float rows[kFoldRows][kEmbed];
  const int q = blockIdx.y;
  const int v0 = blockIdx.x * kFoldRows;
  for (int i = threadIdx.x; i < kFoldRows * kEmbed; i += blockDim.x) {
    const int r = i / kEmbed, k = i % kEmbed;
    rows[r][k] = v0 + r < kVocab ? bf2f(emb[(static_cast<int64_t>(q) * kVocab + v0 + r) * kEmbed + k]) : 0.f;
  }
  __syncthreads();
  for (int n = threadIdx.x; n < d; n += blockDim.x) {
    float acc[kFoldRows];
#pragma unroll
    for (int r = 0; r < kFoldRows; ++r) acc[r] = 0.f;
    const __nv_bfloat16* wr = w + static_cast<int64_t>(n) * kEmbed;
    for (int k = 0; k < kEmbed; k += 8) {
      const uint4 wv = *reinterpret_cast<const uint4*>(wr + k);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float wf = bf2f(wb[j]);
#pragma unroll
        for (int r = 0; r < kFoldRows; ++r) acc[r] = fmaf(rows[r][k + j], wf, acc[r]);
      }
    }
    const float bias = bf2f(b[n]);
#pragma unroll
    for (int r = 0; r < kFoldRows; ++r) {
      if (v0 + r < kVocab) out[(static_cast<int64_t>(q) * kVocab + v0 + r) * d + n] = f2bf(__fadd_rn(acc[r], bias));
    }
  }
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API size_t mtt_b200_fold_in_projection_bytes(const mtt_b200_local_ar_shape_t* shape) {
  if (shape == nullptr || shape->d_model <= 0 || shape->d_model == mtt::kEmbed) return 0;
  return static_cast<size_t>(mtt::kPositions) * mtt::kVocab * shape->d_model * sizeof(__nv_bfloat16);
}

extern "C" MTT_B200_API int mtt_b200_launch_fold_in_projection(const mtt_b200_local_ar_shape_t* shape,
                                                              const mtt_b200_local_ar_weights_t* w, void* out,
                                                              void* stream) {
  if (shape == nullptr || w == nullptr || out == nullptr || shape->d_model <= 0 || shape->d_model == mtt::kEmbed ||
      shape->d_model % 8 != 0 || w->emb == nullptr || w->in_proj_w == nullptr || w->in_proj_b == nullptr) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  const dim3 grid((mtt::kVocab + mtt::kFoldRows - 1) / mtt::kFoldRows, mtt::kPositions);
  mtt::fold_kernel<<<grid, mtt::kFoldThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w->emb), static_cast<const __nv_bfloat16*>(w->in_proj_w),
      static_cast<const __nv_bfloat16*>(w->in_proj_b), static_cast<__nv_bfloat16*>(out), shape->d_model);
  return cudaPeekAtLastError() == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}
