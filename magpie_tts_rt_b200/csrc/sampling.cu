// Sampling launchers: the drop-in replacement for launch_local_ar_sampling
// (plugins/local_ar_plugins.cu:4127-4165) and device test hooks.
#include "../../include/magpie_tts_rt_b200.h"
#include "sampling.cuh"

namespace mtt {
namespace {

// One session, one position: the reference plugin's I/O (grid 1, 256 threads).
__global__ void __launch_bounds__(kSampleThreads) dropin_sampling_kernel(
    const uint16_t* logits, const bool* unfinished, const bool* finished, const bool* forbid_eos,
    const int64_t* rng_seed, const int64_t* rng_counter, const __nv_bfloat16* embedding,
    int64_t* sampled_token, __nv_bfloat16* next_embedding, int64_t* updated_rng_counter,
    int32_t* invalid_rows) {
  __shared__ SampleShared sh;
  __shared__ __align__(16) unsigned char scratch[kSampleScratchBytes];
  SampleCall c;
  c.logits = logits;
  c.uncond_offset = kVocab;
  c.kind = kLogitsBf16Cfg;
  c.unfinished = unfinished[0];
  c.finished = finished[0];
  c.forbid_eos = forbid_eos[0];
  c.seed = rng_seed[0];
  c.counter = rng_counter[0];
  int invalid = 0;
  const SamplingParams reference_params{80, 0.6f, 2.5f, 0};  // local_ar_plugins.cu:41-43
  const int token = sample_block(c, reference_params, sh, scratch, &invalid);
  if (threadIdx.x == 0) {
    const bool counter_valid = c.counter >= 0 && c.counter <= kMaxCounter;
    sampled_token[0] = token;
    updated_rng_counter[0] = counter_valid ? c.counter + 1 : c.counter;
    invalid_rows[0] = invalid;
  }
  const __nv_bfloat16* row = embedding + static_cast<int64_t>(token) * kEmbed;
  for (int w = threadIdx.x; w < kEmbed; w += blockDim.x) {
    const __nv_bfloat16 v = row[w];
    next_embedding[w] = v;
    next_embedding[kEmbed + w] = v;
  }
}

__global__ void test_gumbel_kernel(const float* u, float* g, size_t n) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) g[i] = clamped_gumbel(u[i]);
}

__global__ void test_log_kernel(const float* x, float* y, size_t n) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    y[i] = log_cr(x[i]);
  }
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API int mtt_b200_launch_local_ar_sampling(
    const void* logits_bf16, const bool* unfinished, const bool* finished, const bool* forbid_eos,
    const int64_t* rng_seed, const int64_t* rng_counter, const void* embedding_weight_bf16,
    int64_t* sampled_token, void* next_embedding_bf16, int64_t* updated_rng_counter,
    int32_t* invalid_rows, void* stream) {
  if (!logits_bf16 || !unfinished || !finished || !forbid_eos || !rng_seed || !rng_counter ||
      !embedding_weight_bf16 || !sampled_token || !next_embedding_bf16 || !updated_rng_counter ||
      !invalid_rows) {
    return -1;
  }
  mtt::dropin_sampling_kernel<<<1, mtt::kSampleThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(logits_bf16), unfinished, finished, forbid_eos, rng_seed, rng_counter,
      static_cast<const __nv_bfloat16*>(embedding_weight_bf16), sampled_token,
      static_cast<__nv_bfloat16*>(next_embedding_bf16), updated_rng_counter, invalid_rows);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

extern "C" MTT_B200_API int mtt_b200_launch_test_clamped_gumbel(const float* uniform, float* gumbel,
                                                                size_t count, void* stream) {
  if (!uniform || !gumbel || count == 0) return -1;
  const unsigned blocks = static_cast<unsigned>((count + 255) / 256);
  mtt::test_gumbel_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(uniform, gumbel, count);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

extern "C" MTT_B200_API int mtt_b200_launch_test_log(const float* x, float* out, size_t count, void* stream) {
  if (!x || !out || count == 0) return -1;
  mtt::test_log_kernel<<<148 * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, out, count);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}
