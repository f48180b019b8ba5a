// Drop-in replacement for launch_finalize_local_step
// (src/runtime/synthesis_kernels.cu:53-86,177-214): commit one Local AR
// step's tokens into the [8][8] batch aggregate and its diagnostics into the
// step slots, advance the canonical RNG counter and latch EOS.
#include "../../include/magpie_tts_rt_b200.h"
#include "common.cuh"

namespace mtt {
namespace {

constexpr uint32_t kSteadyFrames = 8;

__global__ void finalize_local_step_kernel(const int64_t* step_codec_tokens, int64_t* aggregate,
                                           uint32_t frame_offset, const int32_t* canonical_invalid,
                                           const int32_t* canonical_end, int32_t* step_invalid,
                                           int32_t* step_end, const int64_t* updated_counter,
                                           int64_t* counter, bool* generation_finished) {
  const uint32_t i = threadIdx.x;
  if (i < kCodebooks * kFrames) {
    const uint32_t codebook = i / kFrames, frame = i % kFrames;
    aggregate[codebook * kSteadyFrames + frame_offset + frame] = step_codec_tokens[i];
  }
  if (i == 0) {
    const int32_t end = canonical_end[0];
    step_invalid[0] = canonical_invalid[0];
    step_end[0] = end;
    counter[0] = updated_counter[0];
    if (end == 0 || end == 1) generation_finished[0] = true;
  }
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API int mtt_b200_launch_finalize_local_step(
    const int64_t* step_codec_tokens, int64_t* aggregate_codec_tokens, uint32_t frame_offset,
    const int32_t* canonical_invalid_rows, const int32_t* canonical_end_frame_index,
    int32_t* step_invalid_rows, int32_t* step_end_frame_index, const int64_t* updated_rng_counter,
    int64_t* rng_counter, bool* generation_finished, void* stream) {
  if (!step_codec_tokens || !aggregate_codec_tokens || frame_offset > mtt::kSteadyFrames - mtt::kFrames ||
      frame_offset % mtt::kFrames != 0 || !canonical_invalid_rows || !canonical_end_frame_index ||
      !step_invalid_rows || !step_end_frame_index || !updated_rng_counter || !rng_counter ||
      !generation_finished) {
    return -1;
  }
  mtt::finalize_local_step_kernel<<<1, mtt::kCodebooks * mtt::kFrames, 0, static_cast<cudaStream_t>(stream)>>>(
      step_codec_tokens, aggregate_codec_tokens, frame_offset, canonical_invalid_rows, canonical_end_frame_index,
      step_invalid_rows, step_end_frame_index, updated_rng_counter, rng_counter, generation_finished);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}
