// Drop-in replacement for local_ar_eos_workspace_size / launch_local_ar_eos
// (plugins/local_ar_plugins.cu:4167-4216): one session, flags read on the
// device, no host synchronisation.
#include "../../include/magpie_tts_rt_b200.h"
#include "eos.cuh"

namespace mtt {
namespace {

// The reference's workspace size: aligned(16 * 2017 * 4, 256) + 2 * 4 bytes.
constexpr size_t kReferenceEosWorkspace = ((static_cast<size_t>(kPositions) * kCompactEosVocab * 4 + 255) & ~size_t(255)) +
                                          2 * sizeof(int32_t);
// This build's use of that workspace.
constexpr size_t kListOffset = 0;         // int32 eos_list[1]
constexpr size_t kCountOffset = 4;        // int32 eos_count
constexpr size_t kPartialOffset = 256;    // float [16][kEosChunks]
constexpr size_t kEosLogitOffset = kPartialOffset + sizeof(float) * kPositions * kEosChunks;  // float [16]
static_assert(kEosLogitOffset + sizeof(float) * kPositions <= kReferenceEosWorkspace, "workspace");

__global__ void dropin_eos_setup_kernel(const bool* unfinished, const bool* finished, const bool* forbid_eos,
                                        int32_t* list, int32_t* count) {
  list[0] = 0;
  count[0] = (!unfinished[0] && !finished[0] && !forbid_eos[0]) ? 1 : 0;
}

__global__ void dropin_eos_finish_kernel(const int64_t* codec_tokens, const bool* finished, const int32_t* count,
                                         const float* partial, const float* eos_logit, int32_t* end_frame_index) {
  int32_t tokens[kPositions];
  for (int p = 0; p < kPositions; ++p) {
    tokens[p] = static_cast<int32_t>(codec_tokens[(p % kCodebooks) * kFrames + p / kCodebooks]);
  }
  end_frame_index[0] = eos_decide(partial, eos_logit, tokens, count[0] != 0, finished[0]);
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API size_t mtt_b200_local_ar_eos_workspace_size(void) { return mtt::kReferenceEosWorkspace; }

extern "C" MTT_B200_API int mtt_b200_launch_local_ar_eos(const void* decoder_hidden_bf16, const int64_t* codec_tokens,
                                                        const bool* unfinished, const bool* finished,
                                                        const bool* forbid_eos, const void* final_weight_bf16,
                                                        const void* final_bias_bf16, void* workspace,
                                                        int32_t* end_frame_index, void* stream) {
  if (!decoder_hidden_bf16 || !codec_tokens || !unfinished || !finished || !forbid_eos || !final_weight_bf16 ||
      !final_bias_bf16 || !workspace || !end_frame_index) {
    return -1;
  }
  using namespace mtt;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int32_t* list = reinterpret_cast<int32_t*>(ws + kListOffset);
  int32_t* count = reinterpret_cast<int32_t*>(ws + kCountOffset);
  float* partial = reinterpret_cast<float*>(ws + kPartialOffset);
  float* eos_logit = reinterpret_cast<float*>(ws + kEosLogitOffset);
  dropin_eos_setup_kernel<<<1, 1, 0, st>>>(unfinished, finished, forbid_eos, list, count);
  EosArgs a;
  a.hidden = static_cast<const __nv_bfloat16*>(decoder_hidden_bf16);
  a.hidden_stream_stride = 2 * kEmbed;
  a.uncond_offset = kEmbed;
  a.weight = static_cast<const __nv_bfloat16*>(final_weight_bf16);
  a.bias = static_cast<const __nv_bfloat16*>(final_bias_bf16);
  a.cfg_scale = 2.5f;
  a.eos_list = list;
  a.eos_count = count;
  a.partial_max = partial;
  a.eos_logit = eos_logit;
  eos_project_kernel<<<dim3(kEosChunks, kPositions), kEosThreads, 0, st>>>(a);
  dropin_eos_finish_kernel<<<1, 1, 0, st>>>(codec_tokens, finished, count, partial, eos_logit, end_frame_index);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}
