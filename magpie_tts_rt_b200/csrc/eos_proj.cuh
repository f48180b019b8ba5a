// EOS projection as one tensor-core GEMM over every session that needs it.
//
// The reference evaluates EOS per session with a 32,272-CTA GEMV over the
// 16 x 2017 compact rows of the Main Decoder final projection
// (plugins/local_ar_plugins.cu:1372-1432, launcher :4167-4216;
// _reference_eos in tools/export/local_ar_wrapper.py:424-476).  Here the
// sessions' conditional and unconditional hidden rows are gathered into a
// compact [2 n][768] block and multiplied by the whole [16 x 2024][768]
// projection on tcgen05 (gemm_tc.cuh: weight rows as M, the 2 n session rows
// as N), so the 49.6 MB of weights stream once per 128 sessions instead of
// once per session.  The epilogue forms the guided logits with the
// reference's roundings,
//   c = bf16(dot(h_c, w) + b), u = bf16(dot(h_u, w) + b),
//   g = bf16(bf16(u (1 - cfg)) + c cfg),
// and reduces them on the fly: per (session, position) the largest guided
// code logit (tokens 0..2015) as an order-preserving key (atomic max) and
// the EOS logit (token 2017) as a value.  Tokens 2016 and 2018..2023 are
// outside the compact rows and ignored.
#pragma once

#include "common.cuh"

namespace mtt {

// Order-preserving 32-bit key of a float (larger float, larger key); 0 is
// below every key and stands for "no value" (-inf).
__host__ __device__ __forceinline__ uint32_t order_key(float f) {
#ifdef __CUDA_ARCH__
  const uint32_t u = __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  if (k == 0u) return -CUDART_INF_F;
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// The EOS decision of one session from its projection (max_key / eos_logit:
// [16] each) and its 16 position-major tokens: position p votes EOS when
// its guided EOS logit is above every guided code logit or when its sampled
// token is EOS; frames vote with any() over their 8 codebooks; the first
// voting frame is the end frame (-1: none).  finished forces 0, a session
// with EOS disabled gives -1 (local_ar_plugins.cu:1434-1495).
__device__ __forceinline__ int eos_decide_proj(const uint32_t* max_key, const float* eos_logit, const int32_t* tokens,
                                               bool enabled, bool finished) {
  if (finished) return 0;
  if (!enabled) return -1;
  bool frame_eos[kFrames] = {false, false};
  for (int p = 0; p < kPositions; ++p) {
    const bool argmax_eos = eos_logit[p] > key_value(max_key[p]);
    const bool sampled_eos = tokens[p] == kEosId;
    if (argmax_eos || sampled_eos) frame_eos[p / kCodebooks] = true;
  }
  return frame_eos[0] ? 0 : (frame_eos[1] ? 1 : -1);
}

struct EosProjArgs {
  const __nv_bfloat16* hidden;  // session s: conditional row at hidden + s * hidden_stream_stride
  int64_t hidden_stream_stride;  // elements
  int64_t uncond_offset;         // elements from the conditional to the unconditional row (0: no CFG)
  const int32_t* list;           // optional: slot e projects session list[e] (null: session e)
  const int32_t* count;          // optional device count of slots (null: n_max)
  int n_max;                     // largest slot count (grid and map sizing)
  const __nv_bfloat16* weight;   // [16 x 2024][768]
  const __nv_bfloat16* bias;     // [16 x 2024]
  float cfg_scale;               // 1 without CFG
  __nv_bfloat16* rows;           // scratch: [2 n_max][768], 16-byte aligned
  uint32_t* max_key;             // out [slot][16], slot stride proj_stride
  float* eos_logit;              // out [slot][16], slot stride proj_stride
  int proj_stride;               // 32-bit words between consecutive slots (16: separate arrays)
  int32_t* status;               // out: set to 1 when a bounded wait of the GEMM gave up (zeroed here)
};

// Gathers the rows and clears the maxima (one launch), then runs the GEMM
// (one launch); both with programmatic stream serialization.
cudaError_t launch_eos_projection(const EosProjArgs& a, cudaStream_t stream);

}  // namespace mtt
