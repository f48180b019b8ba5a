// EOS evaluation for Local AR frames.
//
// Restates eos_projection_kernel / eos_reduce_kernel / eos_finalize_kernel
// (plugins/local_ar_plugins.cu:1372-1495; _reference_eos in
// tools/export/local_ar_wrapper.py:424-476):
//   guided[p][ct] = bf16(bf16(bf16(u + b) * -1.5) + bf16(c + b) * 2.5)
// for the 16 x 2017 compact rows (2016 codes + EOS) of the Main Decoder final
// projection (row p * 2024 + token), where c / u are the conditional and
// unconditional hidden rows' dot products; position p votes EOS when
// guided[p][EOS] > max over the 2016 code logits, or when the sampled token at
// p is EOS; frames vote with any() over their 8 codebooks; the first voting
// frame is end_frame_index (-1 when none).  finished forces 0;
// unfinished || forbid_eos skips evaluation (-1).
//
// Instead of materialising the 16 x 2017 guided logits, each projection
// block reduces its slice of rows to a partial maximum (and the EOS logit when
// its slice holds it); a per-stream reduce kernel finishes the decision.
//
// Kernels live in an anonymous namespace: every translation unit that
// includes this header gets its own copies.
#pragma once

#include "common.cuh"

namespace mtt {
namespace {

constexpr int kEosChunks = 16;                                            // slices per position
constexpr int kEosChunkRows = (kCompactEosVocab + kEosChunks - 1) / kEosChunks;  // 127
constexpr int kEosThreads = 256;

struct EosArgs {
  const __nv_bfloat16* hidden;  // stream s: cond row at hidden + s * hidden_stream_stride
  int64_t hidden_stream_stride;  // elements
  int64_t uncond_offset;         // elements from the cond row to the uncond row (0 without CFG)
  const __nv_bfloat16* weight;   // [16*2024][768]
  const __nv_bfloat16* bias;     // [16*2024]
  float cfg_scale;
  const int32_t* eos_list;   // enabled stream ids
  const int32_t* eos_count;  // number of enabled streams
  float* partial_max;        // [slot][16][kEosChunks]
  float* eos_logit;          // [slot][16]
};

__global__ void __launch_bounds__(kEosThreads) eos_project_kernel(EosArgs a) {
  __shared__ __align__(16) float hs[2][kEmbed];
  __shared__ float warp_max[kEosThreads / 32];
  wait_prior_grid();  // launched after the frame kernel with programmatic serialization
  const int chunk = blockIdx.x;
  const int p = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_enabled = *a.eos_count;
  const int ct0 = chunk * kEosChunkRows;
  const int ct1 = min(kCompactEosVocab, ct0 + kEosChunkRows);
  for (int e = 0; e < n_enabled; ++e) {
    const int s = a.eos_list[e];
    const __nv_bfloat16* h = a.hidden + static_cast<int64_t>(s) * a.hidden_stream_stride;
    __syncthreads();
    for (int k = threadIdx.x; k < kEmbed; k += blockDim.x) {
      hs[0][k] = bf2f(h[k]);
      hs[1][k] = bf2f(h[a.uncond_offset + k]);
    }
    __syncthreads();
    float local_max = -CUDART_INF_F;
    for (int ct = ct0 + warp; ct < ct1; ct += kEosThreads / 32) {
      const int token = ct == kCodebook ? kEosId : ct;
      const int64_t row = static_cast<int64_t>(p) * kVocab + token;
      const __nv_bfloat16* w = a.weight + row * kEmbed;
      float dc = 0.f, du = 0.f;
#pragma unroll
      for (int i = 0; i < kEmbed / 256; ++i) {
        const int k = i * 256 + lane * 8;
        const uint4 wv = *reinterpret_cast<const uint4*>(w + k);
        const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float wf = bf2f(wb[j]);
          dc = fmaf(hs[0][k + j], wf, dc);
          du = fmaf(hs[1][k + j], wf, du);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        dc += __shfl_xor_sync(0xffffffffu, dc, o);
        du += __shfl_xor_sync(0xffffffffu, du, o);
      }
      const float b = bf2f(a.bias[row]);
      const float c = round_bf16(__fadd_rn(dc, b));
      const float u = round_bf16(__fadd_rn(du, b));
      const float us = round_bf16(__fmul_rn(u, __fsub_rn(1.0f, a.cfg_scale)));
      const float g = round_bf16(__fadd_rn(us, __fmul_rn(c, a.cfg_scale)));
      if (ct == kCodebook) {
        if (lane == 0) a.eos_logit[e * kPositions + p] = g;
      } else {
        local_max = fmaxf(local_max, g);
      }
    }
    if (lane == 0) warp_max[warp] = local_max;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m = warp_max[0];
      for (int w = 1; w < kEosThreads / 32; ++w) m = fmaxf(m, warp_max[w]);
      a.partial_max[(e * kPositions + p) * kEosChunks + chunk] = m;
    }
  }
}

// Per-stream EOS decision from the projection partials.
//   tokens: position-major [16] token ids of this stream's frame
// Returns end_frame_index.
__device__ __forceinline__ int eos_decide(const float* partial_max /*[16][kEosChunks]*/, const float* eos_logit,
                                          const int32_t* tokens, bool enabled, bool finished) {
  if (finished) return 0;
  if (!enabled) return -1;
  bool frame_eos[kFrames] = {false, false};
  for (int p = 0; p < kPositions; ++p) {
    float m = -CUDART_INF_F;
    for (int c = 0; c < kEosChunks; ++c) m = fmaxf(m, partial_max[p * kEosChunks + c]);
    const bool argmax_eos = eos_logit[p] > m;
    const bool sampled_eos = tokens[p] == kEosId;
    if (argmax_eos || sampled_eos) frame_eos[p / kCodebooks] = true;
  }
  return frame_eos[0] ? 0 : (frame_eos[1] ? 1 : -1);
}

}  // namespace
}  // namespace mtt
