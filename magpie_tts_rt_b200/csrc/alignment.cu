// The alignment (attention-prior) controller and the Local AR's EOS inputs,
// batched over sessions: one warp per session, every load of a step issued
// at once.
//
// Reference: src/runtime/alignment_kernel.cu:16-154 -- one 256-thread CTA
// per launch for one utterance, its thread 0 walking the search window, the
// text row and the counter array serially -- called once per Main Decoder
// step by SynthesisPipeline::advance_alignment (synthesis_pipeline.cpp:
// 496-509).  The Local AR inputs the pipeline then prepares on the host
// (forbid_eos = generated_decoder_steps < 2, an H2D copy, and the D2D copy of
// `unfinished`; synthesis_pipeline.cpp:511-530) and the `finished` latch of
// launch_finalize_local_step (synthesis_kernels.cu:79-84) are produced here
// on the device, so a decoder step needs no host round trip between the
// alignment and the Local AR frame.
//
// Per session the warp reads, in one wave of independent loads, the
// conditional score row (<= 512 bf16 = 1 KB: two 16-byte chunks per lane),
// the visit counters (<= 512 u32 = 2 KB: four chunks per lane) and the
// scalars, then resolves everything with shuffles: the counter of the last
// attended token and of the new one come from their owner lanes, the window
// argmax and the last sink position are warp reductions.  Writes: the prior
// (two rows), one counter, five scalars.  The unconditional score row is
// never read, as in the reference.
#include "../../include/magpie_tts_rt_b200.h"
#include "common.cuh"

namespace mtt {
namespace {

constexpr uint32_t kMaxText = 512;            // alignment_kernel.cu:12
constexpr uint32_t kU32Max = 0xFFFFFFFFu;
constexpr int kAlignWarps = 4;                // sessions per CTA
constexpr int kRowChunks = kMaxText / 8 / 32;    // 16-byte score chunks per lane
constexpr int kCountChunks = kMaxText / 4 / 32;  // 16-byte counter chunks per lane

struct AlignArgs {
  int n;
  uint32_t stride;    // elements between a session's score / prior rows; its counter row
  uint32_t single_t;  // text length when text_length == nullptr
  uint32_t ignored, short_max, lookahead, sink;
  const uint32_t* text_length;
  const bool* active;
  const uint16_t* scores;
  uint32_t* counters;
  uint32_t* last_attended;
  uint16_t* prior;
  int64_t* attended;
  bool* unfinished;
  int32_t* invalid;
  int64_t* steps;
  bool* forbid;
  const int32_t* end_frame;
  bool* finished;
};

__device__ __forceinline__ bool bf16_finite(uint32_t b) { return (b & 0x7F80u) != 0x7F80u; }

// Element e (0..7) of a 16-byte chunk of bf16 values.
__device__ __forceinline__ uint32_t chunk_u16(const uint4& c, int e) {
  const uint32_t w = e < 2 ? c.x : e < 4 ? c.y : e < 6 ? c.z : c.w;
  return (e & 1) ? (w >> 16) : (w & 0xFFFFu);
}
__device__ __forceinline__ uint32_t chunk_u32(const uint4& c, int e) {
  return e == 0 ? c.x : e == 1 ? c.y : e == 2 ? c.z : c.w;
}

// Chunks of the elements below `lim`.  kVec: rows start 16-byte aligned and
// lim (the stride, capped at 512) is a multiple of 8, so whole 16-byte chunks
// are loaded; else element loads.
template <bool kVec>
__device__ __forceinline__ uint4 load_row_chunk(const uint16_t* row, uint32_t first, uint32_t lim) {
  if (first >= lim) return make_uint4(0, 0, 0, 0);
  if constexpr (kVec) return __ldg(reinterpret_cast<const uint4*>(row + first));
  uint32_t h[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) h[e] = first + e < lim ? row[first + e] : 0u;
  return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
}
template <bool kVec>
__device__ __forceinline__ uint4 load_count_chunk(const uint32_t* cnt, uint32_t first, uint32_t lim) {
  if (first >= lim) return make_uint4(0, 0, 0, 0);
  if constexpr (kVec) return *reinterpret_cast<const uint4*>(cnt + first);
  uint32_t h[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = first + e < lim ? cnt[first + e] : 0u;
  return make_uint4(h[0], h[1], h[2], h[3]);
}

// counters[i] from the lane that loaded it (i < t).
__device__ __forceinline__ uint32_t counter_at(const uint4 (&c)[kCountChunks], uint32_t i) {
  const uint32_t chunk = i >> 2, owner = chunk & 31u, j = chunk >> 5, e = i & 3u;
  uint32_t v = 0;
#pragma unroll
  for (int jj = 0; jj < kCountChunks; ++jj) {
    if (static_cast<uint32_t>(jj) == j) v = chunk_u32(c[jj], static_cast<int>(e));
  }
  return __shfl_sync(0xFFFFFFFFu, v, static_cast<int>(owner));
}

template <bool kVec>
__global__ void __launch_bounds__(kAlignWarps * 32) alignment_gate_kernel(const AlignArgs a) {
  const uint32_t lane = threadIdx.x & 31u;
  const int s = static_cast<int>(blockIdx.x) * kAlignWarps + static_cast<int>(threadIdx.x >> 5);
  if (s >= a.n) return;

  // Every load of the step is issued before any is used: the session's
  // scalars and its score / counter chunks -- up to the stride on the 16-byte
  // path (in bounds whatever the text length; entries past it are masked
  // below), up to the text length on the element path.
  const bool act = a.active == nullptr || a.active[s];
  const uint32_t t = a.text_length != nullptr ? a.text_length[s] : a.single_t;
  const uint32_t la = a.last_attended[s];
  const int64_t steps = a.steps != nullptr ? a.steps[s] : 0;
  const int32_t end_frame = a.end_frame != nullptr ? a.end_frame[s] : -1;
  const size_t base = static_cast<size_t>(s) * 2u * a.stride;
  const uint16_t* row = a.scores + base;
  uint32_t* cnt = a.counters + static_cast<size_t>(s) * a.stride;
  const uint32_t lim = kVec ? min(a.stride, kMaxText) : min(min(t, a.stride), kMaxText);
  uint4 rc[kRowChunks], cc[kCountChunks];
#pragma unroll
  for (int j = 0; j < kRowChunks; ++j) rc[j] = load_row_chunk<kVec>(row, 8u * (lane + 32u * j), lim);
#pragma unroll
  for (int j = 0; j < kCountChunks; ++j) cc[j] = load_count_chunk<kVec>(cnt, 4u * (lane + 32u * j), lim);
  if (!act) return;

  // Local AR EOS inputs, whatever the alignment outcome (the host computes
  // them unconditionally, synthesis_pipeline.cpp:525-569).
  if (lane == 0) {
    if (a.steps != nullptr) {
      a.forbid[s] = steps < 2;
      a.steps[s] = steps + 1;
    }
    if (a.end_frame != nullptr && (end_frame == 0 || end_frame == 1)) a.finished[s] = true;
  }

  // alignment_kernel.cu:33-37 (t > stride: rows would overlap, also rejected)
  if (t == 0 || t > kMaxText || t > a.stride || t <= a.ignored || a.lookahead == 0 || a.sink == 0) {
    if (lane == 0) a.invalid[s] = 1;
    return;
  }

  // search window (alignment_kernel.cu:39-59)
  bool invalid = false;
  uint32_t ss = la;
  if (counter_at(cc, min(la, t - 1u)) >= a.sink) {
    if (ss == kU32Max) invalid = true;
    else ++ss;
  }
  ss = min(ss, t);
  const uint32_t content_end = t - a.ignored;
  const uint32_t window_end = static_cast<uint32_t>(
      min(min(static_cast<uint64_t>(ss) + a.lookahead, static_cast<uint64_t>(kU32Max)),
          static_cast<uint64_t>(content_end)));

  // non-finite anywhere in the row, and the window argmax
  // (alignment_kernel.cu:61-88).  The serial scan seeds `best` with the
  // window's first entry even when it is non-finite and skips later
  // non-finite entries; so a NaN or +inf first entry holds the window, and
  // otherwise the result is the left-most maximum over the first entry and
  // the finite rest.
  bool bad = false;
  float bv = -CUDART_INF_F;
  uint32_t bi = kU32Max;
#pragma unroll
  for (int j = 0; j < kRowChunks; ++j) {
    const uint32_t first = 8u * (lane + 32u * j);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t i = first + e;
      const uint32_t b = chunk_u16(rc[j], e);
      const bool fin = bf16_finite(b);
      if (i < t && !fin) bad = true;
      if (i >= ss && i < window_end && (fin || i == ss)) {
        const float v = bits2f(static_cast<uint16_t>(b));
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad)) invalid = true;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  uint32_t att = t - 1u;
  if (window_end > ss) {
    // the first entry's own bits decide whether it holds the window
    const uint32_t fb = [&] {
      const uint32_t chunk = ss >> 3, owner = chunk & 31u, j = chunk >> 5, e = ss & 7u;
      uint32_t v = 0;
#pragma unroll
      for (int jj = 0; jj < kRowChunks; ++jj) {
        if (static_cast<uint32_t>(jj) == j) {
#pragma unroll
          for (int ee = 0; ee < 8; ++ee) {
            if (static_cast<uint32_t>(ee) == e) v = chunk_u16(rc[jj], ee);
          }
        }
      }
      return __shfl_sync(0xFFFFFFFFu, v, static_cast<int>(owner));
    }();
    const bool holds = (fb & 0x7FFFu) > 0x7F80u || fb == 0x7F80u;  // NaN or +inf
    att = holds ? ss : bi;
  }

  // sinks: the last index whose count, after this step's increment, reaches
  // the threshold (alignment_kernel.cu:90-104)
  const uint32_t c_att = counter_at(cc, att);
  if (c_att == kU32Max) invalid = true;
  int msp = -1;
#pragma unroll
  for (int j = 0; j < kCountChunks; ++j) {
    const uint32_t first = 4u * (lane + 32u * j);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t i = first + e;
      uint32_t c = chunk_u32(cc[j], e);
      if (i == att && c != kU32Max) ++c;
      if (i < t && c >= a.sink) msp = static_cast<int>(i);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) msp = max(msp, __shfl_xor_sync(0xFFFFFFFFu, msp, off));

  if (lane == 0) {
    if (c_att != kU32Max) cnt[att] = c_att + 1u;
    a.last_attended[s] = att;
    a.attended[s] = static_cast<int64_t>(att);
    a.unfinished[s] = att < content_end;
    a.invalid[s] = invalid ? 1 : 0;
  }
  if (invalid) return;

  // next prior [2][t] (alignment_kernel.cu:115-153): epsilon, and in the
  // conditional row 1.0 at the history, attended and look-ahead tokens (or
  // everywhere for short texts) past the last sink
  const uint32_t history = max(att == 0 ? 0u : att - 1u, min(1u, t - 1u));
  const uint32_t ahead = static_cast<uint32_t>(min(static_cast<uint64_t>(att) + a.lookahead,
                                                   static_cast<uint64_t>(t - 1u)));
  const bool all_one = t <= a.short_max;
  const uint32_t eps = __bfloat16_as_ushort(__float2bfloat16_rn(0.1f));
  const uint32_t one = __bfloat16_as_ushort(__float2bfloat16_rn(1.0f));
  uint16_t* p0 = a.prior + base;
  uint16_t* p1 = p0 + a.stride;
  for (uint32_t first = 8u * lane; first < t; first += 256u) {
    uint32_t h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t i = first + e;
      const bool on = all_one || i == history || (i >= att && i <= ahead);
      h[e] = (on && static_cast<int>(i) > msp) ? one : eps;
    }
    if (kVec && first + 8u <= t) {
      *reinterpret_cast<uint4*>(p0 + first) =
          make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
      *reinterpret_cast<uint4*>(p1 + first) = make_uint4(eps * 0x10001u, eps * 0x10001u, eps * 0x10001u,
                                                         eps * 0x10001u);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (first + e < t) {
          p0[first + e] = static_cast<uint16_t>(h[e]);
          p1[first + e] = static_cast<uint16_t>(eps);
        }
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t launch_gate(const AlignArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return cudaSuccess;
  const bool vec = a.stride % 8u == 0 && aligned16(a.scores) && aligned16(a.prior) && aligned16(a.counters);
  const dim3 grid(static_cast<unsigned>((a.n + kAlignWarps - 1) / kAlignWarps));
  if (vec) alignment_gate_kernel<true><<<grid, kAlignWarps * 32, 0, stream>>>(a);
  else alignment_gate_kernel<false><<<grid, kAlignWarps * 32, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API int mtt_b200_launch_alignment_controller(
    const void* alignment_scores_bf16, const mtt_b200_alignment_contract_t* contract, uint32_t* counters,
    uint32_t* last_attended, void* next_prior_bf16, int64_t* attended_token_index, bool* unfinished_text,
    int32_t* invalid_state, void* stream) {
  if (alignment_scores_bf16 == nullptr || contract == nullptr || counters == nullptr || last_attended == nullptr ||
      next_prior_bf16 == nullptr || attended_token_index == nullptr || unfinished_text == nullptr ||
      invalid_state == nullptr) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  mtt::AlignArgs a{};
  a.n = 1;
  a.single_t = contract->text_length;
  a.stride = contract->text_length;  // scores [2][T], prior [2][1][T], counters [T]
  a.ignored = contract->ignored_terminal_tokens;
  a.short_max = contract->short_text_no_prior_max_tokens;
  a.lookahead = contract->lookahead;
  a.sink = contract->sink_threshold;
  a.scores = static_cast<const uint16_t*>(alignment_scores_bf16);
  a.counters = counters;
  a.last_attended = last_attended;
  a.prior = static_cast<uint16_t*>(next_prior_bf16);
  a.attended = attended_token_index;
  a.unfinished = unfinished_text;
  a.invalid = invalid_state;
  return static_cast<int>(mtt::launch_gate(a, static_cast<cudaStream_t>(stream)));
}

extern "C" MTT_B200_API int mtt_b200_launch_alignment_batch(const mtt_b200_alignment_batch_t* b, void* stream) {
  if (b == nullptr || b->n_sessions < 0) return MTT_B200_STATUS_INVALID_ARGUMENT;
  if (b->n_sessions == 0) return MTT_B200_STATUS_OK;
  if (b->token_stride == 0 || b->text_length == nullptr || b->alignment_scores == nullptr ||
      b->counters == nullptr || b->last_attended == nullptr || b->next_prior == nullptr ||
      b->attended_token_index == nullptr || b->unfinished == nullptr || b->invalid_state == nullptr ||
      (b->decoder_steps == nullptr) != (b->forbid_eos == nullptr) ||
      (b->end_frame_index == nullptr) != (b->finished == nullptr)) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  mtt::AlignArgs a{};
  a.n = b->n_sessions;
  a.stride = b->token_stride;
  a.ignored = b->ignored_terminal_tokens;
  a.short_max = b->short_text_no_prior_max_tokens;
  a.lookahead = b->lookahead;
  a.sink = b->sink_threshold;
  a.text_length = b->text_length;
  a.active = b->active;
  a.scores = static_cast<const uint16_t*>(b->alignment_scores);
  a.counters = b->counters;
  a.last_attended = b->last_attended;
  a.prior = static_cast<uint16_t*>(b->next_prior);
  a.attended = b->attended_token_index;
  a.unfinished = b->unfinished;
  a.invalid = b->invalid_state;
  a.steps = b->decoder_steps;
  a.forbid = b->forbid_eos;
  a.end_frame = b->end_frame_index;
  a.finished = b->finished;
  return mtt::launch_gate(a, static_cast<cudaStream_t>(stream)) == cudaSuccess ? MTT_B200_STATUS_OK
                                                                               : MTT_B200_STATUS_CUDA_ERROR;
}
