// Frame description shared by the two batched-frame implementations
// (phase kernels in frame.cu, fused cluster kernel in frame_fused.cu).
#pragma once

#include <algorithm>

#include <cuda.h>

#include <cstddef>

#include "common.cuh"
#include "eos.cuh"
#include "eos_proj.cuh"

namespace mtt {

using bf16 = __nv_bfloat16;

struct Frame {
  int d, L, H, F, rp, n, in_proj;
  SamplingParams prm;
  const bf16 *in_w, *in_b, *pos, *ln1, *qkv, *o, *ln2, *w1, *w2, *head_w, *head_b, *emb, *final_w, *final_b;
  const bf16* emb_proj;  // optional folded in-projection tables [16][2024][d]
  const bf16* hidden;
  const bool *unfinished, *finished, *forbid, *active;
  const int64_t* seed;
  int64_t* counter_io;
  int64_t* codec_tokens;
  int codec_stride, codec_offset;  // frames per codebook row of codec_tokens, first frame written
  bool* finished_latch;            // optional: set where the frame's EOS decision ends the utterance
  int32_t* codec_frames;           // optional: audio frames in the emission aggregate (see commit_end)
  int32_t* invalid_rows;
  int32_t* end_frame;
  bf16* next_emb;
  const int64_t* forced;
  bf16* logits_out;
  const uint32_t* eos_pre;  // optional [n][32]: the EOS projection from the Main Decoder step
  uint64_t* trace;          // optional phase clock stamps of the first CTA (fused cluster kernel)
  // workspace
  int32_t *list, *count, *eos_list, *eos_count, *eos_slot;
  bf16 *x, *q, *kc, *vc, *att, *h, *logits;
  int32_t* tokens;
  float* emb_acc;
  int64_t* ctr;
  int32_t* inv;
  float *eos_partial, *eos_logit;
  float* part;  // phase kernels: f32 partial sums of the split residual GEMMs
};

// Position p of session s in codec_tokens: codebook p % 8, frame p / 8 of
// this frame call, frames codec_offset + {0, 1} of a row codec_stride frames
// wide ([n][8][2] by default, or the [n][8][8] emission aggregate that
// finalize_local_step assembles, synthesis_kernels.cu:53-86).
__device__ __forceinline__ int64_t codec_index(const Frame& f, int s, int p) {
  return (static_cast<int64_t>(s) * kCodebooks + p % kCodebooks) * f.codec_stride + f.codec_offset + p / kCodebooks;
}

// end_frame_index of session s, and the finished latch of
// finalize_local_step (synthesis_kernels.cu:79-84) when the caller asked for it.
// With codec_frames, also the session's count of audio frames in the
// aggregate (eos_contract.hpp:14-30, retained_codec_frames_before_eos: the
// EOS frame itself is not audio): offset + 2 after a frame without EOS,
// offset + end at the EOS frame, unchanged for a session already finished.
__device__ __forceinline__ void commit_end(const Frame& f, int s, int32_t end) {
  f.end_frame[s] = end;
  if (f.finished_latch != nullptr && (end == 0 || end == 1)) f.finished_latch[s] = true;
  if (f.codec_frames != nullptr && !f.finished[s]) f.codec_frames[s] = f.codec_offset + (end >= 0 ? end : kFrames);
}

struct Layout {
  size_t list, count, eos_list, eos_count, eos_slot, x, q, kc, vc, att, h, logits, tokens, emb_acc, ctr, inv,
      eos_partial, eos_logit, part, total;
};

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// K splits of a phase-kernel tensor-core GEMM whose output feeds the residual
// (o-projection, FFN2): the largest divisor of its 64-column K chunks, up to
// 8, that keeps rows/128 x n/256 tiles x splits within one wave of 148 CTAs.
// The f32 partial sums go to the workspace's `part` region.
// The benchmark shape (d 256, 1 layer, FFN 1024) runs on the fused kernels;
// the phase kernels serve it only when asked, without splitting K, so its
// workspace keeps no room for partial sums.
inline bool fused_frame_shape(int d, int L, int F) { return d == 256 && L == 1 && F == 1024; }
constexpr int kPhaseGemmItems = 148;
constexpr int kMaxPhaseSplits = 8;
inline int phase_splits(int rows, int n, int k) {
  const int tiles = ((rows + 127) / 128) * ((n + 255) / 256);
  const int chunks = k / 64;
  int best = 1;
  for (int s = 2; s <= kMaxPhaseSplits; ++s) {
    if (chunks % s == 0 && tiles * s <= kPhaseGemmItems) best = s;
  }
  return best;
}

inline Layout make_layout(int d, int L, int F, int n, int rp) {
  Layout lo{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  const size_t R = static_cast<size_t>(n) * rp;
  lo.list = take(4 * static_cast<size_t>(n));
  lo.count = take(4);
  lo.eos_list = take(4 * static_cast<size_t>(n));
  lo.eos_count = take(4);
  lo.eos_slot = take(4 * static_cast<size_t>(n));
  lo.x = take(2 * R * d);
  lo.q = take(2 * R * d);
  lo.kc = take(2 * static_cast<size_t>(L) * R * kPositions * d);
  lo.vc = take(2 * static_cast<size_t>(L) * R * kPositions * d);
  lo.att = take(2 * R * d);
  lo.h = take(2 * R * F);
  lo.logits = take(2 * R * kVocab);
  lo.tokens = take(4 * static_cast<size_t>(n) * kPositions);
  lo.emb_acc = take(4 * static_cast<size_t>(n) * kEmbed);
  lo.ctr = take(8 * static_cast<size_t>(n));
  lo.inv = take(4 * static_cast<size_t>(n));
  lo.eos_partial = take(4 * static_cast<size_t>(n) * kPositions * kEosChunks);
  lo.eos_logit = take(4 * static_cast<size_t>(n) * kPositions);
  const int splits = fused_frame_shape(d, L, F)
                         ? 0
                         : std::max(phase_splits(static_cast<int>(R), d, d), phase_splits(static_cast<int>(R), d, F));
  lo.part = take(4 * static_cast<size_t>(splits) * R * d);
  lo.total = off;
  return lo;
}


// Fused cluster kernel (frame_fused.cu).  Returns false when the shape or the
// device cannot run it (the caller then uses the phase kernels).
bool fused_frame_supported(const Frame& f);
// Clusters of the fused kernel that fit on the device at once (0: unsupported).
int fused_frame_clusters();
cudaError_t launch_fused_frame(const Frame& f, cudaStream_t stream);

// Tile kernel (frame_tile.cu): one CTA per 16-row tile, KV cache in TMEM.
bool tile_frame_supported(const Frame& f);
int tile_frame_clusters();
cudaError_t launch_tile_frame(const Frame& f, cudaStream_t stream);

// Pair kernel (frame_pair.cu): a 2-CTA cluster per 16 sessions, each CTA
// streaming half of every weight matrix.
bool pair_frame_supported(const Frame& f);
int pair_frame_clusters();
cudaError_t launch_pair_frame(const Frame& f, cudaStream_t stream);

// Split kernel (frame_split.cu): a cluster of `split` CTAs (1, 2, 4, 8) per
// tile of `rows` rows (16: 8 sessions; 32: 16 sessions, split 2 only), each
// CTA streaming 1/split of every weight matrix, GEMMs on tcgen05 with TMEM
// accumulators.
bool split_frame_supported(const Frame& f, int split, int rows);
// Clusters of `split` CTAs that fit on the device at once (0: unsupported).
int split_frame_clusters(int split, int rows);
cudaError_t launch_split_frame(const Frame& f, int split, int rows, cudaStream_t stream);

// Quad kernel (frame_quad.cu): a 4-CTA cluster per 16-session tile (32 rows),
// one attention head per CTA, tcgen05 GEMMs on 32-row tiles.
bool quad_frame_supported(const Frame& f);
int quad_frame_clusters();
cudaError_t launch_quad_frame(const Frame& f, cudaStream_t stream);
// Octo kernel (frame_quad.cu): the same 16-session tile on an 8-CTA cluster,
// two CTAs per attention head, each streaming an eighth of the FFN and head
// weights.
bool octo_frame_supported(const Frame& f);
int octo_frame_clusters();
cudaError_t launch_octo_frame(const Frame& f, cudaStream_t stream);

// EOS projection (tcgen05 GEMM, eos_proj.cuh) + decision for the sessions a
// frame kernel registered in eos_list / eos_count.
cudaError_t launch_frame_eos(const Frame& f, cudaStream_t stream);
// The projection arguments of a frame: the registered sessions' rows, the
// maxima in eos_partial (as keys), the EOS logits in eos_logit.
EosProjArgs frame_eos_args(const Frame& f);

// The EOS projection of session s (registered in slot e): the frame's own
// (slot arrays) or the one the Main Decoder step computed (eos_pre).
__device__ __forceinline__ const uint32_t* eos_keys(const Frame& f, int s, int e) {
  return f.eos_pre != nullptr ? f.eos_pre + static_cast<int64_t>(s) * 2 * kPositions
                              : reinterpret_cast<const uint32_t*>(f.eos_partial) + static_cast<int64_t>(e) * kPositions;
}
__device__ __forceinline__ const float* eos_logits(const Frame& f, int s, int e) {
  return f.eos_pre != nullptr ? reinterpret_cast<const float*>(f.eos_pre + static_cast<int64_t>(s) * 2 * kPositions) +
                                    kPositions
                              : f.eos_logit + static_cast<int64_t>(e) * kPositions;
}

// 2D bf16 tensor map over a row-major [rows][cols] matrix, box 64 columns x
// box_rows rows, 128-byte swizzle (false if the driver entry point is missing).
bool make_weight_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows);

}  // namespace mtt
