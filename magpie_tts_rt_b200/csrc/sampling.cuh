// Block-cooperative sampling of one (stream, position) call.
//
// Restates sampling_kernel (plugins/local_ar_plugins.cu:1211-1370) and the
// argmax kernel (magpietts_fused_sampling.py:136-197) without a full sort:
//   1. constrained guided logits (CFG rounded twice, forbidden specials, EOS
//      gate, finished -> EOS only, non-finite -> -inf + invalid);
//   2. the inclusive top-k threshold (the k-th largest value, ties included)
//      by an exact radix select over order-preserving keys: 2 passes of 8 bits
//      for bf16-valued logits, 4 passes for f32 logits, each pass one
//      per-warp shared-memory histogram summed by warp 0;
//   3. the finite eligible tokens (value >= threshold) compacted in token
//      order, so each thread scores about one of them: Philox-Gumbel score,
//      left-most argmax over the block.  A -inf value scores -inf for every
//      finite Gumbel and can only be chosen when nothing is finite, which
//      makes the row invalid with token 0; such tokens are not scored.
// One block of kSampleThreads threads; thread t owns tokens [8t, 8t+8).
#pragma once

#include "common.cuh"

namespace mtt {

constexpr int kSampleThreads = 256;
constexpr int kItems = 8;  // tokens per thread
constexpr int kSampleWarps = kSampleThreads / 32;
// Scratch (shared memory, 16-byte aligned) for one call: per-warp histograms
// [8][256] u32 followed by the eligible-token list [2048] u16.
constexpr int kSampleScratchBytes = kSampleWarps * 256 * 4 + 2048 * 2;

struct SampleShared {
  uint32_t digit_and_remaining[2];
  uint32_t warp_nonfinite[kSampleWarps];
  uint32_t warp_count[kSampleWarps];
  uint32_t warp_finite[kSampleWarps];
  uint32_t warp_max[kSampleWarps];
  uint32_t window_ok;
  float warp_best[kSampleWarps];
  int32_t warp_best_id[kSampleWarps];
  int32_t finite_count;
  int32_t nonfinite;
  int32_t n_eligible;
  int32_t token;
  int32_t invalid;
};

enum LogitKind : int32_t { kLogitsBf16Cfg = 0, kLogitsBf16 = 1, kLogitsF32 = 2 };

struct SampleCall {
  const void* logits;   // kLogitsBf16Cfg: cond row at logits, uncond row at logits + uncond_offset
  int64_t uncond_offset;  // elements
  int32_t kind;
  bool unfinished, finished, forbid_eos;
  int64_t seed;
  int64_t counter;
};

// The constrained value of token t from its raw (guided) logit: forbidden
// specials, the EOS gate, finished -> EOS only; a non-finite raw value
// becomes -inf and sets *nonfinite.
__device__ __forceinline__ float constrain_token(int t, float raw, bool unfinished, bool finished, bool forbid_eos,
                                                 bool* nonfinite) {
  float x = raw;
  if (!isfinite(x)) {
    *nonfinite = true;
    x = -CUDART_INF_F;
  }
  const bool forbidden_special = t >= kCodebook && t != kEosId;
  if (forbidden_special || ((unfinished || forbid_eos) && t == kEosId)) x = -CUDART_INF_F;
  if (finished) x = (t == kEosId) ? 0.0f : -CUDART_INF_F;
  return x;
}

// Loads this thread's 8 constrained values.  Returns per-thread non-finite flag.
__device__ __forceinline__ bool load_constrained(const SampleCall& c, const SamplingParams& prm,
                                                 float (&v)[kItems]) {
  const int base = threadIdx.x * kItems;
  bool nonfinite = false;
  float raw[kItems];
  if (base < kVocab) {
    if (c.kind == kLogitsF32) {
      const float* l = static_cast<const float*>(c.logits) + base;
#pragma unroll
      for (int i = 0; i < kItems; ++i) raw[i] = (base + i < kVocab) ? l[i] : -CUDART_INF_F;
    } else {
      const uint16_t* l = static_cast<const uint16_t*>(c.logits) + base;
      uint16_t cb[kItems], ub[kItems];
      const bool vec = ((reinterpret_cast<uintptr_t>(l) & 15u) == 0) && base + kItems <= kVocab &&
                       (c.kind != kLogitsBf16Cfg || ((reinterpret_cast<uintptr_t>(l + c.uncond_offset) & 15u) == 0));
      if (vec) {
        const uint4 a = *reinterpret_cast<const uint4*>(l);
        memcpy(cb, &a, 16);
        if (c.kind == kLogitsBf16Cfg) {
          const uint4 b = *reinterpret_cast<const uint4*>(l + c.uncond_offset);
          memcpy(ub, &b, 16);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
          cb[i] = (base + i < kVocab) ? l[i] : 0;
          ub[i] = (c.kind == kLogitsBf16Cfg && base + i < kVocab) ? l[c.uncond_offset + i] : 0;
        }
      }
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        raw[i] = c.kind == kLogitsBf16Cfg ? guided_logit(bits2f(cb[i]), bits2f(ub[i]), prm.cfg_scale)
                                          : bits2f(cb[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int t = base + i;
    v[i] = t < kVocab ? constrain_token(t, raw[i], c.unfinished, c.finished, c.forbid_eos, &nonfinite)
                      : -CUDART_INF_F;
  }
  return nonfinite;
}

__device__ __forceinline__ uint32_t f32_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_f32(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Sums the per-warp histograms bin by bin into the first one (thread t owns
// bin t: no two threads touch the same word), then publishes it.
__device__ __forceinline__ void fold_histograms(uint32_t* hist) {
  static_assert(kSampleThreads == 256, "one thread per bin");
  uint32_t t = 0;
#pragma unroll
  for (int w = 0; w < kSampleWarps; ++w) t += hist[w * 256 + threadIdx.x];
  hist[threadIdx.x] = t;
  __syncthreads();
}

// Lane l's eight consecutive bins 8l .. 8l+7 of the folded histogram.
__device__ __forceinline__ void lane_bins(const uint32_t* hist, int lane, uint32_t (&c)[8]) {
  const uint4 a = reinterpret_cast<const uint4*>(hist + 8 * lane)[0];
  const uint4 b = reinterpret_cast<const uint4*>(hist + 8 * lane)[1];
  c[0] = a.x; c[1] = a.y; c[2] = a.z; c[3] = a.w;
  c[4] = b.x; c[5] = b.y; c[6] = b.z; c[7] = b.w;
}

// One radix pass: histogram of digit (key >> shift) & 0xff over keys matching
// (prefix, mask); warp 0 finds the digit holding the `remaining`-th largest.
// Also sums the per-warp finite counts / non-finite flags on the first pass.
template <bool kFirst>
__device__ __forceinline__ void radix_pass(const uint32_t (&key)[kItems], int shift, uint32_t prefix, uint32_t mask,
                                           uint32_t remaining, SampleShared& sh, uint32_t* hist) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = threadIdx.x * kItems;
  uint32_t* wh = hist + warp * 256;
#pragma unroll
  for (int i = lane; i < 256; i += 32) wh[i] = 0;
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    if (base + i < kVocab && (key[i] & mask) == prefix) atomicAdd(&wh[(key[i] >> shift) & 0xffu], 1u);
  }
  __syncthreads();
  fold_histograms(hist);
  if (warp == 0) {
    // lane l owns digits 255 - 8l - j (descending), j = 0..7
    uint32_t c[8], d[8];
    lane_bins(hist, 31 - lane, d);
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = d[7 - j];
      sum += c[j];
    }
    if (kFirst && lane == 0) {
      uint32_t finite = 0, nf = 0;
#pragma unroll
      for (int w = 0; w < kSampleWarps; ++w) {
        finite += sh.warp_finite[w];
        nf |= sh.warp_nonfinite[w];
      }
      sh.finite_count = static_cast<int32_t>(finite);
      sh.nonfinite = nf ? 1 : 0;
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t excl = incl - sum;
    if (excl < remaining && remaining <= incl) {
      uint32_t acc = excl;
      int j = 0;
      for (; j < 7; ++j) {
        if (remaining <= acc + c[j]) break;
        acc += c[j];
      }
      sh.digit_and_remaining[0] = 255u - lane * 8u - j;
      sh.digit_and_remaining[1] = remaining - acc;
    }
  }
  __syncthreads();
}

// Fast path for 16-bit keys: the k-th largest usually lies within 255 key
// steps (bf16 ulps) below the maximum key M.  One histogram of M - key over
// that window; if it holds at least k keys, the k-th largest is exact.
// Returns false (nothing decided) otherwise.  Also publishes the finite count.
__device__ __forceinline__ bool window_kth_key16(const uint32_t (&key)[kItems], int k, SampleShared& sh,
                                                 uint32_t* hist, uint32_t* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = threadIdx.x * kItems;
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < kItems; ++i) m = (base + i < kVocab && key[i] > m) ? key[i] : m;
  m = __reduce_max_sync(0xffffffffu, m);
  uint32_t* wh = hist + warp * 256;
#pragma unroll
  for (int i = lane; i < 256; i += 32) wh[i] = 0;
  if (lane == 0) sh.warp_max[warp] = m;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kSampleWarps; ++w) m = sh.warp_max[w] > m ? sh.warp_max[w] : m;
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const uint32_t dist = m - key[i];
    if (base + i < kVocab && dist < 256u) atomicAdd(&wh[dist], 1u);
  }
  __syncthreads();
  fold_histograms(hist);
  if (warp == 0) {
    // lane l owns distances 8l .. 8l+7 (descending keys)
    uint32_t c[8];
    lane_bins(hist, lane, c);
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += c[j];
    if (lane == 0) {
      uint32_t finite = 0, nf = 0;
#pragma unroll
      for (int w = 0; w < kSampleWarps; ++w) {
        finite += sh.warp_finite[w];
        nf |= sh.warp_nonfinite[w];
      }
      sh.finite_count = static_cast<int32_t>(finite);
      sh.nonfinite = nf ? 1 : 0;
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t excl = incl - sum;
    const uint32_t kk = static_cast<uint32_t>(k);
    if (lane == 31) sh.window_ok = incl >= kk ? 1u : 0u;
    if (excl < kk && kk <= incl) {
      uint32_t acc = excl;
      int j = 0;
      for (; j < 7; ++j) {
        if (kk <= acc + c[j]) break;
        acc += c[j];
      }
      sh.digit_and_remaining[0] = m - static_cast<uint32_t>(lane * 8 + j);
    }
  }
  __syncthreads();
  *out = sh.digit_and_remaining[0];
  const bool ok = sh.window_ok != 0;
  __syncthreads();  // sh is rewritten by the fallback passes
  return ok;
}

// Exact k-th largest key over the block (k >= 1, k <= number of valid tokens).
// KEY_BITS is 16 (bf16-valued logits: key = top half of the f32 key) or 32.
template <int KEY_BITS>
__device__ __forceinline__ uint32_t block_kth_key(const uint32_t (&key)[kItems], int k, SampleShared& sh,
                                                  uint32_t* hist) {
  if constexpr (KEY_BITS == 16) {
    uint32_t t;
    if (window_kth_key16(key, k, sh, hist, &t)) return t;
  }
  uint32_t prefix = 0, mask = 0;
  uint32_t remaining = static_cast<uint32_t>(k);
  radix_pass<true>(key, KEY_BITS - 8, prefix, mask, remaining, sh, hist);
  prefix = sh.digit_and_remaining[0] << (KEY_BITS - 8);
  mask = 0xffu << (KEY_BITS - 8);
  remaining = sh.digit_and_remaining[1];
#pragma unroll
  for (int shift = KEY_BITS - 16; shift >= 0; shift -= 8) {
    radix_pass<false>(key, shift, prefix, mask, remaining, sh, hist);
    prefix |= sh.digit_and_remaining[0] << shift;
    mask |= 0xffu << shift;
    remaining = sh.digit_and_remaining[1];
  }
  return prefix;
}

// Left-most arg-max of (best, id) over the block; returns the block-uniform pair in sh.
__device__ __forceinline__ void block_argmax(float best, int best_id, SampleShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_down_sync(0xffffffffu, best, o);
    const int oi = __shfl_down_sync(0xffffffffu, best_id, o);
    if (ob > best || (ob == best && oi < best_id)) {
      best = ob;
      best_id = oi;
    }
  }
  if (lane == 0) {
    sh.warp_best[warp] = best;
    sh.warp_best_id[warp] = best_id;
  }
  __syncthreads();
  if (warp == 0) {
    float b = lane < kSampleWarps ? sh.warp_best[lane] : -CUDART_INF_F;
    int bi = lane < kSampleWarps ? sh.warp_best_id[lane] : kVocab;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      const float ob = __shfl_down_sync(0xffffffffu, b, o);
      const int oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (ob > b || (ob == b && oi < bi)) {
        b = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      sh.warp_best[0] = b;
      sh.warp_best_id[0] = bi;
    }
  }
  __syncthreads();
}

// Returns the sampled token (block-uniform) and sets *invalid_out (block-uniform).
// scratch: kSampleScratchBytes of 16-byte aligned shared memory.
__device__ __forceinline__ int sample_block(const SampleCall& c, const SamplingParams& prm, SampleShared& sh,
                                            void* scratch, int* invalid_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = threadIdx.x * kItems;
  uint32_t* hist = static_cast<uint32_t*>(scratch);
  uint16_t* elig = reinterpret_cast<uint16_t*>(hist + kSampleWarps * 256);
  float v[kItems];
  const bool nonfinite = load_constrained(c, prm, v);
  const unsigned nf = __ballot_sync(0xffffffffu, nonfinite);
  uint32_t fin = 0;
#pragma unroll
  for (int i = 0; i < kItems; ++i) fin += (base + i < kVocab && v[i] != -CUDART_INF_F) ? 1u : 0u;
  fin = __reduce_add_sync(0xffffffffu, fin);
  if (lane == 0) {
    sh.warp_nonfinite[warp] = nf;
    sh.warp_finite[warp] = fin;
  }

  float best = -CUDART_INF_F;
  int best_id = kVocab;
  int invalid = 0;
  if (prm.argmax) {
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int t = base + i;
      if (t < kVocab && (v[i] > best || (v[i] == best && t < best_id))) {
        best = v[i];
        best_id = t;
      }
    }
    block_argmax(best, best_id, sh);  // its barriers publish warp_finite / warp_nonfinite
    uint32_t total = 0, anynf = 0;
#pragma unroll
    for (int w = 0; w < kSampleWarps; ++w) {
      total += sh.warp_finite[w];
      anynf |= sh.warp_nonfinite[w];
    }
    invalid = (anynf || total == 0) ? 1 : 0;
  } else {
    uint32_t threshold_key;
    float threshold;
    if (c.kind == kLogitsF32) {
      uint32_t key[kItems];
#pragma unroll
      for (int i = 0; i < kItems; ++i) key[i] = f32_key(v[i]);
      threshold_key = block_kth_key<32>(key, prm.top_k, sh, hist);
      threshold = key_f32(threshold_key);
    } else {
      uint32_t key[kItems];
#pragma unroll
      for (int i = 0; i < kItems; ++i) key[i] = f32_key(v[i]) >> 16;
      threshold_key = block_kth_key<16>(key, prm.top_k, sh, hist);
      threshold = key_f32((threshold_key << 16) | ((threshold_key & 0x8000u) ? 0u : 0xffffu));
    }
    invalid = (sh.nonfinite || sh.finite_count == 0) ? 1 : 0;
    if (c.unfinished && c.finished) invalid = 1;
    if (c.finished && c.forbid_eos) invalid = 1;
    const bool seed_valid = c.seed >= 0 && static_cast<uint64_t>(c.seed) < (1ull << 32);
    const bool counter_valid = c.counter >= 0 && c.counter <= kMaxCounter;
    if (!seed_valid || !counter_valid) invalid = 1;

    // compact the finite eligible tokens in token order
    uint32_t emask = 0;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      if (base + i < kVocab && v[i] >= threshold && v[i] != -CUDART_INF_F) emask |= 1u << i;
    }
    const uint32_t cnt = __popc(emask);
    uint32_t incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) sh.warp_count[warp] = incl;
    __syncthreads();
    uint32_t off = incl - cnt;
    uint32_t total = 0;
#pragma unroll
    for (int w = 0; w < kSampleWarps; ++w) {
      const uint32_t wc = sh.warp_count[w];
      off += w < warp ? wc : 0u;
      total += wc;
    }
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      if (emask & (1u << i)) elig[off++] = static_cast<uint16_t>(base + i);
    }
    __syncthreads();
    const uint32_t seed32 = seed_valid ? static_cast<uint32_t>(c.seed) : 0u;
    const uint64_t off64 = counter_valid ? static_cast<uint64_t>(c.counter) * kPhiloxStride : 0ull;
    // the constrained value of token t lives in the owning thread's registers;
    // recompute it from the logits (cheap, exact) instead of exchanging it
    auto value_of = [&](int t) {
      float value;
      if (c.kind == kLogitsF32) {
        value = static_cast<const float*>(c.logits)[t];
      } else {
        const uint16_t* l = static_cast<const uint16_t*>(c.logits);
        value = c.kind == kLogitsBf16Cfg ? guided_logit(bits2f(l[t]), bits2f(l[c.uncond_offset + t]), prm.cfg_scale)
                                         : bits2f(l[t]);
      }
      return c.finished ? 0.0f : value;  // only EOS (value 0) is finite for a finished row
    };
    bool exact = true;
    if (total <= blockDim.x) {
      // fast scores (library logf) first; the exact Gumbel only when more than
      // one token lies within kVerifyMargin of the best fast score
      const int t1 = threadIdx.x < total ? elig[threadIdx.x] : -1;
      const float v1 = t1 >= 0 ? value_of(t1) : 0.0f;
      const float f1 = t1 >= 0 ? __fadd_rn(__fdiv_rn(v1, prm.temperature),
                                           fast_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t1))))
                               : -CUDART_INF_F;
      block_argmax(f1, t1 >= 0 ? t1 : kVocab, sh);
      const bool near = t1 >= 0 && f1 >= sh.warp_best[0] - kVerifyMargin;
      if (__syncthreads_count(near) == 1) {
        exact = false;  // sh holds the winner
      } else if (near) {
        const float g = clamped_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t1)));
        best = __fadd_rn(__fdiv_rn(v1, prm.temperature), g);
        best_id = t1;
      }
      if (exact) block_argmax(best, best_id, sh);
    } else {
      for (uint32_t e = threadIdx.x; e < total; e += blockDim.x) {
        const int t = elig[e];
        const float g = clamped_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t)));
        const float score = __fadd_rn(__fdiv_rn(value_of(t), prm.temperature), g);
        if (score > best || (score == best && t < best_id)) {
          best = score;
          best_id = t;
        }
      }
      block_argmax(best, best_id, sh);
    }
  }
  const float b = sh.warp_best[0];
  int token = sh.warp_best_id[0];
  if (token >= kVocab || b == -CUDART_INF_F) {
    invalid = 1;
    token = 0;
  }
  *invalid_out = invalid;
  __syncthreads();  // sh is reused by the next call
  return token;
}

// ---------------------------------------------------------------------------
// Pre-scored form (fused cluster kernel): the CTAs that hold a row's logits
// compute every token's constrained value and fast Philox-Gumbel score where
// the logits are; the row's owner receives, per token, the 16-bit order key
// of the value and the fast score, and selects: the inclusive top-k
// threshold on the keys (block_kth_key<16>), the left-most arg-max of the
// fast scores of the finite tokens at or above it, and, when any other such
// token lies within kVerifyMargin of that best, the arg-max of the exact
// scores (value / T + clamped_gumbel) of those near tokens.  Same result as
// sample_block on the same logits (the same fast-then-verify rule; the keys
// order the bf16-valued values exactly).
// ---------------------------------------------------------------------------

constexpr uint32_t kNegInfKey16 = 0x007fu;  // f32_key(-inf) >> 16

__device__ __forceinline__ uint32_t value_key16(float v) { return f32_key(v) >> 16; }
// The bf16-valued value a 16-bit key stands for (exact inverse of value_key16).
__device__ __forceinline__ float key16_value(uint32_t k) {
  return key_f32((k << 16) | ((k & 0x8000u) ? 0u : 0xffffu));
}

// Philox stream of one (session, position) call: seed and counter offset
// (0 where invalid; the call is then flagged invalid by the sampler).
__device__ __forceinline__ uint32_t call_seed32(int64_t seed) {
  return (seed >= 0 && static_cast<uint64_t>(seed) < (1ull << 32)) ? static_cast<uint32_t>(seed) : 0u;
}
__device__ __forceinline__ uint64_t call_offset(int64_t counter) {
  return (counter >= 0 && counter <= kMaxCounter) ? static_cast<uint64_t>(counter) * kPhiloxStride : 0ull;
}

// Fast score of token t with constrained value v (-inf: not a candidate):
// value / T + fast_gumbel, within 1e-4 of the exact score; the selecting
// block rescores exactly whenever another candidate is within kVerifyMargin.
__device__ __forceinline__ float token_score_fast(float v, int t, float temperature, uint32_t seed32, uint64_t off64) {
  if (v == -CUDART_INF_F) return -CUDART_INF_F;
  return __fadd_rn(__fdiv_rn(v, temperature), fast_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t))));
}

// keys[t], fast scores[t] for t < kVocab (shared memory, 16-byte aligned);
// any_nonfinite: a raw value of the row was non-finite.  c supplies the
// flags, seed and counter (its logits are not read).  Returns the token
// (block-uniform) and sets *invalid_out as sample_block does.
__device__ __forceinline__ int sample_block_scored(const uint16_t* keys, const float* scores, bool any_nonfinite,
                                                   const SampleCall& c, const SamplingParams& prm, SampleShared& sh,
                                                   void* scratch, int* invalid_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = threadIdx.x * kItems;
  uint32_t* hist = static_cast<uint32_t*>(scratch);
  uint32_t key[kItems];
  if (base + kItems <= kVocab) {
    const uint4 k4 = *reinterpret_cast<const uint4*>(keys + base);
    const uint16_t* kk = reinterpret_cast<const uint16_t*>(&k4);
#pragma unroll
    for (int i = 0; i < kItems; ++i) key[i] = kk[i];
  } else {
#pragma unroll
    for (int i = 0; i < kItems; ++i) key[i] = base + i < kVocab ? keys[base + i] : kNegInfKey16;
  }
  uint32_t fin = 0;
#pragma unroll
  for (int i = 0; i < kItems; ++i) fin += (base + i < kVocab && key[i] != kNegInfKey16) ? 1u : 0u;
  fin = __reduce_add_sync(0xffffffffu, fin);
  if (lane == 0) {
    sh.warp_nonfinite[warp] = any_nonfinite ? 1u : 0u;
    sh.warp_finite[warp] = fin;
  }
  float best = -CUDART_INF_F;
  int best_id = kVocab;
  int invalid = 0;
  // values compared as floats, as sample_block does (-0 and +0 tie)
  float v[kItems];
#pragma unroll
  for (int i = 0; i < kItems; ++i) v[i] = key16_value(key[i]);
  if (prm.argmax) {
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int t = base + i;
      if (t < kVocab && (v[i] > best || (v[i] == best && t < best_id))) {
        best = v[i];
        best_id = t;
      }
    }
    block_argmax(best, best_id, sh);
    uint32_t total = 0;
#pragma unroll
    for (int w = 0; w < kSampleWarps; ++w) total += sh.warp_finite[w];
    invalid = (any_nonfinite || total == 0) ? 1 : 0;
  } else {
    const float threshold = key16_value(block_kth_key<16>(key, prm.top_k, sh, hist));
    invalid = (sh.nonfinite || sh.finite_count == 0) ? 1 : 0;
    if (c.unfinished && c.finished) invalid = 1;
    if (c.finished && c.forbid_eos) invalid = 1;
    const bool seed_valid = c.seed >= 0 && static_cast<uint64_t>(c.seed) < (1ull << 32);
    const bool counter_valid = c.counter >= 0 && c.counter <= kMaxCounter;
    if (!seed_valid || !counter_valid) invalid = 1;
    uint32_t elig = 0;
    float fs[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int t = base + i;
      fs[i] = -CUDART_INF_F;
      if (t < kVocab && v[i] >= threshold && v[i] != -CUDART_INF_F) {
        elig |= 1u << i;
        fs[i] = scores[t];
        if (fs[i] > best || (fs[i] == best && t < best_id)) {
          best = fs[i];
          best_id = t;
        }
      }
    }
    block_argmax(best, best_id, sh);
    const float fast_best = sh.warp_best[0];
    uint32_t near = 0;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      if ((elig >> i & 1u) && fs[i] >= fast_best - kVerifyMargin) near |= 1u << i;
    }
    const int threads_near = __syncthreads_count(near != 0);
    const int several = __syncthreads_or(__popc(near) > 1);
    if (threads_near != 1 || several) {  // rescore the near tokens exactly (sh is rewritten)
      const uint32_t seed32 = call_seed32(c.seed);
      const uint64_t off64 = call_offset(c.counter);
      best = -CUDART_INF_F;
      best_id = kVocab;
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        if (near >> i & 1u) {
          const int t = base + i;
          const float g = clamped_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t)));
          const float sc = __fadd_rn(__fdiv_rn(v[i], prm.temperature), g);
          if (sc > best || (sc == best && t < best_id)) {
            best = sc;
            best_id = t;
          }
        }
      }
      block_argmax(best, best_id, sh);
    }
  }
  const float b = sh.warp_best[0];
  int token = sh.warp_best_id[0];
  if (token >= kVocab || b == -CUDART_INF_F) {
    invalid = 1;
    token = 0;
  }
  *invalid_out = invalid;
  __syncthreads();  // sh is reused by the next call
  return token;
}

}  // namespace mtt
