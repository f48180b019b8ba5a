// Block-cooperative sampling of one (stream, position) call.
//
// Restates sampling_kernel (plugins/local_ar_plugins.cu:1211-1370) and the
// argmax kernel (magpietts_fused_sampling.py:136-197) without a full sort:
//   1. constrained guided logits (CFG rounded twice, forbidden specials, EOS
//      gate, finished -> EOS only, non-finite -> -inf + invalid);
//   2. the inclusive top-k threshold (the k-th largest value, ties included)
//      by an exact radix select over order-preserving keys: 2 passes of 8 bits
//      for bf16-valued logits, 4 passes for f32 logits;
//   3. Philox-Gumbel scores for eligible tokens only (a -inf value scores
//      -inf for every finite Gumbel, so it is skipped without changing the
//      result), left-most argmax over the block.
// One block of kThreads threads; thread t owns tokens [8t, 8t+8).
#pragma once

#include "common.cuh"

namespace mtt {

constexpr int kSampleThreads = 256;
constexpr int kItems = 8;  // tokens per thread

struct SampleShared {
  uint32_t hist[256];
  uint32_t digit_and_remaining[2];
  float warp_best[kSampleThreads / 32];
  int32_t warp_best_id[kSampleThreads / 32];
  int32_t flags;  // bit0 invalid (non-finite), bits 8.. finite count
  int32_t finite_count;
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
    float x = -CUDART_INF_F;
    if (t < kVocab) {
      x = raw[i];
      if (!isfinite(x)) {
        nonfinite = true;
        x = -CUDART_INF_F;
      }
      const bool forbidden_special = t >= kCodebook && t != kEosId;
      if (forbidden_special || ((c.unfinished || c.forbid_eos) && t == kEosId)) x = -CUDART_INF_F;
      if (c.finished) x = (t == kEosId) ? 0.0f : -CUDART_INF_F;
    }
    v[i] = x;
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

// Exact k-th largest key over the block (k >= 1, k <= number of valid tokens).
// KEY_BITS is 16 (bf16-valued logits: key = top half of the f32 key) or 32.
template <int KEY_BITS>
__device__ __forceinline__ uint32_t block_kth_key(const uint32_t (&key)[kItems], int k, SampleShared& sh) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int base = threadIdx.x * kItems;
  uint32_t prefix = 0, mask = 0;
  uint32_t remaining = static_cast<uint32_t>(k);
#pragma unroll
  for (int shift = KEY_BITS - 8; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sh.hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const bool part = (base + i < kVocab) && ((key[i] & mask) == prefix);
      const uint32_t digit = part ? ((key[i] >> shift) & 0xffu) : 256u;
      const unsigned peers = __match_any_sync(0xffffffffu, digit);
      if (part && lane == __ffs(peers) - 1) atomicAdd(&sh.hist[digit], __popc(peers));
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending)
      uint32_t c[8];
      uint32_t sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = sh.hist[255 - lane * 8 - j];
        sum += c[j];
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
    prefix |= sh.digit_and_remaining[0] << shift;
    mask |= 0xffu << shift;
    remaining = sh.digit_and_remaining[1];
    __syncthreads();
  }
  return prefix;
}

// Returns the sampled token (block-uniform) and sets *invalid_out (block-uniform).
__device__ __forceinline__ int sample_block(const SampleCall& c, const SamplingParams& prm, SampleShared& sh,
                                            int* invalid_out) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int base = threadIdx.x * kItems;
  if (threadIdx.x == 0) {
    sh.invalid = 0;
    sh.finite_count = 0;
  }
  __syncthreads();
  float v[kItems];
  const bool nonfinite = load_constrained(c, prm, v);
  int finite = 0;
#pragma unroll
  for (int i = 0; i < kItems; ++i) finite += (base + i < kVocab && isfinite(v[i])) ? 1 : 0;
  finite = __reduce_add_sync(0xffffffffu, finite);
  const unsigned nf = __ballot_sync(0xffffffffu, nonfinite);
  if (lane == 0) {
    if (finite) atomicAdd(&sh.finite_count, finite);
    if (nf) atomicOr(&sh.invalid, 1);
  }
  __syncthreads();
  int invalid = sh.invalid | (sh.finite_count == 0 ? 1 : 0);

  float best = -CUDART_INF_F;
  int best_id = kVocab;
  if (prm.argmax) {
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int t = base + i;
      if (t < kVocab && (v[i] > best || (v[i] == best && t < best_id))) {
        best = v[i];
        best_id = t;
      }
    }
  } else {
    if (c.unfinished && c.finished) invalid = 1;
    if (c.finished && c.forbid_eos) invalid = 1;
    const bool seed_valid = c.seed >= 0 && static_cast<uint64_t>(c.seed) < (1ull << 32);
    const bool counter_valid = c.counter >= 0 && c.counter <= kMaxCounter;
    if (!seed_valid || !counter_valid) invalid = 1;
    float threshold;
    if (c.kind == kLogitsF32) {
      uint32_t key[kItems];
#pragma unroll
      for (int i = 0; i < kItems; ++i) key[i] = f32_key(v[i]);
      threshold = key_f32(block_kth_key<32>(key, prm.top_k, sh));
    } else {
      uint32_t key[kItems];
#pragma unroll
      for (int i = 0; i < kItems; ++i) key[i] = f32_key(v[i]) >> 16;
      const uint32_t k16 = block_kth_key<16>(key, prm.top_k, sh);
      threshold = key_f32((k16 << 16) | ((k16 & 0x8000u) ? 0u : 0xffffu));
    }
    const uint32_t seed32 = seed_valid ? static_cast<uint32_t>(c.seed) : 0u;
    const uint64_t off = counter_valid ? static_cast<uint64_t>(c.counter) * kPhiloxStride : 0ull;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int t = base + i;
      if (t >= kVocab || v[i] < threshold) continue;
      float score;
      if (v[i] == -CUDART_INF_F) {
        score = -CUDART_INF_F;
      } else {
        const float g = clamped_gumbel(philox_uniform(seed32, off + static_cast<uint64_t>(t)));
        score = __fadd_rn(__fdiv_rn(v[i], prm.temperature), g);
      }
      if (score > best || (score == best && t < best_id)) {
        best = score;
        best_id = t;
      }
    }
  }
  // block arg-max, left-most on ties
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
  if (threadIdx.x == 0) {
    float b = sh.warp_best[0];
    int bi = sh.warp_best_id[0];
    for (int w = 1; w < kSampleThreads / 32; ++w) {
      if (sh.warp_best[w] > b || (sh.warp_best[w] == b && sh.warp_best_id[w] < bi)) {
        b = sh.warp_best[w];
        bi = sh.warp_best_id[w];
      }
    }
    int inv = invalid;
    if (bi >= kVocab || b == -CUDART_INF_F) {
      inv = 1;
      bi = 0;
    }
    sh.token = bi;
    sh.invalid = inv;
  }
  __syncthreads();
  *invalid_out = sh.invalid;
  const int token = sh.token;
  __syncthreads();
  return token;
}

}  // namespace mtt
