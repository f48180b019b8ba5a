// Shared device helpers for the MagpieTTS-RT Local AR hot path (sm_100a).
//
// The sampling arithmetic restates the reference plugin's contract
// (plugins/local_ar_plugins.cu:1149-1196; docs/engine-contracts.md:262-299):
// Philox-4x32-10 keyed (seed, 0) on counter (offset_lo, offset_hi, 0, 0),
// uniform = signed-magnitude(c0) * 4.6566127342e-10f, clamp to
// [6e-8, 0.99999994], Gumbel = -log(-log u), CFG rounded twice to bf16.
//
// Every floating-point operation whose rounding is part of the contract is
// written with an explicit round-to-nearest intrinsic, so the compiler cannot
// fuse or reorder it and the C oracle (built with -ffp-contract=off) performs
// the identical sequence.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

namespace mtt {

constexpr int kVocab = 2024;
constexpr int kCodebook = 2016;
constexpr int kEosId = 2017;
constexpr int kCompactEosVocab = kCodebook + 1;
constexpr int kEmbed = 768;
constexpr int kPositions = 16;
constexpr int kCodebooks = 8;
constexpr int kFrames = 2;
constexpr int kHeadDim = 64;
constexpr int kPhiloxStride = 2048;
constexpr int64_t kMaxCounter = (INT64_MAX - (kPhiloxStride - 1)) / kPhiloxStride;

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float bits2f(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// Philox-4x32-10, word c0 only.
__device__ __forceinline__ uint32_t philox_word(uint32_t seed, uint64_t offset) {
  uint32_t c0 = static_cast<uint32_t>(offset);
  uint32_t c1 = static_cast<uint32_t>(offset >> 32);
  uint32_t c2 = 0, c3 = 0, k0 = seed, k1 = 0;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t p0 = c0, p2 = c2;
    c0 = __umulhi(0xCD9E8D57u, p2) ^ c1 ^ k0;
    c2 = __umulhi(0xD2511F53u, p0) ^ c3 ^ k1;
    c1 = 0xCD9E8D57u * p2;
    c3 = 0xD2511F53u * p0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

__device__ __forceinline__ float philox_uniform(uint32_t seed, uint64_t offset) {
  const int32_t w = static_cast<int32_t>(philox_word(seed, offset));
  const int64_t magnitude = w < 0 ? -static_cast<int64_t>(w) - 1 : static_cast<int64_t>(w);
  return __fmul_rn(__ll2float_rn(magnitude), 4.6566127342e-10f);
}

// Natural log of a positive normal f32, correctly rounded to f32 (this
// build's own routine: atanh series in double, m in [sqrt(1/2), sqrt(2)),
// 12 terms, then one rounding to f32).  Identical operation sequence to
// orc_log_double in the C oracle.
__device__ __forceinline__ float log_cr(float x) {
  const uint32_t bits = __float_as_uint(x);
  int exponent = static_cast<int>((bits >> 23) & 0xffu) - 127;
  double m = static_cast<double>(__uint_as_float((bits & 0x007fffffu) | 0x3f800000u));
  if (m > 1.4142135623730951) {
    m = __dmul_rn(m, 0.5);
    exponent += 1;
  }
  const double f = __dsub_rn(m, 1.0);
  const double s = __ddiv_rn(f, __dadd_rn(2.0, f));
  const double z = __dmul_rn(s, s);
  double p = 0.04;
  p = __dadd_rn(__dmul_rn(p, z), 0.043478260869565216);
  p = __dadd_rn(__dmul_rn(p, z), 0.047619047619047616);
  p = __dadd_rn(__dmul_rn(p, z), 0.05263157894736842);
  p = __dadd_rn(__dmul_rn(p, z), 0.058823529411764705);
  p = __dadd_rn(__dmul_rn(p, z), 0.06666666666666667);
  p = __dadd_rn(__dmul_rn(p, z), 0.07692307692307693);
  p = __dadd_rn(__dmul_rn(p, z), 0.09090909090909091);
  p = __dadd_rn(__dmul_rn(p, z), 0.1111111111111111);
  p = __dadd_rn(__dmul_rn(p, z), 0.14285714285714285);
  p = __dadd_rn(__dmul_rn(p, z), 0.2);
  p = __dadd_rn(__dmul_rn(p, z), 0.3333333333333333);
  const double two_s = __dadd_rn(s, s);
  const double log_m = __dadd_rn(two_s, __dmul_rn(two_s, __dmul_rn(z, p)));
  const double e = static_cast<double>(exponent);
  const double r = __dadd_rn(__dmul_rn(e, 0.69314718036912381649017333984375),
                             __dadd_rn(__dmul_rn(e, 1.9082149292705877e-10), log_m));
  return __double2float_rn(r);
}

__device__ __forceinline__ float clamped_gumbel(float u) {
  u = fmaxf(0.00000006f, fminf(0.99999994f, u));
  const float inner = log_cr(u);
  return -log_cr(-inner);
}

// bf16(bf16(cond * scale) + uncond * (1 - scale)).
__device__ __forceinline__ float guided_logit(float cond, float uncond, float cfg_scale) {
  const float scaled = round_bf16(__fmul_rn(cond, cfg_scale));
  const float sum = __fadd_rn(scaled, __fmul_rn(uncond, __fsub_rn(1.0f, cfg_scale)));
  return round_bf16(sum);
}

// Order-preserving 16-bit key of a bf16 bit pattern (larger value, larger key).
__device__ __forceinline__ uint32_t bf16_key(uint16_t b) {
  return (b & 0x8000u) ? (~static_cast<uint32_t>(b) & 0xffffu) : (static_cast<uint32_t>(b) | 0x8000u);
}
__device__ __forceinline__ uint16_t key_bf16(uint32_t key) {
  return static_cast<uint16_t>((key & 0x8000u) ? (key & 0x7fffu) : (~key & 0xffffu));
}

struct SamplingParams {
  int32_t top_k;
  float temperature;
  float cfg_scale;
  int32_t argmax;
};

}  // namespace mtt
