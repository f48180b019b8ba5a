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

#include <map>
#include <mutex>

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
// build's own routine, Tang-style table reduction evaluated in double, one
// rounding to f32): x = 2^e m, m in [sqrt(1/2), sqrt(2)); j = nearest(64(m-1));
// t = m * inv_j - 1 (exact, |t| < 0.0113); log(m) = L_j + t + t^2 q(t).
// No division; the operation sequence is identical to orc_log_double in the
// C oracle, so the two agree bit for bit.
__device__ const double kLogTable[47][2] = {
    {0x1.6c16c17000000p+0, -0x1.68ac83f4c6a14p-2},  /* j = -19 */
    {0x1.642c859000000p+0, -0x1.522ae0718a3d8p-2},  /* j = -18 */
    {0x1.5c9882c000000p+0, -0x1.3c25278733184p-2},  /* j = -17 */
    {0x1.5555555000000p+0, -0x1.269621034db92p-2},  /* j = -16 */
    {0x1.4e5e0a7000000p+0, -0x1.1178e8197e47cp-2},  /* j = -15 */
    {0x1.47ae148000000p+0, -0x1.f991c6eb3b379p-3},  /* j = -14 */
    {0x1.4141414000000p+0, -0x1.d1037f1e55e7bp-3},  /* j = -13 */
    {0x1.3b13b14000000p+0, -0x1.a93ed3e8ad9e3p-3},  /* j = -12 */
    {0x1.3521cfb000000p+0, -0x1.823c16431a3c2p-3},  /* j = -11 */
    {0x1.2f684be000000p+0, -0x1.5bf406dd43db2p-3},  /* j = -10 */
    {0x1.29e412a000000p+0, -0x1.365fcb0d59016p-3},  /* j = -9 */
    {0x1.2492492000000p+0, -0x1.1178e8027e47cp-3},  /* j = -8 */
    {0x1.1f7047e000000p+0, -0x1.da727670446a2p-4},  /* j = -7 */
    {0x1.1a7b961000000p+0, -0x1.9335e5bd94989p-4},  /* j = -6 */
    {0x1.15b1e5f000000p+0, -0x1.4d31156607eacp-4},  /* j = -5 */
    {0x1.1111111000000p+0, -0x1.08598b49e3a07p-4},  /* j = -4 */
    {0x1.0c97150000000p+0, -0x1.894aa1c9fb343p-5},  /* j = -3 */
    {0x1.0842108000000p+0, -0x1.0415d81e74444p-5},  /* j = -2 */
    {0x1.0410410000000p+0, -0x1.0205648935847p-6},  /* j = -1 */
    {0x1.0000000000000p+0, 0x0.0p+0},  /* j = 0 */
    {0x1.f81f820000000p-1, 0x1.fc0a890fc03e4p-7},  /* j = 1 */
    {0x1.f07c1f0000000p-1, 0x1.f829b1e783300p-6},  /* j = 2 */
    {0x1.e9131ac000000p-1, 0x1.77458f532dcfcp-5},  /* j = 3 */
    {0x1.e1e1e1e000000p-1, 0x1.f0a30c21162a6p-5},  /* j = 4 */
    {0x1.dae6077000000p-1, 0x1.341d793bbd1d1p-4},  /* j = 5 */
    {0x1.d41d41d000000p-1, 0x1.6f0d28d256b4cp-4},  /* j = 6 */
    {0x1.cd85689000000p-1, 0x1.a926d3a6ad563p-4},  /* j = 7 */
    {0x1.c71c71c000000p-1, 0x1.e2707722af2e6p-4},  /* j = 8 */
    {0x1.c0e0704000000p-1, 0x1.0d77e7a908e59p-3},  /* j = 9 */
    {0x1.bacf915000000p-1, 0x1.29552f6fff523p-3},  /* j = 10 */
    {0x1.b4e81b5000000p-1, 0x1.44d2b6c5b7d1ep-3},  /* j = 11 */
    {0x1.af286bd000000p-1, 0x1.5ff306ee793d4p-3},  /* j = 12 */
    {0x1.a98ef60000000p-1, 0x1.7ab890410d909p-3},  /* j = 13 */
    {0x1.a41a41a000000p-1, 0x1.9525a9e3456b4p-3},  /* j = 14 */
    {0x1.9ec8e95000000p-1, 0x1.af3c94ed0bff3p-3},  /* j = 15 */
    {0x1.999999a000000p-1, 0x1.c8ff7c59a9a22p-3},  /* j = 16 */
    {0x1.948b0fd000000p-1, 0x1.e27076d5af2e6p-3},  /* j = 17 */
    {0x1.8f9c190000000p-1, 0x1.fb9186b5e3e2bp-3},  /* j = 18 */
    {0x1.8acb90f000000p-1, 0x1.0a324e38b90e3p-2},  /* j = 19 */
    {0x1.8618618000000p-1, 0x1.1675cacaba60ep-2},  /* j = 20 */
    {0x1.8181818000000p-1, 0x1.22941fc0f7966p-2},  /* j = 21 */
    {0x1.7d05f41000000p-1, 0x1.2e8e2bc311d31p-2},  /* j = 22 */
    {0x1.78a4c81000000p-1, 0x1.3a64c56b145eap-2},  /* j = 23 */
    {0x1.745d174000000p-1, 0x1.4618bc31c5ec2p-2},  /* j = 24 */
    {0x1.702e05c000000p-1, 0x1.51aad874df82dp-2},  /* j = 25 */
    {0x1.6c16c17000000p-1, 0x1.5d1bdbea809cap-2},  /* j = 26 */
    {0x1.6816817000000p-1, 0x1.686c81d3314afp-2},  /* j = 27 */
};

__device__ __forceinline__ float log_cr(float x) {
  const uint32_t bits = __float_as_uint(x);
  int exponent = static_cast<int>((bits >> 23) & 0xffu) - 127;
  double m = static_cast<double>(__uint_as_float((bits & 0x007fffffu) | 0x3f800000u));
  if (m > 1.4142135623730951) {
    m = __dmul_rn(m, 0.5);
    exponent += 1;
  }
  const int j = __double2int_rn(__dmul_rn(__dsub_rn(m, 1.0), 64.0));
  const double inv = __ldg(&kLogTable[j + 19][0]);
  const double L = __ldg(&kLogTable[j + 19][1]);
  const double t = __fma_rn(m, inv, -1.0);
  double q = 0x1.745d1745d1746p-4;
  q = __fma_rn(q, t, -0x1.999999999999ap-4);
  q = __fma_rn(q, t, 0x1.c71c71c71c71cp-4);
  q = __fma_rn(q, t, -0x1.0000000000000p-3);
  q = __fma_rn(q, t, 0x1.2492492492492p-3);
  q = __fma_rn(q, t, -0x1.5555555555555p-3);
  q = __fma_rn(q, t, 0x1.999999999999ap-3);
  q = __fma_rn(q, t, -0x1.0000000000000p-2);
  q = __fma_rn(q, t, 0x1.5555555555555p-2);
  q = __fma_rn(q, t, -0x1.0000000000000p-1);
  const double t2 = __dmul_rn(t, t);
  const double log_m = __dadd_rn(L, __fma_rn(t2, q, t));
  const double e = static_cast<double>(exponent);
  const double r = __dadd_rn(__dmul_rn(e, 0x1.62e42feep-1), __dadd_rn(__dmul_rn(e, 1.9082149292705877e-10), log_m));
  return __double2float_rn(r);
}

__device__ __forceinline__ float clamped_gumbel(float u) {
  u = fmaxf(0.00000006f, fminf(0.99999994f, u));
  const float inner = log_cr(u);
  return -log_cr(-inner);
}

// Gumbel with the library logf: within 1e-5 of clamped_gumbel (both logs
// within about 1 ulp), so scores built from it are within 1e-4 of the exact
// ones.  Samplers rank candidates with it and rescore with clamped_gumbel
// whenever another candidate lies within kVerifyMargin of the best.
constexpr float kVerifyMargin = 1.0e-3f;

__device__ __forceinline__ float fast_gumbel(float u) {
  u = fmaxf(0.00000006f, fminf(0.99999994f, u));
  return -logf(-logf(u));
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

// Programmatic dependent launch.  A kernel launched by launch_serialized may
// be scheduled while the previous launch on the stream drains; it calls
// wait_prior_grid() before its first global memory access, which returns once
// that launch has completed and its writes are visible.  Launched without the
// attribute the wait is a no-op.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_serialized(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// One int per device ordinal, computed by `make` the first time it is asked
// for with that device current.  A kernel's dynamic shared-memory opt-in
// (cudaFuncSetAttribute) is a setting of the current device's context and
// its occupancy a property of that device, so a process that runs frames on
// several GPUs must make the setting on each of them.  Returns -1 when the
// current device cannot be queried.
class PerDeviceInt {
 public:
  template <typename Make>
  int get(Make make) {
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    const std::lock_guard<std::mutex> lock(mu_);
    auto it = values_.find(device);
    if (it != values_.end()) return it->second;
    const int v = make();
    values_.emplace(device, v);
    return v;
  }

 private:
  std::mutex mu_;
  std::map<int, int> values_;
};

}  // namespace mtt
