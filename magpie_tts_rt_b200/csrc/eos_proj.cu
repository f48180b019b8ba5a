// EOS projection on tcgen05 (eos_proj.cuh): row gather + one GEMM whose
// epilogue reduces the guided logits to per-(session, position) maxima.
#include "eos_proj.cuh"
#include "frame_common.cuh"
#include "gemm_tc.cuh"

namespace mtt {
namespace {

constexpr int kEosRowsThreads = 128;
constexpr int kEosProjRows = kPositions * kVocab;  // 32,384 final-projection rows
static_assert(kEosProjRows % 128 == 0, "weight tiles");

// Epilogue: lane = final-projection row m = p * 2024 + token; columns come
// in (conditional, unconditional) pairs, one pair per slot.  A warp's 32
// rows span at most two positions (2024 > 32): the lanes of each position
// reduce separately, and lane 0 folds each maximum into the slot's key.
struct EpiEos {
  const bf16* bias;
  float cfg;
  uint32_t* max_key;
  float* eos_logit;

  __device__ __forceinline__ void chunk(int m, int n0, int /*ks*/, const uint32_t (&v)[32], int n_rows) const {
    const int lane = threadIdx.x & 31;
    const int p = m / kVocab, token = m - p * kVocab;
    const bool is_code = token < kCodebook, is_eos = token == kEosId;
    const float b = bf2f(bias[m]);
    const int p0 = __shfl_sync(0xffffffffu, p, 0);
    const bool second = p != p0;
    const bool any_second = __any_sync(0xffffffffu, second);
    const float uncond_scale = __fsub_rn(1.0f, cfg);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int e = (n0 >> 1) + j;
      if (2 * e >= n_rows) break;  // warp-uniform
      const float c = round_bf16(__fadd_rn(__uint_as_float(v[2 * j]), b));
      const float u = round_bf16(__fadd_rn(__uint_as_float(v[2 * j + 1]), b));
      const float us = round_bf16(__fmul_rn(u, uncond_scale));
      const float g = round_bf16(__fadd_rn(us, __fmul_rn(c, cfg)));
      if (is_eos) eos_logit[e * kPositions + p] = g;
      const float val = (is_code && g == g) ? g : -CUDART_INF_F;  // a NaN never wins (fmaxf semantics)
      float a = second ? -CUDART_INF_F : val;
      float z = second ? val : -CUDART_INF_F;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        z = fmaxf(z, __shfl_xor_sync(0xffffffffu, z, o));
      }
      if (lane == 0) {
        if (a > -CUDART_INF_F) atomicMax(&max_key[e * kPositions + p0], order_key(a));
        if (any_second && z > -CUDART_INF_F) atomicMax(&max_key[e * kPositions + p0 + 1], order_key(z));
      }
    }
  }
};

// Slot e: the conditional and unconditional rows of session list[e] (or e)
// into rows 2e and 2e + 1 (the conditional row twice without CFG), and the
// slot's maxima cleared.
__global__ void __launch_bounds__(kEosRowsThreads) eos_rows_kernel(EosProjArgs a) {
  wait_prior_grid();
  const int count = a.count != nullptr ? *a.count : a.n_max;
  constexpr int kUnits = kEmbed / 8;  // 16-byte units per row
  for (int e = blockIdx.x; e < count; e += gridDim.x) {
    const int s = a.list != nullptr ? a.list[e] : e;
    const bf16* hc = a.hidden + static_cast<int64_t>(s) * a.hidden_stream_stride;
    const bf16* hu = hc + a.uncond_offset;
    uint4* dst = reinterpret_cast<uint4*>(a.rows + static_cast<int64_t>(2 * e) * kEmbed);
    for (int i = threadIdx.x; i < 2 * kUnits; i += blockDim.x) {
      const bf16* src = i < kUnits ? hc : hu;
      dst[i] = reinterpret_cast<const uint4*>(src)[i % kUnits];
    }
    if (threadIdx.x < kPositions) a.max_key[e * kPositions + threadIdx.x] = 0u;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.status != nullptr) *a.status = 0;
}

}  // namespace

cudaError_t launch_eos_projection(const EosProjArgs& a, cudaStream_t stream) {
  if (a.n_max <= 0) return cudaSuccess;
  if (a.hidden == nullptr || a.weight == nullptr || a.bias == nullptr || a.rows == nullptr || a.max_key == nullptr ||
      a.eos_logit == nullptr) {
    return cudaErrorInvalidValue;
  }
  const int rows = 2 * a.n_max;
  const int bn = rows <= 64 ? 64 : (rows <= 128 ? 128 : 256);
  CUtensorMap amap, bmap;
  if (!make_weight_map(&amap, a.weight, kEmbed, kEosProjRows, 128) ||
      !make_weight_map(&bmap, a.rows, kEmbed, static_cast<uint64_t>(rows), static_cast<uint32_t>(bn))) {
    return cudaErrorInvalidValue;
  }
  const int gather_grid = a.n_max < 4 * 148 ? a.n_max : 4 * 148;
  cudaError_t e = launch_serialized(eos_rows_kernel, dim3(gather_grid), dim3(kEosRowsThreads), 0, stream, a);
  if (e != cudaSuccess) return e;
  GemmProblem pr;
  pr.m_tiles = kEosProjRows / 128;
  pr.n_rows = rows;
  pr.n_rows_dev = a.count;
  pr.n_rows_scale = 2;
  pr.k_chunks = kEmbed / kGemmKChunk;
  pr.splits = 1;
  pr.status = a.status;
  pr.b_constant = 0;  // the gathered rows come from the launch before
  EpiEos epi{a.bias, a.cfg_scale, a.max_key, a.eos_logit};
  switch (bn) {
    case 64: return launch_gemm_tc<64>(amap, bmap, pr, epi, stream);
    case 128: return launch_gemm_tc<128>(amap, bmap, pr, epi, stream);
    default: return launch_gemm_tc<256>(amap, bmap, pr, epi, stream);
  }
}

}  // namespace mtt
