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

// GEMM orientation: the gathered session rows are the MMA's M side (128 per
// tile: 64 slots, rows 2e / 2e + 1 = conditional / unconditional on adjacent
// lanes) and the final-projection rows its N side (256 per tile, row
// n = p * 2024 + token).  Epilogue: each lane holds 32 final rows of its own
// session row per chunk; the partner lane's value gives the other CFG row,
// both lanes form the guided logits with the reference's roundings, and the
// even lane keeps a running maximum of the code logits for the (at most two)
// positions the tile's 256 final rows span, in shared memory per epilogue
// warp half; at the end of the tile the two halves are folded and each slot
// makes at most two atomic maxima on its global keys.  The EOS logit (token
// 2017) is written by the one lane that sees it.
template <int BN>
struct EpiEos {
  static constexpr bool kTileEnd = true;
  const bf16* bias;
  float cfg;
  uint32_t* max_key;
  float* eos_logit;
  int stride;
  int slots;  // 0 when the slot count lives on the device: see n_slots()
  const int* slot_count;

  __device__ __forceinline__ int n_slots() const { return slot_count != nullptr ? *slot_count : slots; }

  // running maxima [warp half][row of the tile][position segment]
  __device__ __forceinline__ static float (&acc())[2][128][2] {
    __shared__ float a[2][128][2];
    return a;
  }

  __device__ __forceinline__ void tile_begin(int /*mt*/, int /*nt*/) const {
    const int tid = static_cast<int>(threadIdx.x) - 64;
    float* flat = &acc()[0][0][0];
    for (int i = tid; i < 2 * 128 * 2; i += 32 * kGemmEpiWarps) flat[i] = -CUDART_INF_F;
  }

  __device__ __forceinline__ void chunk(int m, int n0, int /*ks*/, const uint32_t (&v)[32], int n_rows) const {
    const int lane = threadIdx.x & 31;
    const bool cond_row = (lane & 1) == 0;
    const int e = m >> 1;
    const bool live = e < n_slots();
    const int p_tile = ((n0 / BN) * BN) / kVocab;  // position of the tile's first final row
    // the chunk's 32 final rows: position p0 up to row `next`, then p0 + 1
    const int p0 = n0 / kVocab;
    const int next = (p0 + 1) * kVocab;
    const float bias_lane = n0 + lane < n_rows ? bf2f(bias[n0 + lane]) : 0.f;  // one coalesced load
    const float uncond_scale = __fsub_rn(1.0f, cfg);
    float mx0 = -CUDART_INF_F, mx1 = -CUDART_INF_F;  // the tile's first and second position
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float self = __uint_as_float(v[j]);
      const float partner = __shfl_xor_sync(0xffffffffu, self, 1);
      const float b = __shfl_sync(0xffffffffu, bias_lane, j);
      const int n = n0 + j;
      const bool later = n >= next;                    // position p0 + 1
      const int token = n - (later ? next : next - kVocab);
      const float c = round_bf16(__fadd_rn(cond_row ? self : partner, b));
      const float u = round_bf16(__fadd_rn(cond_row ? partner : self, b));
      const float us = round_bf16(__fmul_rn(u, uncond_scale));
      const float g = round_bf16(__fadd_rn(us, __fmul_rn(c, cfg)));
      if (token == kEosId) {
        if (cond_row && live) eos_logit[e * stride + p0 + (later ? 1 : 0)] = g;
      } else if (token < kCodebook && g == g) {  // a NaN never wins (fmaxf semantics)
        if (p0 + (later ? 1 : 0) == p_tile) {
          mx0 = fmaxf(mx0, g);
        } else {
          mx1 = fmaxf(mx1, g);
        }
      }
    }
    if (cond_row) {
      const int half = gemm_epi_warp() >> 2, r = m & 127;
      acc()[half][r][0] = fmaxf(acc()[half][r][0], mx0);
      acc()[half][r][1] = fmaxf(acc()[half][r][1], mx1);
    }
  }

  __device__ __forceinline__ void tile_end(int mt, int nt, int /*n_rows*/) const {
    const int tid = static_cast<int>(threadIdx.x) - 64;
    const int p_tile = (nt * BN) / kVocab;
    const int total = n_slots();
    for (int i = tid; i < 64 * 2; i += 32 * kGemmEpiWarps) {
      const int r = 2 * (i >> 1), seg = i & 1;
      const int e = mt * 64 + (r >> 1);
      const float v = fmaxf(acc()[0][r][seg], acc()[1][r][seg]);
      if (e < total && v > -CUDART_INF_F && p_tile + seg < kPositions) {
        atomicMax(&max_key[e * stride + p_tile + seg], order_key(v));
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
    if (threadIdx.x < kPositions) a.max_key[e * a.proj_stride + threadIdx.x] = 0u;
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
  CUtensorMap amap, bmap;
  if (!make_weight_map(&amap, a.rows, kEmbed, static_cast<uint64_t>(rows), 128) ||
      !make_weight_map(&bmap, a.weight, kEmbed, kEosProjRows, 256)) {
    return cudaErrorInvalidValue;
  }
  const int gather_grid = a.n_max < 4 * 148 ? a.n_max : 4 * 148;
  cudaError_t e = launch_serialized(eos_rows_kernel, dim3(gather_grid), dim3(kEosRowsThreads), 0, stream, a);
  if (e != cudaSuccess) return e;
  if (a.proj_stride < kPositions) return cudaErrorInvalidValue;
  GemmProblem pr;
  pr.m_tiles = (rows + 127) / 128;
  pr.m_rows_dev = a.count;  // null: all n_max slots
  pr.m_rows_scale = 2;
  pr.n_rows = kEosProjRows;
  pr.n_rows_dev = nullptr;
  pr.n_rows_scale = 1;
  pr.k_chunks = kEmbed / kGemmKChunk;
  pr.splits = 1;
  pr.status = a.status;
  pr.b_constant = 0;
  EpiEos<256> epi{a.bias, a.cfg_scale, a.max_key, a.eos_logit, a.proj_stride, a.n_max, a.count};
  return launch_gemm_tc<256>(amap, bmap, pr, epi, stream);
}

}  // namespace mtt
