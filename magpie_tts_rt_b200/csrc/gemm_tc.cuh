// Persistent tcgen05 GEMM for weight-times-rows products:
//
//   D[m][n] = sum_k A[m][k] B[n][k]
//
// A = a weight matrix [M][K] (PyTorch [out][in] layout, K contiguous), B =
// activation rows [N][K] (K contiguous), f32 accumulation in tensor memory.
// One operand is the MMA's M side (128 rows per tile) and the other its N
// side (BN = 64, 128 or 256 per tile).  On B200 a tcgen05.mma of M = 128,
// K = 16 issued back to back costs about 47 SM cycles for N <= 64 and N / 2
// from N = 128 (the dense peak), so BN = 64 and 128 tiles run at about the
// same time per instruction: callers pick the narrowest BN that keeps the
// grid in one wave when few tiles would otherwise occupy few SMs.
//
// One CTA per SM walks the tiles (m, n, k-split) with a stride of the grid,
// n fastest so that CTAs running at the same time share the weight tile in
// L2.  Warp roles (320 threads):
//   warp 0  TMA producer: one A box (64 K x 128 rows) and one B box (64 K x
//           BN rows) per stage, 128-byte swizzle, no multicast, into a ring
//           of kStages stages;
//   warp 1  allocates tensor memory and issues the MMAs from one thread
//           (tcgen05.mma kind::f16, A and B from shared memory), committing
//           each stage back to the producer and each finished tile to the
//           epilogue; accumulators alternate between two BN-column buffers
//           so the epilogue of one tile overlaps the MMAs of the next;
//   warps 2-9 epilogue: warp w reads tensor-memory lanes [32 (w % 4), +32)
//           (its 32 rows of the M side) with 32-column loads, warps w and w + 4
//           taking alternate 32-column chunks, and hands each chunk to the
//           epilogue functor.
// Every wait is bounded; a timeout sets *status = 1 and the CTA winds down
// (it waits for its own MMAs and copies before freeing tensor memory).
//
// The N extent may live on the device (n_rows_dev): tiles past it are not
// computed, so a launch can be sized for the largest batch while only the
// rows present that frame cost time.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "ptx.cuh"

namespace mtt {

constexpr int kGemmEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kGemmEpiWarps;
constexpr int kGemmKChunk = 64;  // K columns per stage: one 128-byte swizzle row of bf16

struct GemmProblem {
  int m_tiles;             // M / 128 (with m_rows_dev: the largest)
  const int* m_rows_dev;   // optional device count: M = m_rows_scale * *m_rows_dev
  int m_rows_scale;
  int n_rows;              // N when n_rows_dev is null, else the largest N (grid sizing)
  const int* n_rows_dev;   // optional device count: N = n_rows_scale * *n_rows_dev
  int n_rows_scale;
  int k_chunks;            // K / 64 per split
  int splits;              // K splits (partial sums combined by the caller)
  int* status;             // optional: set to 1 when a bounded wait gave up
  int b_constant;          // B (e.g. the weights) is not written by the previous launch: its first
                           // stages are fetched before waiting on that launch (needs n_rows_dev null)
};

template <int BN>
struct GemmCfg {
  static_assert(BN == 64 || BN == 128 || BN == 256, "row tile");
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr uint32_t kABytes = 128 * kGemmKChunk * 2;  // 16 KB
  static constexpr uint32_t kBBytes = BN * kGemmKChunk * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulator buffers (a power of two >= 128)
  static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStageBytes + 1024;
  static constexpr uint32_t kIdesc = umma_idesc_bf16(128, BN);
};

__device__ __forceinline__ void tmem_ld32(uint32_t (&v)[32], uint32_t taddr) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
                 "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]),
                 "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                 "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

__device__ __forceinline__ int gemm_epi_warp() { return (static_cast<int>(threadIdx.x) >> 5) - 2; }
__device__ __forceinline__ void gemm_epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kGemmEpiWarps) : "memory");
}
template <class Epi, class = void>
struct EpiHasTileEnd {
  static constexpr bool value = false;
};
template <class Epi>
struct EpiHasTileEnd<Epi, decltype(void(Epi::kTileEnd))> {
  static constexpr bool value = Epi::kTileEnd;
};

__device__ __forceinline__ int gemm_n_rows(const GemmProblem& pr) {
  return pr.n_rows_dev != nullptr ? pr.n_rows_scale * *pr.n_rows_dev : pr.n_rows;
}

// Epi: a functor with
//   __device__ void chunk(int m, int n0, int ks, const uint32_t (&v)[32], int n_rows) const;
// called by every lane of an epilogue warp together (warp-uniform n0): lane
// holds D[m][n0 + j] (f32 bits) of its row m for j < 32; columns at or past
// n_rows are padding.  gemm_epi_warp() (0..7) names the calling warp.  With
// `static constexpr bool kTileEnd = true` it also has
//   __device__ void tile_begin(int mt, int nt) const;  __device__ void tile_end(int mt, int nt, int n_rows) const;
// called by all epilogue threads before the first and after the last chunk
// of each tile, between barriers of the epilogue warps (for per-tile
// reductions in shared memory).
template <int BN, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                   GemmProblem pr, Epi epi) {
  using G = GemmCfg<BN>;
  constexpr int S = G::kStages;
  extern __shared__ unsigned char gemm_smem_raw[];
  __shared__ unsigned long long full[S], empty[S], tfull[2], tempty[2], fin;
  __shared__ uint32_t tmem_base;
  __shared__ int err;
  __shared__ int last_issued[S];
  const uint32_t pad = (1024u - (smem_addr(gemm_smem_raw) & 1023u)) & 1023u;
  unsigned char* ring = gemm_smem_raw + pad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Set-up that touches no global memory runs before the wait on the
  // previous launch (programmatic serialization), overlapping its tail.
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      last_issued[s] = -1;
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kGemmEpiWarps);
    }
    mbar_init(&fin, 1);
    err = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, G::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bmap)) : "memory");
  }
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem = tmem_base;
  volatile int* errv = &err;
  // The next launch on the stream may be scheduled now (this grid is one wave);
  // it waits for this grid's completion before reading what it wrote.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  auto decode = [&](int i, int n_tiles_, int m_tiles_, int& mt, int& nt, int& ks) {
    nt = i % n_tiles_;
    const int rest = i / n_tiles_;
    mt = rest % m_tiles_;
    ks = rest / m_tiles_;
  };
  // Stages whose constant B box was issued before the wait (first tile only).
  int pre = 0;
  if (warp == 0 && lane == 0 && pr.b_constant && pr.n_rows_dev == nullptr && pr.m_rows_dev == nullptr) {
    const int n_tiles0 = (pr.n_rows + BN - 1) / BN;
    if (static_cast<int>(blockIdx.x) < pr.m_tiles * n_tiles0 * pr.splits) {
      int mt, nt, ks;
      decode(blockIdx.x, n_tiles0, pr.m_tiles, mt, nt, ks);
      pre = pr.k_chunks < S ? pr.k_chunks : S;
      for (int kc = 0; kc < pre; ++kc) {
        unsigned char* sa = ring + static_cast<size_t>(kc) * G::kStageBytes;
        mbar_expect_tx(&full[kc], G::kStageBytes);
        tma_load_2d(sa + G::kABytes, &bmap, (ks * pr.k_chunks + kc) * kGemmKChunk, nt * BN, &full[kc]);
        last_issued[kc] = kc;
      }
    }
  }

  wait_prior_grid();  // inputs (and the device row counts) of the previous launch
  const int n_rows = gemm_n_rows(pr);
  const int n_tiles = (n_rows + BN - 1) / BN;
  const int m_tiles = pr.m_rows_dev != nullptr ? (pr.m_rows_scale * *pr.m_rows_dev + 127) / 128 : pr.m_tiles;
  const int items = m_tiles * n_tiles * pr.splits;  // a CTA past the work only frees its tensor memory

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int i = blockIdx.x; i < items && *errv == 0; i += gridDim.x) {
        int mt, nt, ks;
        decode(i, n_tiles, m_tiles, mt, nt, ks);
        for (int kc = 0; kc < pr.k_chunks; ++kc, ++it) {
          const int s = it % S;
          if (it >= S && !mbar_wait_cta(&empty[s], ((it / S) - 1) & 1)) *errv = 1;
          if (*errv) break;
          unsigned char* sa = ring + static_cast<size_t>(s) * G::kStageBytes;
          const int kx = (ks * pr.k_chunks + kc) * kGemmKChunk;
          if (it < pre) {  // B already on its way, bytes announced
            tma_load_2d(sa, &amap, kx, mt * 128, &full[s]);
          } else {
            mbar_expect_tx(&full[s], G::kStageBytes);
            tma_load_2d(sa, &amap, kx, mt * 128, &full[s]);
            tma_load_2d(sa + G::kABytes, &bmap, kx, nt * BN, &full[s]);
          }
          last_issued[s] = it;
        }
      }
      // no copy may still be landing in shared memory when the CTA leaves
      for (int s = 0; s < S; ++s) {
        const int last = last_issued[s];
        if (last >= 0) mbar_wait_cta(&full[s], (last / S) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, t = 0;
      for (int i = blockIdx.x; i < items && *errv == 0; i += gridDim.x, ++t) {
        const int buf = t & 1, use = t >> 1;
        if (use >= 1 && !mbar_wait_cta(&tempty[buf], (use - 1) & 1)) {
          *errv = 1;
          break;
        }
        tmem_fence_after_sync();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
        // BN <= 128: two stages (K = 128) at a time, waiting for both, then
        // their 8 MMAs as one straight-line burst (a wait between tcgen05.mma
        // instructions roughly doubles their issue cost at these widths);
        // BN = 256: stage by stage (each MMA costs twice as much, and waiting
        // for a second stage only delays the first)
        constexpr bool kPairs = BN < 256;
        for (int kc = 0; kc < pr.k_chunks; kc += kPairs ? 2 : 1) {
          const bool two = kPairs && kc + 1 < pr.k_chunks;
          const int s0 = it % S, s1 = (it + 1) % S;
          bool ok = mbar_wait_cta(&full[s0], (it / S) & 1);
          if (two) ok = ok && mbar_wait_cta(&full[s1], ((it + 1) / S) & 1);
          if (!ok) {
            *errv = 1;
            break;
          }
          tmem_fence_after_sync();
          const unsigned char* sa0 = ring + static_cast<size_t>(s0) * G::kStageBytes;
          const unsigned char* sa1 = ring + static_cast<size_t>(s1) * G::kStageBytes;
          const uint64_t ad0 = umma_desc_sw128(sa0), bd0 = umma_desc_sw128(sa0 + G::kABytes);
          const uint64_t ad1 = umma_desc_sw128(sa1), bd1 = umma_desc_sw128(sa1 + G::kABytes);
#pragma unroll
          for (int kk = 0; kk < kGemmKChunk / 16; ++kk) {
            umma_bf16(d, ad0 + 2 * kk, bd0 + 2 * kk, G::kIdesc, (kc | kk) != 0);
          }
          if (two) {
#pragma unroll
            for (int kk = 0; kk < kGemmKChunk / 16; ++kk) umma_bf16(d, ad1 + 2 * kk, bd1 + 2 * kk, G::kIdesc, true);
          }
          umma_commit(&empty[s0]);
          if (two) umma_commit(&empty[s1]);
          it += two ? 2 : 1;
        }
        umma_commit(&tfull[buf]);
      }
      // every MMA this thread issued has completed before tensor memory is freed
      umma_commit(&fin);
      mbar_wait_cta(&fin, 0);
    }
  } else {
    const int q = warp & 3;             // the tensor-memory lane quadrant this warp may read
    const int half = (warp - 2) >> 2;   // which alternate 32-column chunks it takes
    int t = 0;
    for (int i = blockIdx.x; i < items; i += gridDim.x, ++t) {
      const int buf = t & 1, use = t >> 1;
      const bool ok = *errv == 0 && mbar_wait_cta(&tfull[buf], use & 1);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) *errv = 1;
        break;
      }
      tmem_fence_after_sync();
      int mt, nt, ks;
      decode(i, n_tiles, m_tiles, mt, nt, ks);
      if constexpr (EpiHasTileEnd<Epi>::value) {
        epi.tile_begin(mt, nt);
        gemm_epi_sync();
      }
      const int m = mt * 128 + 32 * q + lane;
      const uint32_t ta = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(buf * BN);
#pragma unroll 1
      for (int c0 = 32 * half; c0 < BN; c0 += 64) {
        const int n0 = nt * BN + c0;
        if (n0 >= n_rows) break;
        uint32_t v[32];
        tmem_ld32(v, ta + static_cast<uint32_t>(c0));
        epi.chunk(m, n0, ks, v, n_rows);
      }
      tmem_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      if constexpr (EpiHasTileEnd<Epi>::value) {
        gemm_epi_sync();
        epi.tile_end(mt, nt, n_rows);
        gemm_epi_sync();
      }
    }
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tmem_fence_after_sync();
    tmem_dealloc(tmem, G::kTmemCols);
  }
  if (threadIdx.x == 0 && *errv != 0 && pr.status != nullptr) atomicExch(pr.status, 1);
}

// Host side: 2D bf16 tensor map over a row-major [rows][cols] matrix with a
// box of 64 columns x box_rows rows and the 128-byte swizzle (frame_fused.cu).
bool make_weight_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows);

// make_weight_map behind a process-wide cache: the same (pointer, shape,
// box) recurs every step of a layer, and encoding a map costs host time.
bool cached_map(CUtensorMap* out, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows);

// Grid for a persistent GEMM: at most one CTA per SM (0 when the device
// cannot be queried).
int gemm_grid(int tiles);

// Sets the dynamic shared-memory opt-in of gemm_tc_kernel<BN, Epi> on the
// current device once (a per-device setting).
template <int BN, class Epi>
bool gemm_prepare() {
  static PerDeviceInt cache;
  return cache.get([] {
    const bool ok = cudaFuncSetAttribute(gemm_tc_kernel<BN, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(GemmCfg<BN>::kSmem)) == cudaSuccess;
    cudaGetLastError();
    return ok ? 1 : 0;
  }) == 1;
}

template <int BN, class Epi>
cudaError_t launch_gemm_tc(const CUtensorMap& amap, const CUtensorMap& bmap, const GemmProblem& pr, const Epi& epi,
                           cudaStream_t stream) {
  if (!gemm_prepare<BN, Epi>()) return cudaErrorInvalidValue;
  const int max_tiles = pr.m_tiles * ((pr.n_rows + BN - 1) / BN) * pr.splits;
  const int grid = gemm_grid(max_tiles);
  if (grid <= 0) return cudaErrorInvalidValue;
  return launch_serialized(gemm_tc_kernel<BN, Epi>, dim3(grid), dim3(kGemmThreads), GemmCfg<BN>::kSmem, stream, amap,
                           bmap, pr, epi);
}

}  // namespace mtt
