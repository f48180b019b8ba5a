// Measurement hooks behind two design decisions of the frame kernels (no
// reference counterpart; bench.py reports their results):
//
// * mtt_b200_test_umma_cycles: SM cycles of one tcgen05.mma kind::f16
//   (M = 128, K = 16, A and B in shared memory) for a given N, issued back to
//   back from one thread into `accumulators` independent TMEM accumulators
//   (n_mma a multiple of 16, accumulators a power of two).  On B200 an
//   instruction costs N / 2 cycles for N >= 128 (the dense peak) and about 46
//   cycles for every N <= 32, whatever the number of accumulators: below
//   N = 128 a narrower row tile leaves that fraction of the tensor core idle.
// * mtt_b200_test_dsmem_bytes_per_cycle: the bytes per SM cycle that each CTA
//   of an 8-CTA cluster pushes into its 7 peers' shared memory with bulk
//   copies (cp.async.bulk shared::cta -> shared::cluster), rounds separated
//   by cluster barriers: the bandwidth available to cluster-wide exchanges of
//   activations.
#include <cooperative_groups.h>

#include "../../include/magpie_tts_rt_b200.h"
#include "common.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace mtt {
namespace {

constexpr int kProbeMmaSmem = 48 * 1024 + 1024;  // A: 128 x 64 bf16, B: 256 x 64 bf16 (128-byte swizzle rows)

__global__ void __launch_bounds__(128) umma_probe_kernel(int n_mma, int n, int accumulators,
                                                          unsigned long long* cycles) {
  extern __shared__ unsigned char raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint32_t tmem_base;
  __shared__ unsigned long long bar;
  for (int i = threadIdx.x; i < 48 * 1024 / 16; i += blockDim.x) {
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  }
  if (threadIdx.x < 32) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_proxy_async();
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  if (threadIdx.x == 0) {
    const uint32_t idesc = umma_idesc_bf16(128, n);
    const uint64_t a0 = umma_desc_sw128(smem);
    const uint64_t b0 = umma_desc_sw128(smem + 16384);
    // 16 MMAs per iteration with precomputed operands, so the loop itself
    // issues faster than the tensor core retires (accumulators: a power of two)
    const uint32_t amask = static_cast<uint32_t>(accumulators - 1);
    const long long t0 = clock64();
    for (int i = 0; i < n_mma; i += 16) {
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const uint32_t d = tmem_base + ((static_cast<uint32_t>(u) & amask) * static_cast<uint32_t>(n));
        umma_bf16(d, a0 + 2 * (u & 3), b0 + 2 * (u & 3), idesc, i + u >= accumulators);
      }
    }
    umma_commit(&bar);
    const bool ok = mbar_wait(&bar, 0, 100000000ull);
    const long long t1 = clock64();
    cycles[blockIdx.x] = ok ? static_cast<unsigned long long>(t1 - t0) : 0ull;
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) {
    tmem_fence_after_sync();
    tmem_dealloc(tmem_base, 512);
  }
}

constexpr int kPeerSlot = 16384;
constexpr int kProbeDsmemSmem = kPeerSlot * 9 + 128;

__device__ __forceinline__ void bulk_to_peer(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                             uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(smem_addr(src)), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

// Every CTA runs every round (the cluster barrier counts always match); a
// round whose bytes do not all land within its bounded wait records 0.
__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(128)
    dsmem_probe_kernel(int rounds, int bytes, unsigned long long* cycles) {
  extern __shared__ unsigned char raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 127) & ~uintptr_t(127));
  unsigned char* send = smem;
  unsigned char* recv = smem + kPeerSlot;  // one 16 KB slot per sender rank
  __shared__ unsigned long long bar;
  cg::cluster_group cl = cg::this_cluster();
  const int rank = static_cast<int>(cl.block_rank());
  for (int i = threadIdx.x; i < kPeerSlot / 16; i += blockDim.x) {
    reinterpret_cast<uint4*>(send)[i] = make_uint4(rank, i, 1, 2);
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_proxy_async();
  cl.sync();
  const long long t0 = clock64();
  bool ok = true;
  for (int r = 0; r < rounds; ++r) {
    if (threadIdx.x == 0) mbar_expect_tx(&bar, 7u * static_cast<uint32_t>(bytes));
    cl.sync();  // every receiver has announced this round's bytes
    if (threadIdx.x < 8 && threadIdx.x != rank) {
      const int peer = threadIdx.x;
      bulk_to_peer(cluster_addr(recv + rank * kPeerSlot, peer), send, static_cast<uint32_t>(bytes),
                   cluster_addr(&bar, peer));
    }
    bool w = true;
    if (threadIdx.x == 0) w = mbar_wait(&bar, r & 1, 50000000ull);
    ok = __syncthreads_and(w) && ok;
  }
  const long long t1 = clock64();
  cl.sync();
  if (threadIdx.x == 0) cycles[blockIdx.x] = ok ? static_cast<unsigned long long>(t1 - t0) : 0ull;
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API int mtt_b200_test_umma_cycles(int32_t n, int32_t accumulators, int32_t n_mma,
                                                     int32_t ctas, uint64_t* cycles, void* stream) {
  using namespace mtt;
  if (cycles == nullptr || n < 16 || n > 256 || n % 16 != 0 || accumulators < 1 ||
      (accumulators & (accumulators - 1)) != 0 || accumulators * n > 512 || n_mma < 16 || n_mma % 16 != 0 ||
      ctas < 1 || ctas > 1024) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  if (cudaFuncSetAttribute(umma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeMmaSmem) !=
      cudaSuccess) {
    return MTT_B200_STATUS_CUDA_ERROR;
  }
  umma_probe_kernel<<<ctas, 128, kProbeMmaSmem, static_cast<cudaStream_t>(stream)>>>(
      n_mma, n, accumulators, reinterpret_cast<unsigned long long*>(cycles));
  return cudaPeekAtLastError() == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}

extern "C" MTT_B200_API int mtt_b200_test_dsmem_cycles(int32_t bytes_per_peer, int32_t rounds, int32_t clusters,
                                                      uint64_t* cycles, void* stream) {
  using namespace mtt;
  if (cycles == nullptr || bytes_per_peer < 16 || bytes_per_peer > kPeerSlot || bytes_per_peer % 16 != 0 ||
      rounds < 1 || clusters < 1 || clusters > 128) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  if (cudaFuncSetAttribute(dsmem_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeDsmemSmem) !=
      cudaSuccess) {
    return MTT_B200_STATUS_CUDA_ERROR;
  }
  dsmem_probe_kernel<<<8 * clusters, 128, kProbeDsmemSmem, static_cast<cudaStream_t>(stream)>>>(
      rounds, bytes_per_peer, reinterpret_cast<unsigned long long*>(cycles));
  return cudaPeekAtLastError() == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}
