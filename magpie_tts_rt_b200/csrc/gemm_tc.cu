// Host helpers of the persistent tcgen05 GEMM (gemm_tc.cuh).
#include "gemm_tc.cuh"

namespace mtt {

int gemm_grid(int tiles) {
  static PerDeviceInt sms_cache;
  const int sms = sms_cache.get([] {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return sms;
  });
  if (sms <= 0 || tiles <= 0) return 0;
  return tiles < sms ? tiles : sms;
}

}  // namespace mtt
