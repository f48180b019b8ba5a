// Host helpers of the persistent tcgen05 GEMM (gemm_tc.cuh).
#include "gemm_tc.cuh"

#include <map>
#include <mutex>
#include <tuple>

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

// Tensor maps are host-encoded; the same (pointer, shape, box) recurs every
// step, so they are kept (a few hundred per process at most).
bool cached_map(CUtensorMap* out, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, uint64_t, uint64_t, uint32_t>, CUtensorMap> maps;
  const auto key = std::make_tuple(base, cols, rows, box_rows);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = maps.find(key);
    if (it != maps.end()) {
      *out = it->second;
      return true;
    }
  }
  CUtensorMap m;
  if (!make_weight_map(&m, base, cols, rows, box_rows)) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (maps.size() > 4096) maps.clear();
  maps.emplace(key, m);
  *out = m;
  return true;
}

}  // namespace mtt
