// Error-message storage behind evie_last_global_error(), and the per-device kernel attribute cache.
#include <cstdlib>
#include <map>
#include <mutex>
#include <set>
#include <tuple>

#include "common.h"
#include "tmap.h"

namespace evie {
evie_status func_attr(const void* fn, cudaFuncAttribute attr, int value) {
  int dev = 0;
  EVIE_CUDA_TRY(cudaGetDevice(&dev));
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int, int>> done;  // (kernel, device, attribute, value) already set
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, dev, (int)attr, value})) return EVIE_OK;
  EVIE_CUDA_TRY(cudaFuncSetAttribute(fn, attr, value));
  done.insert({fn, dev, (int)attr, value});
  return EVIE_OK;
}
evie_status max_dynamic_smem(const void* fn, int bytes) {
  return func_attr(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  cache[dev] = n;
  return n;
}
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("EVIE_PDL_ALL");
    return e && e[0] == '1';
  }();
  return on;
}

std::string& thread_error() {
  thread_local std::string msg;
  return msg;
}
}  // namespace evie

extern "C" const char* evie_last_global_error(void) { return evie::thread_error().c_str(); }
