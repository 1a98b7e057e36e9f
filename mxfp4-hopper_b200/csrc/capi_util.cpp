// Error reporting and small host utilities behind the C ABI.
#include "capi_util.h"

#include <mutex>
#include <unordered_map>

namespace mxb {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int persistent_ctas(const void* kernel, int threads, size_t smem) {
  // Cached per (kernel, device): occupancy does not change during a process.
  static std::mutex mu;
  static std::unordered_map<const void*, int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache[dev & 63].find(kernel);
    if (it != cache[dev & 63].end()) return it->second;
  }
  int per_sm = 0, sms = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int n = (per_sm > 0 ? per_sm : 1) * (sms > 0 ? sms : 148);
  std::lock_guard<std::mutex> lk(mu);
  cache[dev & 63][kernel] = n;
  return n;
}

}  // namespace mxb

extern "C" const char* mxb_last_error(void) { return mxb::g_err; }
extern "C" const char* mxb_version(void) { return "mxfp4_b200 0.1.0 (sm_100a)"; }
