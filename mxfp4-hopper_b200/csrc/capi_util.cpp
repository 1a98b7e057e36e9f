// Error reporting and small host utilities behind the C ABI.
#include "capi_util.h"

#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>
#include <vector>

namespace mxb {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

static std::mutex& reader_mu() {
  static std::mutex m;
  return m;
}
static std::vector<unsigned int (*)(bool)>& readers() {
  static std::vector<unsigned int (*)(bool)> v;
  return v;
}

bool register_wait_timeout_reader(unsigned int (*reader)(bool reset)) {
  std::lock_guard<std::mutex> lk(reader_mu());
  readers().push_back(reader);
  return true;
}

unsigned int sum_wait_timeouts(bool reset) {
  std::lock_guard<std::mutex> lk(reader_mu());
  unsigned long long total = 0;
  for (auto r : readers()) {
    const unsigned int v = r(reset);
    if (v == 0xFFFFFFFFu) return v;
    total += v;
  }
  return total >= 0xFFFFFFFFull ? 0xFFFFFFFEu : (unsigned int)total;
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

// ---------------------------------------------------------------- tensor maps

namespace mxb {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

bool make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                        int elem_bytes, int64_t rows, int64_t cols, int64_t ld, uint32_t box_cols,
                        uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return false;
  }
  return true;
}

}  // namespace mxb
