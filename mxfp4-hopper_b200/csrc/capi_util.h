// Host-side helpers shared by the C-ABI entry points: argument checks that
// report through mxb_last_error() instead of throwing across the C boundary.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <nvtx3/nvToolsExt.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "mxfp4_b200.h"

namespace mxb {

void set_error(const char* fmt, ...);

// NVTX range over a host-side step (a C-ABI call, a pipeline chunk): shows in
// Nsight Systems timelines; costs nothing when no tool is attached.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

inline cudaStream_t to_cuda(mxb_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// Checks the launch that was just issued; returns MXB_ERR_CUDA with the CUDA
// error text on failure.
inline mxb_status launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
    return MXB_ERR_CUDA;
  }
  return MXB_OK;
}

// Host: 2-D row-major tensor map over [rows, cols] elements of `elem_bytes`
// with row pitch `ld` elements and a box of box_cols x box_rows (no swizzle,
// zero fill out of range).  Reports through set_error on failure.
bool make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                        int elem_bytes, int64_t rows, int64_t cols, int64_t ld, uint32_t box_cols,
                        uint32_t box_rows,
                        CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

// Registry of per-translation-unit wait-timeout counters (see tma.cuh).
// Returns true so that it can initialise a namespace-scope constant.
bool register_wait_timeout_reader(unsigned int (*reader)(bool reset));
// Sum of every registered counter on the current device; with `reset` the
// counters are zeroed after reading.  0xFFFFFFFF if a read failed.
unsigned int sum_wait_timeouts(bool reset);

// Number of resident CTAs worth launching for a grid-stride kernel.
int persistent_ctas(const void* kernel, int threads, size_t smem);

}  // namespace mxb

#define MXB_REQUIRE(cond, status, ...)  \
  do {                                  \
    if (!(cond)) {                      \
      ::mxb::set_error(__VA_ARGS__);    \
      return (status);                  \
    }                                   \
  } while (0)
