// Test infrastructure only. Stand-in for the `vec_dtypes.cuh` that the
// reference's kernel sources include but do not ship
// (code/kernel/per_token_quant_mxfp4.cu:7). `omo::vec_t<T, N>` is a plain
// array of N elements with element-wise loads and stores; it reproduces the
// values the reference kernels see, not their memory-access widths.
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace omo {
template <typename T, size_t N>
struct vec_t {
  T data[N];
  __device__ __forceinline__ T& operator[](size_t i) { return data[i]; }
  __device__ __forceinline__ const T& operator[](size_t i) const { return data[i]; }
  template <typename U>
  __device__ __forceinline__ void cast_load(const U* ptr) {
#pragma unroll
    for (size_t i = 0; i < N; ++i) data[i] = static_cast<T>(ptr[i]);
  }
  __device__ __forceinline__ void load_global_acquire(const T* ptr) {
#pragma unroll
    for (size_t i = 0; i < N; ++i) data[i] = ptr[i];
  }
  template <typename U>
  __device__ __forceinline__ void cast_store(U* ptr) const {
#pragma unroll
    for (size_t i = 0; i < N; ++i) ptr[i] = static_cast<U>(data[i]);
  }
};
}  // namespace omo
