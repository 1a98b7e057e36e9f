// Test infrastructure only. Stand-in for the `utils.h` that the reference's
// kernel sources include but do not ship (code/kernel/per_token_quant_mxfp4.cu:6).
// Provides the check macros, FULL_MASK, FP8_E4M3_MAX and the two dtype
// dispatchers the reference kernels use, so that those sources compile
// unmodified into oracle/_ref/omo_ref*.so (the GPU-side parity oracle).
#pragma once
#include <torch/extension.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#ifndef FULL_MASK
#define FULL_MASK 0xffffffffu
#endif

constexpr float FP8_E4M3_MAX = 448.0f;

#undef CHECK_EQ
#define CHECK_EQ(a, b) TORCH_CHECK((a) == (b), "CHECK_EQ(" #a ", " #b ") failed")
#define REF_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define REF_CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_INPUT(x) \
  REF_CHECK_CUDA(x);   \
  REF_CHECK_CONTIG(x)

// Each dispatcher binds `c_type` to the C++ type of `pytorch_dtype` and runs the
// lambda given as the trailing argument.
#define DISPATCH_PYTORCH_DTYPE_TO_CTYPE_FLOAT_FP16(pytorch_dtype, c_type, ...) \
  [&]() -> bool {                                                              \
    switch (pytorch_dtype) {                                                   \
      case at::ScalarType::Float: {                                            \
        using c_type = float;                                                  \
        return __VA_ARGS__();                                                  \
      }                                                                        \
      case at::ScalarType::Half: {                                             \
        using c_type = __half;                                                 \
        return __VA_ARGS__();                                                  \
      }                                                                        \
      case at::ScalarType::BFloat16: {                                         \
        using c_type = __nv_bfloat16;                                          \
        return __VA_ARGS__();                                                  \
      }                                                                        \
      default:                                                                 \
        TORCH_CHECK(false, "unsupported input dtype");                         \
        return false;                                                          \
    }                                                                          \
  }()

#define DISPATCH_PYTORCH_DTYPE_TO_CTYPE_UINT8(pytorch_dtype, c_type, ...) \
  [&]() -> bool {                                                         \
    switch (pytorch_dtype) {                                              \
      case at::ScalarType::Byte: {                                        \
        using c_type = uint8_t;                                           \
        __VA_ARGS__();                                                    \
        return true;                                                      \
      }                                                                   \
      default:                                                            \
        TORCH_CHECK(false, "unsupported input dtype");                    \
        return false;                                                     \
    }                                                                     \
  }()
