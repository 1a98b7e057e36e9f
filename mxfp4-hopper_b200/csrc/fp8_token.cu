// Per-token FP8 E4M3 quantize / dequantize for sm_100a (MoE dispatch sibling of
// the MXFP4 path).  The reference ships no kernel for it (code/kernel/setup.py:62
// lists per_token_quant_fp8.cu in a comment only), so the arithmetic follows the
// reference's FP8 convention (per_token_Mxfp4RowToBf16ToFp8Col.cu:142,161,
// 173-177):
//   amax = max(eps, max |x|) over the row (NaN ignored)
//   scale[row] = amax / 448,  q = E4M3(clamp(x * (448 / amax), +-448))
//   dequant: out = bf16_rn(float(q) * scale[row])
#include "capi_util.h"
#include "common.cuh"

namespace mxb {
namespace {

constexpr int kTokThreads = 128;
constexpr int kMaxChunks = 16;  // 16-byte chunks per thread kept in registers

// One CTA per row; the row stays in registers between the amax and the
// quantize pass (K <= 8 * 128 * 16 = 16384).  Longer rows re-read from L2.
template <int kChunks>
__global__ void __launch_bounds__(kTokThreads) fp8_quant_rows_kernel(
    const uint8_t* __restrict__ x, int64_t M, int64_t K, float eps, uint8_t* __restrict__ q,
    float* __restrict__ scale) {
  __shared__ uint32_t red_bits[kTokThreads / 32];
  __shared__ float red_f[kTokThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t nch = K / 8;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
    const uint8_t* xr = x + r * K * 2;
    uint4 v[kChunks];
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int64_t c = (int64_t)i * kTokThreads + t;
      v[i] = c < nch ? ld_stream_v4(xr + c * 16) : make_uint4(0, 0, 0, 0);
      m = vmax_u16x2(m, v[i].x & 0x7FFF7FFFu);
      m = vmax_u16x2(m, v[i].y & 0x7FFF7FFFu);
      m = vmax_u16x2(m, v[i].z & 0x7FFF7FFFu);
      m = vmax_u16x2(m, v[i].w & 0x7FFF7FFFu);
    }
    uint32_t mb = max(m & 0xFFFFu, m >> 16);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    if (lane == 0) red_bits[warp] = mb;
    __syncthreads();
    mb = max(max(red_bits[0], red_bits[1]), max(red_bits[2], red_bits[3]));
    float amax;
    if (mb <= 0x7F80u) {
      amax = fmaxf(eps, __uint_as_float(mb << 16));
    } else {  // a NaN is present: the float max ignores it
      float a = eps;
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          a = fmaxf(a, fabsf(bf16lo_to_f(w[j])));
          a = fmaxf(a, fabsf(bf16hi_to_f(w[j])));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
      if (lane == 0) red_f[warp] = a;
      __syncthreads();
      amax = fmaxf(fmaxf(red_f[0], red_f[1]), fmaxf(red_f[2], red_f[3]));
    }
    const float qs = 448.0f / amax;
    if (t == 0) scale[r] = amax / 448.0f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int64_t c = (int64_t)i * kTokThreads + t;
      if (c >= nch) continue;
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      uint32_t o[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float a0 = fminf(fmaxf(bf16lo_to_f(w[2 * j]) * qs, -448.0f), 448.0f);
        float a1 = fminf(fmaxf(bf16hi_to_f(w[2 * j]) * qs, -448.0f), 448.0f);
        float a2 = fminf(fmaxf(bf16lo_to_f(w[2 * j + 1]) * qs, -448.0f), 448.0f);
        float a3 = fminf(fmaxf(bf16hi_to_f(w[2 * j + 1]) * qs, -448.0f), 448.0f);
        o[j] = cvt_e4m3x2(a0, a1) | (cvt_e4m3x2(a2, a3) << 16);
      }
      st_stream_v2(q + r * K + c * 8, make_uint2(o[0], o[1]));
    }
    __syncthreads();  // red_* reused by the next row
  }
}

// Rows too long for registers: amax pass, then a quantize pass that re-reads
// the row (from L2 for rows of this size).
__global__ void __launch_bounds__(kTokThreads) fp8_quant_rows_long_kernel(
    const uint8_t* __restrict__ x, int64_t M, int64_t K, float eps, uint8_t* __restrict__ q,
    float* __restrict__ scale) {
  __shared__ float red_f[kTokThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t nch = K / 8;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
    const uint8_t* xr = x + r * K * 2;
    float a = eps;
    for (int64_t c = t; c < nch; c += kTokThreads) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + c * 16);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        a = fmaxf(a, fabsf(bf16lo_to_f(w[j])));
        a = fmaxf(a, fabsf(bf16hi_to_f(w[j])));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) red_f[warp] = a;
    __syncthreads();
    const float amax = fmaxf(fmaxf(red_f[0], red_f[1]), fmaxf(red_f[2], red_f[3]));
    const float qs = 448.0f / amax;
    if (t == 0) scale[r] = amax / 448.0f;
    for (int64_t c = t; c < nch; c += kTokThreads) {
      const uint4 v = ld_stream_v4(xr + c * 16);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float a0 = fminf(fmaxf(bf16lo_to_f(w[2 * j]) * qs, -448.0f), 448.0f);
        float a1 = fminf(fmaxf(bf16hi_to_f(w[2 * j]) * qs, -448.0f), 448.0f);
        float a2 = fminf(fmaxf(bf16lo_to_f(w[2 * j + 1]) * qs, -448.0f), 448.0f);
        float a3 = fminf(fmaxf(bf16hi_to_f(w[2 * j + 1]) * qs, -448.0f), 448.0f);
        o[j] = cvt_e4m3x2(a0, a1) | (cvt_e4m3x2(a2, a3) << 16);
      }
      st_stream_v2(q + r * K + c * 8, make_uint2(o[0], o[1]));
    }
    __syncthreads();
  }
}

// One lane: 8 FP8 bytes -> 16 bytes of BF16; a warp instruction reads 256
// contiguous bytes and writes 512.
__global__ void __launch_bounds__(256) fp8_dequant_rows_kernel(const uint8_t* __restrict__ q,
                                                               const float* __restrict__ scale,
                                                               int64_t M, int64_t K,
                                                               uint8_t* __restrict__ out) {
  const int64_t nch = M * K / 8, per_row = K / 8;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nch;
       c += (int64_t)gridDim.x * blockDim.x) {
    const uint2 v = ld_stream_v2(q + c * 8);
    const float s = scale[c / per_row];
    // E4M3 pairs decoded by the hardware to f16 pairs (exact, NaN kept), widened
    // on the FMA pipe, scaled in f32 and rounded once to BF16 (a NaN becomes the
    // canonical BF16 NaN, as on the scalar path)
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t pair = (j < 2 ? v.x : v.y) >> (16 * (j & 1));
      float f0, f1;
      asm("{\n .reg .b16 p, lo, hi;\n .reg .b32 h;\n"
          " cvt.u16.u32 p, %2;\n"
          " cvt.rn.f16x2.e4m3x2 h, p;\n"
          " mov.b32 {lo, hi}, h;\n"
          " add.rn.f32.f16 %0, lo, 0f80000000;\n"
          " add.rn.f32.f16 %1, hi, 0f80000000;\n}"
          : "=f"(f0), "=f"(f1)
          : "r"(pair));
      o[j] = cvt_bf16x2(f0 * s, f1 * s);
    }
    st_stream_v4(out + c * 16, make_uint4(o[0], o[1], o[2], o[3]));
  }
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_per_token_quant_fp8(const void* input, int64_t M, int64_t K,
                                              void* output_q, void* output_s, float eps,
                                              mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && K >= 0 && K % 8 == 0, MXB_ERR_INVALID_ARGUMENT,
              "quant_fp8: need K %% 8 == 0, got %lld", (long long)K);
  if (M == 0 || K == 0) return MXB_OK;
  MXB_REQUIRE(input && output_q && output_s, MXB_ERR_INVALID_ARGUMENT, "quant_fp8: null pointer");
  MXB_REQUIRE(aligned(input, 16) && aligned(output_q, 8), MXB_ERR_MISALIGNED,
              "quant_fp8: input must be 16-byte and output_q 8-byte aligned");
  const int64_t nch = K / 8;
  const int per = (int)cdiv(nch, kTokThreads);
  const int grid = (int)(M < 148LL * 64 ? M : 148LL * 64);
  cudaStream_t s = to_cuda(stream);
  auto* xi = (const uint8_t*)input;
  auto* qo = (uint8_t*)output_q;
  auto* so = (float*)output_s;
  if (per <= 4)
    fp8_quant_rows_kernel<4><<<grid, kTokThreads, 0, s>>>(xi, M, K, eps, qo, so);
  else if (per <= 8)
    fp8_quant_rows_kernel<8><<<grid, kTokThreads, 0, s>>>(xi, M, K, eps, qo, so);
  else if (per <= kMaxChunks)
    fp8_quant_rows_kernel<kMaxChunks><<<grid, kTokThreads, 0, s>>>(xi, M, K, eps, qo, so);
  else
    fp8_quant_rows_long_kernel<<<grid, kTokThreads, 0, s>>>(xi, M, K, eps, qo, so);
  return launch_status("quant_fp8");
}

extern "C" mxb_status mxb_per_token_dequant_fp8(const void* input_q, const void* input_s,
                                                int64_t M, int64_t K, void* output,
                                                mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && K >= 0 && K % 8 == 0, MXB_ERR_INVALID_ARGUMENT,
              "dequant_fp8: need K %% 8 == 0, got %lld", (long long)K);
  if (M == 0 || K == 0) return MXB_OK;
  MXB_REQUIRE(input_q && input_s && output, MXB_ERR_INVALID_ARGUMENT, "dequant_fp8: null pointer");
  MXB_REQUIRE(aligned(input_q, 8) && aligned(output, 16), MXB_ERR_MISALIGNED,
              "dequant_fp8: input_q must be 8-byte and output 16-byte aligned");
  const int64_t nch = M * K / 8;
  const int64_t want = cdiv(nch, 256);
  const int64_t cap = (int64_t)persistent_ctas((const void*)fp8_dequant_rows_kernel, 256, 0) * 2;
  const int grid = (int)(want < cap ? want : cap);
  fp8_dequant_rows_kernel<<<grid, 256, 0, to_cuda(stream)>>>(
      (const uint8_t*)input_q, (const float*)input_s, M, K, (uint8_t*)output);
  return launch_status("dequant_fp8");
}
