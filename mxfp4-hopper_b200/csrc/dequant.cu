// MXFP4 -> BF16 dequantize and MXFP4 -> FP8 E4M3 rowwise convert for sm_100a.
//
// DQ-bf16 contract (code/kernel/per_token_Mxfp4ToBf16_dequant.cu:129-156):
//   out = bf16_rn(float(e2m1(nibble)) * float(bf16 bits e<<7))
// The product of an E2M1 value and a power of two is exact in BF16 except on
// overflow (-> Inf, as the float path rounds) and for e in {0, 1, 255}
// (zero / subnormal / Inf-NaN scales), which take the float path.  Everything
// else is one BF16x2 multiply per two outputs.
//
// DQ-fp8-row contract (code/kernel/per_token_Mxfp4ToFp8.cu:157-233), per 1x128
// group of four E8M0 bytes (evaluated through a table, fp8_lut.cuh):
//   g   = (uint16)(max e - 6)       group scale float bits ((uint8)g) << 23
//   adj = (uint16)(g - e)
//   q   = E4M3(clamp(bf16(code_bits - (adj << 7) mod 2^16), +-448))
// which re-bases every block onto the group exponent in integer arithmetic;
// zero codes in blocks more than six binades below the group maximum wrap to
// +-448 exactly as on the reference.
#include "capi_util.h"
#include "common.cuh"
#include "fp8_lut.cuh"

namespace mxb {
namespace {

// ------------------------------------------------------------------ DQ-bf16
// A lane turns 4 code bytes (8 elements) into one 16-byte BF16 store, so each
// warp instruction reads 128 contiguous code bytes and writes 512 contiguous
// output bytes.  Four chunks per lane are in flight per iteration.
constexpr int kDqUnroll = 4;

__device__ __forceinline__ uint4 dq_bf16_chunk(uint32_t w, uint32_t e) {
  uint32_t o[4];
  e2m1x4_to_bf16x4(w, o[0], o[1]);
  e2m1x4_to_bf16x4(w >> 16, o[2], o[3]);
  if (e - 2u <= 252u) {  // e in [2, 254]: exact BF16 product
    const uint32_t s2 = (e << 7) | (e << 23);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = mul_bf16x2(o[i], s2);
  } else {
    const float s = e8m0_to_f(e);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = cvt_bf16x2(bf16lo_to_f(o[i]) * s, bf16hi_to_f(o[i]) * s);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(256) dq_bf16_kernel(const uint8_t* __restrict__ codes,
                                                      const uint8_t* __restrict__ scales,
                                                      int64_t chunks, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * kDqUnroll;
  for (int64_t base = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) * kDqUnroll;
       base < chunks; base += stride) {
    uint32_t w[kDqUnroll], e[kDqUnroll];
#pragma unroll
    for (int k = 0; k < kDqUnroll; ++k) {
      const int64_t c = base + k * 32 + lane;
      if (c < chunks) {
        w[k] = ld_stream_u32(codes + c * 4);
        e[k] = ld_stream_u8(scales + (c >> 2));
      }
    }
#pragma unroll
    for (int k = 0; k < kDqUnroll; ++k) {
      const int64_t c = base + k * 32 + lane;
      if (c < chunks) st_stream_v4(out + c * 16, dq_bf16_chunk(w[k], e[k]));
    }
  }
}

// -------------------------------------------------------------- DQ-fp8-row
// A lane converts 8 code bytes (16 elements, half a 32-element block) into one
// 16-byte FP8 store; eight lanes cover one 1x128 group and read the group's
// four E8M0 bytes as one word.  The element arithmetic is a lookup in the
// compile-time table row for d = max_e - e (fp8_lut.cuh).  Four chunks per lane
// are in flight per iteration.
__device__ const Fp8Lut g_lut_row = make_fp8_lut(false);
__device__ const Fp8Lut g_lut_row_strict = make_fp8_lut_strict();

__device__ __forceinline__ uint32_t max_u8x4(uint32_t s) {
  uint32_t a = max(s & 0xFFu, (s >> 8) & 0xFFu);
  uint32_t b = max((s >> 16) & 0xFFu, s >> 24);
  return max(a, b);
}

constexpr int kFp8RowUnroll = 4;

template <bool kStrict>
__global__ void __launch_bounds__(256) dq_fp8_row_kernel(const uint8_t* __restrict__ codes,
                                                         const uint8_t* __restrict__ scales,
                                                         int64_t M, int64_t Kb,
                                                         uint8_t* __restrict__ out,
                                                         float* __restrict__ scales_out) {
  const int64_t lanes_total = M * Kb / 8;  // one lane per 8 code bytes
  const int64_t groups_per_row = Kb / 64;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * kFp8RowUnroll;
  const int lane = threadIdx.x & 31;
  for (int64_t base = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) * kFp8RowUnroll;
       base < lanes_total; base += stride) {
    // all loads of the iteration first (codes, then the groups' scale words,
    // then the table rows they select), then the arithmetic and the stores
    uint2 w[kFp8RowUnroll];
    uint32_t sw[kFp8RowUnroll];
#pragma unroll
    for (int k = 0; k < kFp8RowUnroll; ++k) {
      const int64_t l = base + k * 32 + lane;
      if (l < lanes_total) {
        w[k] = ld_stream_v2(codes + l * 8);
        sw[k] = ld_stream_u32(scales + (l >> 3) * 4);
      } else {
        w[k] = make_uint2(0u, 0u);
        sw[k] = 0u;
      }
    }
    uint32_t mx[kFp8RowUnroll];
    uint4 t[kFp8RowUnroll];
#pragma unroll
    for (int k = 0; k < kFp8RowUnroll; ++k) {
      const int64_t l = base + k * 32 + lane;
      mx[k] = max_u8x4(sw[k]);
      const uint32_t e = (sw[k] >> (8 * ((l >> 1) & 3))) & 0xFFu;
      t[k] = __ldg(reinterpret_cast<const uint4*>((kStrict ? g_lut_row_strict : g_lut_row).v[mx[k] - e]));
    }
#pragma unroll
    for (int k = 0; k < kFp8RowUnroll; ++k) {
      const int64_t l = base + k * 32 + lane;
      if (l >= lanes_total) continue;
      const uint4 o = make_uint4(lut_lookup4(w[k].x, t[k].x, t[k].y, t[k].z, t[k].w),
                                 lut_lookup4(w[k].x >> 16, t[k].x, t[k].y, t[k].z, t[k].w),
                                 lut_lookup4(w[k].y, t[k].x, t[k].y, t[k].z, t[k].w),
                                 lut_lookup4(w[k].y >> 16, t[k].x, t[k].y, t[k].z, t[k].w));
      st_stream_v4(out + l * 16, o);
      if ((l & 7) == 0) {
        const int64_t grp = l >> 3;
        int64_t r;
        if (grp <= (int64_t)UINT32_MAX) {  // 32-bit division whenever it suffices
          r = (uint32_t)grp / (uint32_t)groups_per_row;
        } else {
          r = grp / groups_per_row;
        }
        const int64_t gc = grp - r * groups_per_row;
        scales_out[gc * M + r] = __uint_as_float(((mx[k] - 6u) & 0xFFu) << 23);
      }
    }
  }
}

// ------------------------------------------------- DQ-fp8 with a per-row scale
// The per-token variant of the rowwise FP8 convert: each row is dequantized
// exactly as DQ-bf16 does (dq_bf16_chunk) and re-quantized with one FP32 scale
// per row, the per-token FP8 convention of this library (fp8_token.cu):
//   amax = max(eps, max |x|) (NaN ignored), scale = amax / 448,
//   q = E4M3(clamp(x * (448 / amax), +-448)).
// One CTA per row; with kWords > 0 a thread keeps its kWords decoded 4-byte
// code words (8 BF16 each) in registers between the amax and the quantize
// pass, otherwise (long rows) it decodes the codes again from L1/L2.
constexpr int kRsThreads = 128;

template <int kWords>
__global__ void __launch_bounds__(kRsThreads) dq_fp8_rowscale_kernel(
    const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales, int64_t M, int64_t Kb,
    float eps, uint8_t* __restrict__ out, float* __restrict__ scale_out) {
  __shared__ uint32_t red_bits[kRsThreads / 32];
  __shared__ float red_f[kRsThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t nw = Kb / 4, S = Kb / 16;
  constexpr int kHeld = kWords > 0 ? kWords : 1;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
    const uint8_t* cr = codes + r * Kb;
    const uint8_t* sr = scales + r * S;
    auto decode = [&](int64_t c) {
      return dq_bf16_chunk(ld_stream_u32(cr + c * 4), (uint32_t)sr[c >> 2]);
    };
    uint4 v[kHeld];
    uint32_t m = 0;
    auto absmax4 = [&](const uint4& d) {
      m = vmax_u16x2(m, d.x & 0x7FFF7FFFu);
      m = vmax_u16x2(m, d.y & 0x7FFF7FFFu);
      m = vmax_u16x2(m, d.z & 0x7FFF7FFFu);
      m = vmax_u16x2(m, d.w & 0x7FFF7FFFu);
    };
    auto fmax4 = [](float a, const uint4& d) {
      const uint32_t w[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        a = fmaxf(a, fabsf(bf16lo_to_f(w[j])));
        a = fmaxf(a, fabsf(bf16hi_to_f(w[j])));
      }
      return a;
    };
    if constexpr (kWords > 0) {
#pragma unroll
      for (int i = 0; i < kWords; ++i) {
        const int64_t c = (int64_t)i * kRsThreads + t;
        v[i] = c < nw ? decode(c) : make_uint4(0, 0, 0, 0);
        absmax4(v[i]);
      }
    } else {
      for (int64_t c = t; c < nw; c += kRsThreads) absmax4(decode(c));
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
      if constexpr (kWords > 0) {
#pragma unroll
        for (int i = 0; i < kWords; ++i) a = fmax4(a, v[i]);
      } else {
        for (int64_t c = t; c < nw; c += kRsThreads) a = fmax4(a, decode(c));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
      if (lane == 0) red_f[warp] = a;
      __syncthreads();
      amax = fmaxf(fmaxf(red_f[0], red_f[1]), fmaxf(red_f[2], red_f[3]));
    }
    const float qs = 448.0f / amax;
    if (t == 0) scale_out[r] = amax / 448.0f;
    auto quant8 = [&](int64_t c, const uint4& d) {
      const uint32_t w[4] = {d.x, d.y, d.z, d.w};
      uint32_t o[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float a0 = fminf(fmaxf(bf16lo_to_f(w[2 * j]) * qs, -448.0f), 448.0f);
        const float a1 = fminf(fmaxf(bf16hi_to_f(w[2 * j]) * qs, -448.0f), 448.0f);
        const float a2 = fminf(fmaxf(bf16lo_to_f(w[2 * j + 1]) * qs, -448.0f), 448.0f);
        const float a3 = fminf(fmaxf(bf16hi_to_f(w[2 * j + 1]) * qs, -448.0f), 448.0f);
        o[j] = cvt_e4m3x2(a0, a1) | (cvt_e4m3x2(a2, a3) << 16);
      }
      st_stream_v2(out + r * 2 * Kb + c * 8, make_uint2(o[0], o[1]));
    };
    if constexpr (kWords > 0) {
#pragma unroll
      for (int i = 0; i < kWords; ++i) {
        const int64_t c = (int64_t)i * kRsThreads + t;
        if (c < nw) quant8(c, v[i]);
      }
    } else {
      for (int64_t c = t; c < nw; c += kRsThreads) quant8(c, decode(c));
    }
    __syncthreads();  // red_* reused by the next row
  }
}

int grid_for(const void* kern, int64_t work_lanes, int per_lane) {
  const int64_t want = cdiv(work_lanes, 256LL * per_lane);
  const int64_t cap = (int64_t)persistent_ctas(kern, 256, 0) * 2;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_per_token_Mxfp4ToBf16_dequant(const void* input, const void* input_s,
                                                        int64_t M, int64_t Kb, void* output,
                                                        mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && Kb >= 0 && Kb % 16 == 0, MXB_ERR_INVALID_ARGUMENT,
              "dequant_bf16: need Kb %% 16 == 0 (one E8M0 byte per 16 code bytes), got %lld",
              (long long)Kb);
  if (M == 0 || Kb == 0) return MXB_OK;
  MXB_REQUIRE(input && input_s && output, MXB_ERR_INVALID_ARGUMENT, "dequant_bf16: null pointer");
  MXB_REQUIRE(aligned(input, 4) && aligned(output, 16), MXB_ERR_MISALIGNED,
              "dequant_bf16: input must be 4-byte and output 16-byte aligned");
  const int64_t chunks = M * Kb / 4;
  const int grid = grid_for((const void*)dq_bf16_kernel, chunks, kDqUnroll);
  dq_bf16_kernel<<<grid, 256, 0, to_cuda(stream)>>>((const uint8_t*)input, (const uint8_t*)input_s,
                                                    chunks, (uint8_t*)output);
  return launch_status("dequant_bf16");
}

static mxb_status mxfp4_to_fp8_rows(const void* input, const void* input_s, int64_t M, int64_t Kb,
                                    void* output_q, void* output_s, bool strict,
                                    mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && Kb >= 0 && Kb % 64 == 0, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8: need Kb %% 64 == 0 (1x128 groups), got %lld", (long long)Kb);
  if (M == 0 || Kb == 0) return MXB_OK;
  MXB_REQUIRE(input && input_s && output_q && output_s, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8: null pointer");
  MXB_REQUIRE(aligned(input, 8) && aligned(input_s, 4) && aligned(output_q, 16) &&
                  aligned(output_s, 4),
              MXB_ERR_MISALIGNED, "mxfp4_to_fp8: misaligned pointer");
  const int64_t lanes = M * Kb / 8;
  const int grid = grid_for((const void*)dq_fp8_row_kernel<false>, lanes, kFp8RowUnroll);
  if (strict)
    dq_fp8_row_kernel<true><<<grid, 256, 0, to_cuda(stream)>>>(
        (const uint8_t*)input, (const uint8_t*)input_s, M, Kb, (uint8_t*)output_q,
        (float*)output_s);
  else
    dq_fp8_row_kernel<false><<<grid, 256, 0, to_cuda(stream)>>>(
        (const uint8_t*)input, (const uint8_t*)input_s, M, Kb, (uint8_t*)output_q,
        (float*)output_s);
  return launch_status("mxfp4_to_fp8");
}

extern "C" mxb_status mxb_per_token_Mxfp4ToFp8(const void* input, const void* input_s, int64_t M,
                                               int64_t Kb, void* output_q, void* output_s,
                                               mxb_stream_t stream) {
  return mxfp4_to_fp8_rows(input, input_s, M, Kb, output_q, output_s, false, stream);
}

extern "C" mxb_status mxb_per_token_Mxfp4ToFp8_strict(const void* input, const void* input_s,
                                                      int64_t M, int64_t Kb, void* output_q,
                                                      void* output_s, mxb_stream_t stream) {
  return mxfp4_to_fp8_rows(input, input_s, M, Kb, output_q, output_s, true, stream);
}

extern "C" mxb_status mxb_per_token_Mxfp4ToFp8_rowscale(const void* input, const void* input_s,
                                                        int64_t M, int64_t Kb, void* output_q,
                                                        void* output_s, float eps,
                                                        mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && Kb >= 0 && Kb % 16 == 0, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_rowscale: need Kb %% 16 == 0, got %lld", (long long)Kb);
  if (M == 0 || Kb == 0) return MXB_OK;
  MXB_REQUIRE(input && input_s && output_q && output_s, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_rowscale: null pointer");
  MXB_REQUIRE(aligned(input, 4) && aligned(output_q, 8) && aligned(output_s, 4),
              MXB_ERR_MISALIGNED, "mxfp4_to_fp8_rowscale: misaligned pointer");
  const int64_t per = cdiv(Kb / 4, kRsThreads);
  const int grid = (int)(M < 148LL * 64 ? M : 148LL * 64);
  cudaStream_t s = to_cuda(stream);
  auto* ci = (const uint8_t*)input;
  auto* si = (const uint8_t*)input_s;
  auto* qo = (uint8_t*)output_q;
  auto* so = (float*)output_s;
  if (per <= 4)
    dq_fp8_rowscale_kernel<4><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  else if (per <= 8)
    dq_fp8_rowscale_kernel<8><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  else if (per <= 16)
    dq_fp8_rowscale_kernel<16><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  else
    dq_fp8_rowscale_kernel<0><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  return launch_status("mxfp4_to_fp8_rowscale");
}

extern "C" mxb_status mxb_per_token_Mxfp4ToBf16ToFp8(const void* input, const void* input_s,
                                                     int64_t M, int64_t Kb, void* output_q,
                                                     void* output_s, mxb_stream_t stream) {
  return mxb_per_token_Mxfp4ToFp8(input, input_s, M, Kb, output_q, output_s, stream);
}
