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
#include <cuda_bf16.h>

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
// A lane converts one 32-element block: 16 code bytes (one 16-byte load) and
// its E8M0 byte into 32 FP8 bytes (two 16-byte stores).  Blocks are contiguous
// in the flat code array and so are their scale bytes, so lane b reads scale
// byte b; the four lanes of a 1x128 group are adjacent (the groups of a row
// start at multiples of 4 blocks), so the group max is two shuffles.  The
// element arithmetic is a lookup in the compile-time table row for
// d = max_e - e (fp8_lut.cuh), four nibbles per lookup.  kRowBlk blocks per
// lane are in flight per iteration.
__device__ const Fp8Lut g_lut_row = make_fp8_lut(false);
__device__ const Fp8Lut g_lut_row_strict = make_fp8_lut_strict();

constexpr int kRowBlk = 4;  // measured on config 3: 1 -> 80.1 us, 2 -> 83.6 us, 4 -> 79.6 us

template <bool kStrict>
__global__ void __launch_bounds__(256) dq_fp8_row_kernel(const uint8_t* __restrict__ codes,
                                                         const uint8_t* __restrict__ scales,
                                                         int64_t M, int64_t Kb,
                                                         uint8_t* __restrict__ out,
                                                         float* __restrict__ scales_out) {
  const int64_t nblk = M * Kb / 16;
  const int64_t groups_per_row = Kb / 64;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * kRowBlk;
  const int lane = threadIdx.x & 31;
  const Fp8Lut& lut = kStrict ? g_lut_row_strict : g_lut_row;
  for (int64_t base = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) * kRowBlk;
       base < nblk; base += stride) {
    uint4 c[kRowBlk];
    uint32_t e[kRowBlk];
#pragma unroll
    for (int k = 0; k < kRowBlk; ++k) {
      const int64_t b = base + k * 32 + lane;
      if (b < nblk) {
        c[k] = ld_stream_v4(codes + b * 16);
        e[k] = ld_stream_u8(scales + b);
      } else {
        c[k] = make_uint4(0u, 0u, 0u, 0u);
        e[k] = 0u;
      }
    }
#pragma unroll
    for (int k = 0; k < kRowBlk; ++k) {
      const int64_t b = base + k * 32 + lane;
      uint32_t mx = max(e[k], __shfl_xor_sync(0xffffffffu, e[k], 1));
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const uint4 t = __ldg(reinterpret_cast<const uint4*>(lut.v[mx - e[k]]));
      if (b >= nblk) continue;
      const uint4 o0 = make_uint4(lut_lookup4(c[k].x, t.x, t.y, t.z, t.w),
                                  lut_lookup4(c[k].x >> 16, t.x, t.y, t.z, t.w),
                                  lut_lookup4(c[k].y, t.x, t.y, t.z, t.w),
                                  lut_lookup4(c[k].y >> 16, t.x, t.y, t.z, t.w));
      const uint4 o1 = make_uint4(lut_lookup4(c[k].z, t.x, t.y, t.z, t.w),
                                  lut_lookup4(c[k].z >> 16, t.x, t.y, t.z, t.w),
                                  lut_lookup4(c[k].w, t.x, t.y, t.z, t.w),
                                  lut_lookup4(c[k].w >> 16, t.x, t.y, t.z, t.w));
      st_stream_v4(out + b * 32, o0);
      st_stream_v4(out + b * 32 + 16, o1);
      if ((lane & 3) == 0) {
        const int64_t grp = b >> 2;
        int64_t r;
        if (grp <= (int64_t)UINT32_MAX && groups_per_row <= (int64_t)UINT32_MAX) {
          r = (uint32_t)grp / (uint32_t)groups_per_row;  // 32-bit division whenever it suffices
        } else {
          r = grp / groups_per_row;
        }
        const int64_t gc = grp - r * groups_per_row;
        scales_out[gc * M + r] = __uint_as_float(((mx - 6u) & 0xFFu) << 23);
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
// One CTA per row.  A thread holds kChunks 16-byte code chunks (one 32-element
// block each) in registers.  The row amax needs no decode: the largest value
// of a block is its largest E2M1 magnitude times the block's factor, one
// product per block, rounded to BF16 as the dequantize rounds it (NaN from
// 0 * Inf never wins a float max).  The second pass decodes each chunk and
// writes its 32 FP8 bytes.  kChunks = 0: rows too long for registers, codes
// re-read (from L1/L2).
constexpr int kRsThreads = 128;


// Largest |value| of one 32-element block as the dequantize produces it.
__device__ __forceinline__ float block_amax(uint4 c, uint32_t e) {
  // the 3-bit magnitude fields of the 32 nibbles, in four groups whose fields
  // sit at the same place of each 16-bit lane (nibbles 0/4, 1/5, 2/6, 3/7 of a
  // word), reduced with the native 16-bit-lane max
  uint32_t g[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t msk = 0x00070007u << (4 * k);
    g[k] = vmax_u16x2(vmax_u16x2(c.x & msk, c.y & msk), vmax_u16x2(c.z & msk, c.w & msk));
  }
  uint32_t m = vmax_u16x2(vmax_u16x2(g[0], g[1] >> 4), vmax_u16x2(g[2] >> 8, g[3] >> 12));
  m = max(m & 0xFFFFu, m >> 16);
  // E2M1 magnitude of m, exactly: {0, .5, 1, 1.5, 2, 3, 4, 6}
  const float mag = m < 2u ? 0.5f * (float)m : (float)((2u | (m & 1u)) << ((m >> 1) - 1u)) * 0.5f;
  const float p = mag * e8m0_to_f(e);  // exact, or the float product the dequantize rounds
  return __bfloat162float(__float2bfloat16_rn(p));
}

__device__ __forceinline__ void quant_chunk32(uint4 c, uint32_t e, float qs, uint8_t* dst) {
  const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 d = dq_bf16_chunk(cw[j], e);
    const uint32_t w[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float a0 = fminf(fmaxf(bf16lo_to_f(w[2 * h]) * qs, -448.0f), 448.0f);
      const float a1 = fminf(fmaxf(bf16hi_to_f(w[2 * h]) * qs, -448.0f), 448.0f);
      const float a2 = fminf(fmaxf(bf16lo_to_f(w[2 * h + 1]) * qs, -448.0f), 448.0f);
      const float a3 = fminf(fmaxf(bf16hi_to_f(w[2 * h + 1]) * qs, -448.0f), 448.0f);
      o[2 * j + h] = cvt_e4m3x2(a0, a1) | (cvt_e4m3x2(a2, a3) << 16);
    }
  }
  st_stream_v4(dst, make_uint4(o[0], o[1], o[2], o[3]));
  st_stream_v4(dst + 16, make_uint4(o[4], o[5], o[6], o[7]));
}

// The same for a block of a row without an E8M0 byte of 255: its values
// e2m1 * f (f = 2^(e-127), exact in BF16) times qs round once either way, so
// the block's factor f * qs (exact: f is a power of two; capped so that an
// all-zero block far above the row's amax keeps its zeros) multiplies the
// decoded codes directly, and every |v| <= 448 (1 + 2^-23) converts under the
// saturating conversion exactly as clamp-then-convert does.
__device__ __forceinline__ void quant_chunk32_fast(uint4 c, uint32_t e, float qs, uint8_t* dst) {
  const float m = fminf(e8m0_to_f(e) * qs, 1e30f);
  const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v[8];
    decode8_scaled(cw[j], m, v);
    o[2 * j] = cvt_e4m3x4(v[0], v[1], v[2], v[3]);
    o[2 * j + 1] = cvt_e4m3x4(v[4], v[5], v[6], v[7]);
  }
  st_stream_v4(dst, make_uint4(o[0], o[1], o[2], o[3]));
  st_stream_v4(dst + 16, make_uint4(o[4], o[5], o[6], o[7]));
}

template <int kChunks>
__global__ void __launch_bounds__(kRsThreads) dq_fp8_rowscale_kernel(
    const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales, int64_t M, int64_t Kb,
    float eps, uint8_t* __restrict__ out, float* __restrict__ scale_out) {
  __shared__ float red[kRsThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t nc = Kb / 16;  // 16-byte chunks (= blocks) per row
  constexpr int kHeld = kChunks > 0 ? kChunks : 1;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
    const uint8_t* cr = codes + r * Kb;
    const uint8_t* sr = scales + r * nc;
    uint8_t* orow = out + r * 2 * Kb;
    uint4 c[kHeld];
    uint32_t e[kHeld];
    float a = eps;
    bool inf_scale = false;  // an E8M0 byte of 255: Inf and NaN values need the clamps
    if constexpr (kChunks > 0) {
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int64_t k = (int64_t)i * kRsThreads + t;
        if (k < nc) {
          c[i] = ld_stream_v4(cr + k * 16);
          e[i] = ld_stream_u8(sr + k);
        } else {
          c[i] = make_uint4(0, 0, 0, 0);
          e[i] = 0;
        }
      }
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        a = fmaxf(a, block_amax(c[i], e[i]));
        inf_scale = inf_scale || e[i] == 255u;
      }
    } else {
      for (int64_t k = t; k < nc; k += kRsThreads) {
        a = fmaxf(a, block_amax(*reinterpret_cast<const uint4*>(cr + k * 16), sr[k]));
        inf_scale = inf_scale || sr[k] == 255u;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) red[warp] = a;
    inf_scale = __syncthreads_or(inf_scale);
    const float amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();  // red is reused by the next row
    const float qs = 448.0f / amax;
    if (t == 0) scale_out[r] = amax / 448.0f;
    if constexpr (kChunks > 0) {
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int64_t k = (int64_t)i * kRsThreads + t;
        if (k >= nc) continue;
        if (inf_scale)
          quant_chunk32(c[i], e[i], qs, orow + k * 32);
        else
          quant_chunk32_fast(c[i], e[i], qs, orow + k * 32);
      }
    } else {
      for (int64_t k = t; k < nc; k += kRsThreads) {
        if (inf_scale)
          quant_chunk32(ld_stream_v4(cr + k * 16), ld_stream_u8(sr + k), qs, orow + k * 32);
        else
          quant_chunk32_fast(ld_stream_v4(cr + k * 16), ld_stream_u8(sr + k), qs, orow + k * 32);
      }
    }
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
  MXB_REQUIRE(aligned(input, 16) && aligned(output_q, 16) && aligned(output_s, 4),
              MXB_ERR_MISALIGNED, "mxfp4_to_fp8: input and output_q must be 16-byte aligned");
  const int64_t lanes = M * Kb / 16;
  const int grid = grid_for((const void*)dq_fp8_row_kernel<false>, lanes, kRowBlk);
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
  MXB_REQUIRE(aligned(input, 16) && aligned(output_q, 16) && aligned(output_s, 4),
              MXB_ERR_MISALIGNED, "mxfp4_to_fp8_rowscale: input and output_q must be 16-byte "
              "aligned");
  const int64_t per = cdiv(Kb / 16, kRsThreads);
  const int grid = (int)(M < 148LL * 64 ? M : 148LL * 64);
  cudaStream_t s = to_cuda(stream);
  auto* ci = (const uint8_t*)input;
  auto* si = (const uint8_t*)input_s;
  auto* qo = (uint8_t*)output_q;
  auto* so = (float*)output_s;
  if (per <= 1)
    dq_fp8_rowscale_kernel<1><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  else if (per <= 2)
    dq_fp8_rowscale_kernel<2><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  else if (per <= 4)
    dq_fp8_rowscale_kernel<4><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  else if (per <= 8)
    dq_fp8_rowscale_kernel<8><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  else
    dq_fp8_rowscale_kernel<0><<<grid, kRsThreads, 0, s>>>(ci, si, M, Kb, eps, qo, so);
  return launch_status("mxfp4_to_fp8_rowscale");
}

extern "C" mxb_status mxb_per_token_Mxfp4ToBf16ToFp8(const void* input, const void* input_s,
                                                     int64_t M, int64_t Kb, void* output_q,
                                                     void* output_s, mxb_stream_t stream) {
  return mxb_per_token_Mxfp4ToFp8(input, input_s, M, Kb, output_q, output_s, stream);
}
