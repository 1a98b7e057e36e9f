// BF16 -> MXFP4 quantize kernels for sm_100a: rowwise (Q-row) and the fused
// one-pass rowwise + columnwise quantize (Q-row + Q-col), with an optional
// tcgen05 swizzled copy of the row scales.
//
// Bit-exact contract (reference: code/kernel/per_token_quant_mxfp4.cu:121-266):
//   amax  = max(eps, max |x|) over a 1x32 block (32x1 for columnwise)
//   y_s   = exp2f(ceilf(log2f(max(amax / fp4_max, 1e-10))))
//   scale = (uint8)((int)log2f(y_s) + 127)
//   code  = E2M1_RNE(clamp(x * (1 / y_s), fp4_min, fp4_max)), sign kept on zero
//
// Fast path (fp4_max = 6, fp4_min = -6, eps <= 6e-10, the reference API's only
// configuration): the block amax is an integer max over BF16 magnitudes, the
// exponent k = ceil(log2 y) is read from y's bits (exact, because a BF16 amax
// divided by 6 is either a power of two or at least 0.5% away from one), and
// the codes come from Blackwell's cvt.rn.satfinite.e2m1x2.f32.  Blocks holding
// Inf/NaN, and every block when the parameters differ from the defaults, take
// the generic path, which evaluates the reference formula literally and
// encodes with the reference's integer rounding.
#include <cuda_bf16.h>

#include "capi_util.h"
#include "common.cuh"

namespace mxb {
namespace {

struct QuantParams {
  float eps, fp4_min, fp4_max;
};

// Reference E2M1 rounding of an already clamped float
// (per_token_quant_mxfp4.cu:213-256): re-bias the exponent from 127 to 1,
// denormalise values below 1.0 by a right shift, round to nearest even on the
// two retained bits, saturate at code 7, keep the sign in bit 3.
__device__ __forceinline__ uint32_t e2m1_encode_generic(float q) {
  const uint32_t b = __float_as_uint(q);
  const uint32_t sign = b >> 28 & 0x8u;
  uint32_t ex = (b >> 23) & 0xFFu;
  uint32_t man = b & 0x7FFFFFu;
  if (ex < 127u) {
    const uint32_t sh = 126u - ex;
    man = sh >= 32u ? 0u : ((0x400000u | (man >> 1)) >> sh);
  }
  ex = (ex > 126u ? ex : 126u) - 126u;
  const uint32_t m2 = man >> 21;
  const uint32_t inc = (m2 & 1u) & (((man & 0x1FFFFFu) != 0u) | ((m2 >> 1) & 1u));
  uint32_t r = (((ex << 2) | m2) + inc) >> 1;
  r = r > 7u ? 7u : r;
  return sign | r;
}

// The reference scale rule, evaluated literally (generic path).
__device__ __forceinline__ void scale_generic(float amax, const QuantParams& p, float& inv,
                                              uint32_t& byte) {
  float y = amax / p.fp4_max;
  y = exp2f(ceilf(log2f(fmaxf(y, 1e-10f))));
  const int t = (int)log2f(y);  // +Inf saturates to INT_MAX, as on the reference path
  byte = ((uint32_t)t + 127u) & 0xFFu;
  inv = 1.0f / y;
}

// Fast scale rule from the largest BF16 magnitude pattern `mb` (finite).
__device__ __forceinline__ void scale_fast(uint32_t mb, float eps, float& inv, uint32_t& byte) {
  const float amax = fmaxf(eps, __uint_as_float(mb << 16));
  const float y = fmaxf(__fdiv_rn(amax, 6.0f), 1e-10f);
  const uint32_t yb = __float_as_uint(y);
  const int k = (int)(yb >> 23) - 127 + ((yb & 0x7FFFFFu) != 0u);
  byte = (uint32_t)(k + 127);
  inv = __uint_as_float((uint32_t)(127 - k) << 23);
}

// Largest |x| BF16 pattern of the 2n values in `w` (NaN patterns sort above Inf).
template <int N>
__device__ __forceinline__ uint32_t max_abs_bits(const uint32_t (&w)[N]) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < N; ++i) m = vmax_u16x2(m, w[i] & 0x7FFF7FFFu);
  return max(m & 0xFFFFu, m >> 16);
}

// Encodes the 2N BF16 values of w (element order) with a known inverse scale
// into N/2 code words (fast path: |x * inv| <= 6 is guaranteed).
template <int N>
__device__ __forceinline__ void encode_fast(const uint32_t (&w)[N], float inv,
                                            uint32_t (&out)[N / 4]) {
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = bf16lo_to_f(w[4 * i + j]) * inv;
      v[2 * j + 1] = bf16hi_to_f(w[4 * i + j]) * inv;
    }
    out[i] = cvt_e2m1x8(v);
  }
}

template <int N>
__device__ __forceinline__ void encode_generic(const uint32_t (&w)[N], float inv,
                                               const QuantParams& p, uint32_t (&out)[N / 4]) {
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    uint32_t r = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float q0 = fminf(fmaxf(bf16lo_to_f(w[4 * i + j]) * inv, p.fp4_min), p.fp4_max);
      const float q1 = fminf(fmaxf(bf16hi_to_f(w[4 * i + j]) * inv, p.fp4_min), p.fp4_max);
      r |= (e2m1_encode_generic(q0) | (e2m1_encode_generic(q1) << 4)) << (8 * j);
    }
    out[i] = r;
  }
}

template <int N>
__device__ __forceinline__ float amax_generic(const uint32_t (&w)[N], float init) {
  float a = init;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    a = fmaxf(a, fabsf(bf16lo_to_f(w[i])));
    a = fmaxf(a, fabsf(bf16hi_to_f(w[i])));
  }
  return a;
}

__device__ __forceinline__ int64_t swizzle_offset(int64_t r, int64_t c, int64_t sp4) {
  return ((r >> 7) * sp4 + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3);
}

// ------------------------------------------------------------------ Q-row
// Two lanes per 32-element block, 16 elements (two 16-byte loads) per lane.
// A warp covers 16 consecutive blocks: 1 KiB of contiguous input per step.
template <bool kFast>
__global__ void __launch_bounds__(256) quant_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                         int64_t M, int64_t K, int64_t ldx,
                                                         uint8_t* __restrict__ codes,
                                                         uint8_t* __restrict__ scales,
                                                         QuantParams p) {
  const int64_t G = K >> 5;
  const int64_t halves = M * G * 2;
  const int lane = threadIdx.x & 31;
  const unsigned pair_mask = 3u << (lane & ~1);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); base < halves;
       base += stride) {
    const int64_t h = base + lane;
    if (h >= halves) continue;  // pairs are both in or both out (halves is even)
    const int64_t grp = h >> 1;
    const int half = (int)(h & 1);
    const int64_t r = grp / G, g = grp - r * G;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(x + r * ldx + g * 32 + half * 16);
    const uint4 a = ld_stream_v4(src), b = ld_stream_v4(src + 16);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t mb = max_abs_bits(w);
    mb = max(mb, __shfl_xor_sync(pair_mask, mb, 1));
    float inv;
    uint32_t byte;
    uint32_t out[2];
    if (kFast && mb < 0x7F80u) {
      scale_fast(mb, p.eps, inv, byte);
      encode_fast(w, inv, out);
    } else {
      float am = amax_generic(w, p.eps);
      am = fmaxf(am, __shfl_xor_sync(pair_mask, am, 1));
      scale_generic(am, p, inv, byte);
      encode_generic(w, inv, p, out);
    }
    st_stream_v2(codes + r * (K >> 1) + g * 16 + half * 8, make_uint2(out[0], out[1]));
    if (half == 0) scales[r * G + g] = (uint8_t)byte;
  }
}

// ------------------------------------------------------- fused Q-row + Q-col
// One CTA quantizes a 128x128 tile: phase 1 reads the tile with 16-byte loads,
// quantizes its rows from registers and parks the BF16 tile in shared memory;
// phase 2 quantizes its columns (32-row blocks) from shared memory.  HBM sees
// every input byte once and every output byte once.
constexpr int kTile = 128;
constexpr int kRowColThreads = 256;

template <bool kFast, bool kRows>
__global__ void __launch_bounds__(kRowColThreads) quant_rowcol_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K, int64_t ldx,
    uint8_t* __restrict__ codes_row, uint8_t* __restrict__ scales_row,
    uint8_t* __restrict__ codes_col, uint8_t* __restrict__ scales_col,
    uint8_t* __restrict__ scales_swz, QuantParams p) {
  __shared__ __align__(16) uint32_t tile[kTile][kTile / 2];  // BF16 pairs, 32 KiB
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t row0 = (int64_t)blockIdx.y * kTile, col0 = (int64_t)blockIdx.x * kTile;
  const int64_t G = K >> 5, Gc = M >> 5;
  const int64_t sp4 = (G + 3) >> 2;

  // ---- phase 1: load, row-quantize, stage
  uint4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = i * kRowColThreads + t;
    const int r = c >> 4, cc = c & 15;
    const bool ok = (row0 + r < M) && (col0 + cc * 8 < K);
    v[i] = ok ? ld_stream_v4(x + (row0 + r) * ldx + col0 + cc * 8) : make_uint4(0, 0, 0, 0);
  }
  const unsigned quad_mask = 0xFu << (lane & ~3);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = i * kRowColThreads + t;
    const int r = c >> 4, cc = c & 15;
    *reinterpret_cast<uint4*>(&tile[r][cc * 4]) = v[i];
    if (kRows) {
      const bool ok = (row0 + r < M) && (col0 + cc * 8 < K);  // uniform per quad
      if (ok) {
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        uint32_t mb = max_abs_bits(w);
        mb = max(mb, __shfl_xor_sync(quad_mask, mb, 1));
        mb = max(mb, __shfl_xor_sync(quad_mask, mb, 2));
        float inv;
        uint32_t byte;
        uint32_t out[1];
        if (kFast && mb < 0x7F80u) {
          scale_fast(mb, p.eps, inv, byte);
          encode_fast(w, inv, out);
        } else {
          float am = amax_generic(w, p.eps);
          am = fmaxf(am, __shfl_xor_sync(quad_mask, am, 1));
          am = fmaxf(am, __shfl_xor_sync(quad_mask, am, 2));
          scale_generic(am, p, inv, byte);
          encode_generic(w, inv, p, out);
        }
        const int64_t gr = row0 + r, gc = col0 + cc * 8;
        st_stream_u32(codes_row + gr * (K >> 1) + (gc >> 1), out[0]);
        if ((cc & 3) == 0) {
          const int64_t g = gc >> 5;
          scales_row[gr * G + g] = (uint8_t)byte;
          if (scales_swz) scales_swz[swizzle_offset(gr, g, sp4)] = (uint8_t)byte;
        }
      }
    }
  }
  __syncthreads();

  // ---- phase 2: column-quantize 32-row blocks from shared memory
  const int rb = warp >> 1;                 // 32-row block of the tile
  const int cp = ((warp & 1) << 5) | lane;  // column pair within the tile
  const int64_t gc = col0 + 2 * cp;
  const int64_t gr = row0 + rb * 32;
  if (gr >= M || gc >= K) return;
  uint32_t w[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) w[i] = tile[rb * 32 + i][cp];
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) m = vmax_u16x2(m, w[i] & 0x7FFF7FFFu);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t mb = h ? (m >> 16) : (m & 0xFFFFu);
    // the 32 values of column gc + h, as BF16 pairs (rows 2i, 2i+1)
    uint32_t cw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      cw[i] = h ? prmt(w[2 * i], w[2 * i + 1], 0x7632u) : prmt(w[2 * i], w[2 * i + 1], 0x5410u);
    float inv;
    uint32_t byte;
    uint32_t out[4];
    if (kFast && mb < 0x7F80u) {
      scale_fast(mb, p.eps, inv, byte);
      encode_fast(cw, inv, out);
    } else {
      scale_generic(amax_generic(cw, p.eps), p, inv, byte);
      encode_generic(cw, inv, p, out);
    }
    const int64_t c = gc + h;
    st_stream_v4(codes_col + c * (M >> 1) + (gr >> 1), make_uint4(out[0], out[1], out[2], out[3]));
    scales_col[c * Gc + (gr >> 5)] = (uint8_t)byte;
  }
}

__global__ void swizzle_scales_kernel(const uint8_t* __restrict__ s, int64_t M, int64_t S,
                                      uint8_t* __restrict__ out) {
  const int64_t Mp = (M + 127) / 128 * 128, Sp = (S + 3) / 4 * 4;
  const int64_t total = Mp * Sp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / Sp, c = i - r * Sp;
    const uint8_t v = (r < M && c < S) ? s[r * S + c] : (uint8_t)0;
    out[swizzle_offset(r, c, Sp >> 2)] = v;
  }
}

bool fast_params(float eps, float fp4_min, float fp4_max) {
  return fp4_max == 6.0f && fp4_min == -6.0f && eps >= 0.0f && eps <= 6e-10f;
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_per_token_group_quant_fp4(const void* input, int64_t M, int64_t K,
                                                    int64_t ldx, void* output_q, void* output_s,
                                                    int group_size, float eps, float fp4_min,
                                                    float fp4_max, int scale_ue8m0,
                                                    mxb_stream_t stream) {
  MXB_REQUIRE(group_size == 32, MXB_ERR_UNSUPPORTED,
              "quant_fp4: group_size must be 32 (got %d)", group_size);
  MXB_REQUIRE(!scale_ue8m0, MXB_ERR_UNSUPPORTED,
              "quant_fp4: scale_ue8m0=True is rejected, as by the reference host assert");
  MXB_REQUIRE(M >= 0 && K >= 0 && K % 32 == 0, MXB_ERR_INVALID_ARGUMENT,
              "quant_fp4: need M >= 0 and K %% 32 == 0 (M=%lld K=%lld)", (long long)M,
              (long long)K);
  MXB_REQUIRE(ldx >= K && ldx % 8 == 0, MXB_ERR_MISALIGNED,
              "quant_fp4: row pitch must be >= K and a multiple of 8 elements");
  if (M == 0 || K == 0) return MXB_OK;
  MXB_REQUIRE(input && output_q && output_s, MXB_ERR_INVALID_ARGUMENT, "quant_fp4: null pointer");
  MXB_REQUIRE(aligned(input, 16) && aligned(output_q, 8), MXB_ERR_MISALIGNED,
              "quant_fp4: input must be 16-byte and output_q 8-byte aligned");
  const QuantParams p{eps, fp4_min, fp4_max};
  const bool fast = fast_params(eps, fp4_min, fp4_max);
  const void* kern = fast ? (const void*)quant_rows_kernel<true> : (const void*)quant_rows_kernel<false>;
  const int64_t halves = M * (K / 32) * 2;
  int64_t want = cdiv(halves, 256);
  const int64_t cap = (int64_t)persistent_ctas(kern, 256, 0) * 4;
  const int grid = (int)(want < cap ? want : cap);
  if (fast)
    quant_rows_kernel<true><<<grid, 256, 0, to_cuda(stream)>>>(
        (const __nv_bfloat16*)input, M, K, ldx, (uint8_t*)output_q, (uint8_t*)output_s, p);
  else
    quant_rows_kernel<false><<<grid, 256, 0, to_cuda(stream)>>>(
        (const __nv_bfloat16*)input, M, K, ldx, (uint8_t*)output_q, (uint8_t*)output_s, p);
  return launch_status("quant_fp4");
}

extern "C" mxb_status mxb_quant_mxfp4_rowcol(const void* input, int64_t M, int64_t K, int64_t ldx,
                                             void* codes_row, void* scales_row, void* codes_col,
                                             void* scales_col, void* scales_row_swizzled,
                                             float eps, float fp4_min, float fp4_max,
                                             mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && K >= 0 && M % 32 == 0 && K % 32 == 0, MXB_ERR_INVALID_ARGUMENT,
              "quant_rowcol: need M %% 32 == 0 and K %% 32 == 0 (M=%lld K=%lld)", (long long)M,
              (long long)K);
  MXB_REQUIRE(ldx >= K && ldx % 8 == 0, MXB_ERR_MISALIGNED,
              "quant_rowcol: row pitch must be >= K and a multiple of 8 elements");
  MXB_REQUIRE((codes_row == nullptr) == (scales_row == nullptr), MXB_ERR_INVALID_ARGUMENT,
              "quant_rowcol: codes_row and scales_row must both be given or both be NULL");
  MXB_REQUIRE(!(scales_row_swizzled && !codes_row), MXB_ERR_INVALID_ARGUMENT,
              "quant_rowcol: a swizzled row-scale output needs the row outputs");
  if (M == 0 || K == 0) return MXB_OK;
  MXB_REQUIRE(input && codes_col && scales_col, MXB_ERR_INVALID_ARGUMENT,
              "quant_rowcol: null pointer");
  MXB_REQUIRE(aligned(input, 16) && aligned(codes_col, 16) && (!codes_row || aligned(codes_row, 4)),
              MXB_ERR_MISALIGNED, "quant_rowcol: input/codes_col must be 16-byte aligned");
  cudaStream_t s = to_cuda(stream);
  if (scales_row_swizzled) {
    const int64_t bytes = (M + 127) / 128 * 128 * ((K / 32 + 3) / 4 * 4);
    cudaError_t e = cudaMemsetAsync(scales_row_swizzled, 0, (size_t)bytes, s);
    MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "quant_rowcol: memset failed: %s",
                cudaGetErrorString(e));
  }
  const QuantParams p{eps, fp4_min, fp4_max};
  const bool fast = fast_params(eps, fp4_min, fp4_max);
  const dim3 grid((unsigned)cdiv(K, kTile), (unsigned)cdiv(M, kTile));
  auto* xi = (const __nv_bfloat16*)input;
  auto* cr = (uint8_t*)codes_row;
  auto* sr = (uint8_t*)scales_row;
  auto* cc = (uint8_t*)codes_col;
  auto* sc = (uint8_t*)scales_col;
  auto* sw = (uint8_t*)scales_row_swizzled;
  if (codes_row) {
    if (fast)
      quant_rowcol_kernel<true, true><<<grid, kRowColThreads, 0, s>>>(xi, M, K, ldx, cr, sr, cc, sc, sw, p);
    else
      quant_rowcol_kernel<false, true><<<grid, kRowColThreads, 0, s>>>(xi, M, K, ldx, cr, sr, cc, sc, sw, p);
  } else {
    if (fast)
      quant_rowcol_kernel<true, false><<<grid, kRowColThreads, 0, s>>>(xi, M, K, ldx, cr, sr, cc, sc, sw, p);
    else
      quant_rowcol_kernel<false, false><<<grid, kRowColThreads, 0, s>>>(xi, M, K, ldx, cr, sr, cc, sc, sw, p);
  }
  return launch_status("quant_rowcol");
}

extern "C" mxb_status mxb_swizzle_scales(const void* scales, int64_t M, int64_t S, void* out,
                                         mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && S >= 0, MXB_ERR_INVALID_ARGUMENT, "swizzle_scales: negative size");
  if (M == 0 || S == 0) return MXB_OK;
  MXB_REQUIRE(scales && out, MXB_ERR_INVALID_ARGUMENT, "swizzle_scales: null pointer");
  const int64_t total = (M + 127) / 128 * 128 * ((S + 3) / 4 * 4);
  const int64_t want = cdiv(total, 256);
  const int grid = (int)(want < 148 * 16 ? want : 148 * 16);
  swizzle_scales_kernel<<<grid, 256, 0, to_cuda(stream)>>>((const uint8_t*)scales, M, S,
                                                           (uint8_t*)out);
  return launch_status("swizzle_scales");
}
