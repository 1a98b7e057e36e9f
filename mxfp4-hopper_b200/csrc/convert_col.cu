// MXFP4 (rowwise) -> transposed FP8 E4M3 converts for sm_100a: the
// columnwise GEMM operands of the reference.
//
//  * col      (code/kernel/per_token_Mxfp4ToFp8_col.cu:110-301): scale per
//    (128-row block, 32-column block) from the largest E8M0 exponent; 8-bit
//    exponent re-basing with the sign bit masked off.
//  * colT     (per_token_Mxfp4RowToBf16ToFp8Col.cu:42-197): true-amax scale
//    per (128-row block, column), amax/448 stored.
//  * colT-split (per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu:51-224): the same
//    per m_split segment with power-of-two scales (1/scale stored) and a
//    contiguous [N, m_i] output block per segment.
//
// All three read a 128-row tile of codes once with 16-byte loads, transpose
// through shared memory and write whole 16-byte runs of the [N, M] output.
#include "capi_util.h"
#include "common.cuh"

namespace mxb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t vmax_u8x4(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("vmax4.u32.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(0u));
  return r;
}

// ------------------------------------------------------------------ col (C4)
// Tile: 128 rows x 64 code bytes (128 elements, four 32-column scale blocks).
constexpr int kColPitch = 144;  // bytes per transposed row in shared memory

__global__ void __launch_bounds__(kThreads) fp8_col_kernel(const uint8_t* __restrict__ codes,
                                                           const uint8_t* __restrict__ scales,
                                                           int64_t M, int64_t Kb,
                                                           uint8_t* __restrict__ out,
                                                           float* __restrict__ scales_out) {
  __shared__ __align__(16) uint8_t tr[128 * kColPitch];  // [element][row] FP8
  __shared__ uint32_t sc_row[128];                        // 4 E8M0 bytes per row
  __shared__ uint32_t red[4];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t row0 = (int64_t)blockIdx.y * 128;
  const int64_t cb0 = (int64_t)blockIdx.x * 64;  // first code byte of the tile
  const int64_t S = Kb / 16;

  if (t < 128) {
    const uint32_t s = ld_stream_u32(scales + (row0 + t) * S + cb0 / 16);
    sc_row[t] = s;
    uint32_t m = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = vmax_u8x4(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
  }
  // codes: 512 chunks of 16 bytes; chunk i -> (scale column q = i / 128, row i % 128)
  uint4 v[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = k * kThreads + t;
    v[k] = ld_stream_v4(codes + (row0 + (i & 127)) * Kb + cb0 + (i >> 7) * 16);
  }
  __syncthreads();
  const uint32_t mx = vmax_u8x4(vmax_u8x4(red[0], red[1]), vmax_u8x4(red[2], red[3]));
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = k * kThreads + t;
    const int r = i & 127, q = i >> 7;
    const uint32_t wa = ((mx >> (8 * q)) - 6u) & 0xFFu;
    const uint32_t e = (sc_row[r] >> (8 * q)) & 0xFFu;
    const uint32_t adj = (wa - e) & 0xFFu;
    const uint32_t off16 = (adj << 7) << 16;
    const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t x[4];
      e2m1x4_to_bf16x4(w[j], x[0], x[1]);
      e2m1x4_to_bf16x4(w[j] >> 16, x[2], x[3]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float lo = __uint_as_float(((x[u] << 16) - off16) & 0x7FFF0000u);
        float hi = __uint_as_float(((x[u] & 0xFFFF0000u) - off16) & 0x7FFF0000u);
        lo = fminf(fmaxf(lo, -448.0f), 448.0f);
        hi = fminf(fmaxf(hi, -448.0f), 448.0f);
        const uint32_t b2 = cvt_e4m3x2(lo, hi);
        const int n = q * 32 + j * 8 + u * 2;
        tr[n * kColPitch + r] = (uint8_t)b2;
        tr[(n + 1) * kColPitch + r] = (uint8_t)(b2 >> 8);
      }
    }
  }
  __syncthreads();
  // scales: [M/128, 2*Kb], each block scale repeated over its 32 columns
  if (t < 128) {
    const uint32_t wa = ((mx >> (8 * (t >> 5))) - 6u) & 0xFFu;
    scales_out[(row0 / 128) * (2 * Kb) + 2 * cb0 + t] = __uint_as_float(wa << 23);
  }
  // output rows n = 2*cb0 + 0..127, 128 FP8 bytes each at columns row0..row0+127
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = k * kThreads + t;
    const int n = i >> 3, part = i & 7;
    const uint4 o = *reinterpret_cast<const uint4*>(&tr[n * kColPitch + part * 16]);
    st_stream_v4(out + (2 * cb0 + n) * M + row0 + part * 16, o);
  }
}

// ------------------------------------------------------- colT / colT-split
// Tile: 128 rows x 128 elements (64 code bytes per row).  Phase 1 decodes the
// tile to BF16 (code x E8M0 scale; exact) in shared memory, phase 2 finds each
// column's amax, phase 3 scales, clamps and converts columns to FP8.
constexpr int kTPitch = 272;  // bytes per BF16 row in shared memory (256 + 16)

struct SplitArgs {
  const int32_t* m_splits;
  const int32_t* split_offsets;
  const int32_t* scale_offsets;
};

template <bool kSplit>
__global__ void __launch_bounds__(kThreads) fp8_colT_kernel(const uint8_t* __restrict__ codes,
                                                            const uint8_t* __restrict__ scales,
                                                            int64_t M, int64_t N, float eps,
                                                            uint8_t* __restrict__ out,
                                                            float* __restrict__ scales_out,
                                                            SplitArgs sa) {
  __shared__ __align__(16) uint8_t tile[128 * kTPitch];
  __shared__ uint32_t part_max[4][128];
  __shared__ float col_qs[128];
  __shared__ int has_special;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

  // tile geometry
  int64_t row_start, rows, out_base, out_pitch, scale_row;
  if (kSplit) {
    const int s = blockIdx.x;
    const int64_t mi = sa.m_splits[s];
    const int64_t b = blockIdx.y;
    if (b * 128 >= mi) return;
    const int64_t o = sa.split_offsets[s];
    row_start = o + b * 128;
    rows = min((int64_t)128, mi - b * 128);
    out_base = o * N + b * 128;  // + n * mi + local row
    out_pitch = mi;
    scale_row = sa.scale_offsets[s] + b;
  } else {
    row_start = (int64_t)blockIdx.x * 128;
    rows = min((int64_t)128, M - row_start);
    out_base = row_start;
    out_pitch = M;
    scale_row = blockIdx.x;
  }
  const int64_t col0 = (int64_t)blockIdx.z * 128;
  const int64_t cols = min((int64_t)128, N - col0);
  const int64_t Kb = N / 2, S = N / 32;
  if (t == 0) has_special = 0;
  __syncthreads();

  // ---- phase 1: decode (row r, 32-element block q) per chunk
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = k * kThreads + t;
    const int r = i & 127, q = i >> 7;
    uint32_t o[16];
    if (r < rows && q * 32 < cols) {
      const int64_t gr = row_start + r;
      const uint4 c = ld_stream_v4(codes + gr * Kb + col0 / 2 + q * 16);
      const uint32_t e = ld_stream_u8(scales + gr * S + col0 / 32 + q);
      const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        e2m1x4_to_bf16x4(w[j], o[4 * j], o[4 * j + 1]);
        e2m1x4_to_bf16x4(w[j] >> 16, o[4 * j + 2], o[4 * j + 3]);
      }
      if (e - 2u <= 252u) {
        const uint32_t s2 = (e << 7) | (e << 23);
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = mul_bf16x2(o[j], s2);
      } else {
        // zero / subnormal / Inf scales: float product, exact or Inf/NaN
        const float s = e8m0_to_f(e);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          o[j] = cvt_bf16x2(bf16lo_to_f(o[j]) * s, bf16hi_to_f(o[j]) * s);
        if (e == 255u) has_special = 1;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = 0u;
    }
    uint4* dst = reinterpret_cast<uint4*>(&tile[r * kTPitch + q * 64]);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
  }
  __syncthreads();

  // ---- phase 2: column amax (thread = column pair x 32-row quarter)
  {
    const int cp = ((warp & 1) << 5) | lane, rq = warp >> 1;
    const bool special = has_special != 0;
    if (!special) {
      uint32_t m = 0;
#pragma unroll 8
      for (int i = 0; i < 32; ++i)
        m = vmax_u16x2(m, *reinterpret_cast<const uint32_t*>(&tile[(rq * 32 + i) * kTPitch + cp * 4]) &
                              0x7FFF7FFFu);
      part_max[rq][2 * cp] = (m & 0xFFFFu) << 16;
      part_max[rq][2 * cp + 1] = m & 0xFFFF0000u;
    } else {
      float a0 = 0.0f, a1 = 0.0f;  // fmaxf ignores NaN, as the reference's loop does
      for (int i = 0; i < 32; ++i) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(&tile[(rq * 32 + i) * kTPitch + cp * 4]);
        a0 = fmaxf(a0, fabsf(bf16lo_to_f(w)));
        a1 = fmaxf(a1, fabsf(bf16hi_to_f(w)));
      }
      part_max[rq][2 * cp] = __float_as_uint(a0);
      part_max[rq][2 * cp + 1] = __float_as_uint(a1);
    }
  }
  __syncthreads();
  if (t < 128) {
    // magnitudes are non-negative floats, so integer order is float order
    const uint32_t mb = max(max(part_max[0][t], part_max[1][t]), max(part_max[2][t], part_max[3][t]));
    const float mxv = __uint_as_float(mb);
    float qs;
    if (!kSplit) {
      const float amax = fmaxf(eps, mxv);
      if (t < cols) scales_out[scale_row * N + col0 + t] = amax / 448.0f;
      qs = (amax > 1e-9f) ? (448.0f / amax) : 0.0f;
    } else {
      const float amax = mxv;  // initialised to 0 on the split path
      float sc;
      if (amax <= eps) {
        sc = 1.0f;
      } else {
        const uint32_t rb = __float_as_uint(amax / 448.0f);
        uint32_t ex = (rb >> 23) & 0xFFu;
        if (rb & 0x7FFFFFu) ex += 1u;
        sc = (float)(1.0 / (double)__uint_as_float(ex << 23));
      }
      if (t < cols) scales_out[scale_row * N + col0 + t] = 1.0f / sc;
      qs = sc;
    }
    col_qs[t] = qs;
  }
  __syncthreads();

  // ---- phase 3: quantize columns; lane -> column, 16-row chunk per task
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int n = ((warp & 3) << 5) | lane;
    const int chunk = (warp >> 2) + 2 * k;  // 0..7
    if (n >= cols || chunk * 16 >= rows) continue;
    const float qs = col_qs[n];
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t word = 0;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = chunk * 16 + j * 4 + u * 2;
        const uint32_t b0 = *reinterpret_cast<const uint16_t*>(&tile[r * kTPitch + n * 2]);
        const uint32_t b1 = *reinterpret_cast<const uint16_t*>(&tile[(r + 1) * kTPitch + n * 2]);
        float q0 = __uint_as_float(b0 << 16) * qs;
        float q1 = __uint_as_float(b1 << 16) * qs;
        q0 = fminf(fmaxf(q0, -448.0f), 448.0f);
        q1 = fminf(fmaxf(q1, -448.0f), 448.0f);
        word |= cvt_e4m3x2(q0, q1) << (16 * u);
      }
      o[j] = word;
    }
    uint8_t* dst = out + out_base + (col0 + n) * out_pitch + chunk * 16;
    const int valid = (int)min((int64_t)16, rows - chunk * 16);
    if (valid == 16 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
      st_stream_v4(dst, make_uint4(o[0], o[1], o[2], o[3]));
    } else {
      for (int j = 0; j < valid; ++j) dst[j] = (uint8_t)(o[j >> 2] >> (8 * (j & 3)));
    }
  }
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_per_token_Mxfp4ToFp8_col(const void* input, const void* input_s,
                                                   int64_t M, int64_t Kb, void* output_q,
                                                   void* output_s, mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && Kb >= 0 && M % 128 == 0 && Kb % 128 == 0, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_col: need M %% 128 == 0 and Kb %% 128 == 0 (the reference tiles "
              "without bounds checks), got M=%lld Kb=%lld",
              (long long)M, (long long)Kb);
  if (M == 0 || Kb == 0) return MXB_OK;
  MXB_REQUIRE(input && input_s && output_q && output_s, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_col: null pointer");
  MXB_REQUIRE(aligned(input, 16) && aligned(input_s, 4) && aligned(output_q, 16),
              MXB_ERR_MISALIGNED, "mxfp4_to_fp8_col: misaligned pointer");
  const dim3 grid((unsigned)(Kb / 64), (unsigned)(M / 128));
  fp8_col_kernel<<<grid, kThreads, 0, to_cuda(stream)>>>((const uint8_t*)input,
                                                         (const uint8_t*)input_s, M, Kb,
                                                         (uint8_t*)output_q, (float*)output_s);
  return launch_status("mxfp4_to_fp8_col");
}

extern "C" mxb_status mxb_per_token_Mxfp4RowToBf16ToFp8Col(const void* input, const void* input_s,
                                                           int64_t M, int64_t N, void* output_q,
                                                           void* output_s, float eps,
                                                           mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && N >= 0 && N % 32 == 0, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT: need N %% 32 == 0, got %lld", (long long)N);
  if (M == 0 || N == 0) return MXB_OK;
  MXB_REQUIRE(input && input_s && output_q && output_s, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT: null pointer");
  MXB_REQUIRE(aligned(input, 16), MXB_ERR_MISALIGNED, "mxfp4_to_fp8_colT: input not 16-byte aligned");
  const dim3 grid((unsigned)cdiv(M, 128), 1, (unsigned)cdiv(N, 128));
  fp8_colT_kernel<false><<<grid, kThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)input, (const uint8_t*)input_s, M, N, eps, (uint8_t*)output_q,
      (float*)output_s, SplitArgs{nullptr, nullptr, nullptr});
  return launch_status("mxfp4_to_fp8_colT");
}

extern "C" mxb_status mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit(
    const void* input, const void* input_s, int64_t total_M, int64_t N, void* output_q,
    void* output_s, const int32_t* m_splits, const int32_t* split_offsets,
    const int32_t* scale_offsets, int64_t num_splits, int64_t max_split_len, float eps,
    mxb_stream_t stream) {
  MXB_REQUIRE(total_M >= 0 && N >= 0 && N % 32 == 0 && num_splits >= 0 && max_split_len >= 0,
              MXB_ERR_INVALID_ARGUMENT, "mxfp4_to_fp8_colT_msplit: need N %% 32 == 0, got %lld",
              (long long)N);
  MXB_REQUIRE(num_splits <= 65535 && cdiv(max_split_len, 128) <= 65535, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT_msplit: too many splits or rows per split");
  if (total_M == 0 || N == 0 || num_splits == 0 || max_split_len == 0) return MXB_OK;
  MXB_REQUIRE(input && input_s && output_q && output_s && m_splits && split_offsets &&
                  scale_offsets,
              MXB_ERR_INVALID_ARGUMENT, "mxfp4_to_fp8_colT_msplit: null pointer");
  MXB_REQUIRE(aligned(input, 16), MXB_ERR_MISALIGNED,
              "mxfp4_to_fp8_colT_msplit: input not 16-byte aligned");
  const dim3 grid((unsigned)num_splits, (unsigned)cdiv(max_split_len, 128), (unsigned)cdiv(N, 128));
  fp8_colT_kernel<true><<<grid, kThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)input, (const uint8_t*)input_s, total_M, N, eps, (uint8_t*)output_q,
      (float*)output_s, SplitArgs{m_splits, split_offsets, scale_offsets});
  return launch_status("mxfp4_to_fp8_colT_msplit");
}
