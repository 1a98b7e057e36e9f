// MXFP4 (rowwise) -> transposed FP8 E4M3 converts for sm_100a: the
// columnwise GEMM operands of the reference.
//
//  * col        (code/kernel/per_token_Mxfp4ToFp8_col.cu:110-301): scale per
//    (128-row block, 32-column block) from the largest E8M0 exponent; 8-bit
//    exponent re-basing with the sign bit masked off (table in fp8_lut.cuh).
//  * colT       (per_token_Mxfp4RowToBf16ToFp8Col.cu:42-197): true-amax scale
//    per (128-row block, column), amax/448 stored; race-free.
//  * colT-split (per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu:51-224): the same
//    per m_split segment with power-of-two scales (1/scale stored) and a
//    contiguous [N, m_i] output block per segment.
//
// Each CTA owns one 128-row x 64-code-byte tile.  One TMA load brings the
// codes into shared memory with the 64-byte swizzle, so that a warp whose
// lanes are 32 consecutive rows reads them without bank conflicts.  Results
// are transposed through shared memory and leave as 128-byte runs of output
// rows, eight lanes per run.  Several CTAs per SM overlap one tile's load
// with the others' work.
#include "capi_util.h"
#include "common.cuh"
#include "fp8_lut.cuh"
#include "tma.cuh"

namespace mxb {
namespace {

constexpr int kThreads = 256;
constexpr uint32_t kCodeTileBytes = 128 * 64;

__device__ const Fp8Lut g_lut_col = make_fp8_lut(true);

__device__ __forceinline__ uint32_t vmax_u8x4(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("vmax4.u32.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(0u));
  return r;
}

// 16-byte chunk c of row r of a 128 x 64-byte tile loaded with the TMA
// 64-byte swizzle (chunk index XOR bits 7..8 of the byte offset).
__device__ __forceinline__ uint4 ld_code_chunk(const uint8_t* tile, int r, int c) {
  return *reinterpret_cast<const uint4*>(tile + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// Loads the tile with one TMA and waits (bounded).  Returns false, for every
// thread of the CTA, if the copy never completed.
__device__ __forceinline__ bool load_code_tile(uint8_t* tile, uint64_t* bar, const CUtensorMap* map,
                                               int32_t x, int32_t y,
                                               uint32_t bytes = kCodeTileBytes) {
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(bar, bytes);
    tma_load_2d(tile, map, x, y, bar);
  }
  const bool ok = mbar_wait(bar, 0);
  return !__syncthreads_or(!ok);
}

// ------------------------------------------------------------------ col (C4)
// Tile: 128 rows x 128 code bytes (256 elements).  Rows are read as 128-byte
// runs (narrower runs at the row pitch of the code matrix cost DRAM bandwidth:
// 64-byte runs stream at ~4.1 TB/s, 128-byte runs at ~6.3 TB/s on B200).  One
// TMA box with the 128-byte swizzle lands the tile so that a warp whose lanes
// are 32 consecutive rows reads it without bank conflicts.  Lane = row: a lane
// maps 4 nibbles per `prmt` through its 32-column block's table row, then four
// neighbouring lanes transpose their 4x4 byte blocks with two shuffles so each
// lane stores four rows of one element as one word of the transposed tile,
// which leaves as 128-byte runs of output rows.
constexpr int kColPitch = 160;                 // bytes per element row of the transposed tile
constexpr uint32_t kColCodeBytes = 128 * 128;  // 16 KiB
constexpr size_t kColSmem = 1024 + kColCodeBytes + 256 * kColPitch + 4 * 8 + 16;

// 4x4 byte transpose across lanes 4m..4m+3: in, lane i holds row i's bytes for
// elements 0..3; out, lane i holds element i's bytes for rows 0..3.
__device__ __forceinline__ uint32_t transpose4x4(uint32_t w, uint32_t sel1, uint32_t sel2) {
  const uint32_t t = prmt(w, __shfl_xor_sync(0xffffffffu, w, 2), sel1);
  return prmt(t, __shfl_xor_sync(0xffffffffu, t, 1), sel2);
}

__global__ void __launch_bounds__(kThreads) fp8_col_kernel(const __grid_constant__ CUtensorMap tmap,
                                                           const uint8_t* __restrict__ scales,
                                                           int64_t M, int64_t Kb,
                                                           uint8_t* __restrict__ out,
                                                           float* __restrict__ scales_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ctile = smem;                                      // 128 x 128 B (128-byte swizzle)
  uint8_t* tr = smem + kColCodeBytes;                         // [element][row] FP8
  uint32_t* red = reinterpret_cast<uint32_t*>(tr + 256 * kColPitch);  // [4 row blocks][2 words]
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + 8);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int rb = warp >> 1, hh = warp & 1;  // 32-row block, 64-byte half of the tile
  const int64_t row0 = (int64_t)blockIdx.y * 128;
  const int64_t cb0 = (int64_t)blockIdx.x * 128;  // first code byte of the tile
  const int64_t S = Kb / 16;
  const int r = rb * 32 + lane;

  // this row's eight E8M0 bytes (one per 32-column block of the tile)
  const uint2 sc = ld_stream_v2(scales + (row0 + r) * S + cb0 / 16);
  if (hh == 0) {
    uint32_t m0 = sc.x, m1 = sc.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      m0 = vmax_u8x4(m0, __shfl_xor_sync(0xffffffffu, m0, o));
      m1 = vmax_u8x4(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    if (lane == 0) {
      red[rb * 2] = m0;
      red[rb * 2 + 1] = m1;
    }
  }
  if (!load_code_tile(ctile, bar, &tmap, (int32_t)cb0, (int32_t)row0, kColCodeBytes)) return;
  const uint32_t mx0 = vmax_u8x4(vmax_u8x4(red[0], red[2]), vmax_u8x4(red[4], red[6]));
  const uint32_t mx1 = vmax_u8x4(vmax_u8x4(red[1], red[3]), vmax_u8x4(red[5], red[7]));
  // lane-dependent byte selectors of the two transpose rounds
  const uint32_t sel1 = (lane & 2) ? 0x3276u : 0x5410u;
  const uint32_t sel2 = (lane & 1) ? 0x3715u : 0x6240u;
  // this lane stores element (4k + (lane & 3)) for rows (lane & ~3) .. +3
  uint8_t* trl = tr + (lane & 3) * kColPitch + rb * 32 + (lane & ~3);

#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int q = 4 * hh + cc;  // 32-column block (16 code bytes) of the tile
    const uint4 v = *reinterpret_cast<const uint4*>(ctile + r * 128 + ((q ^ (r & 7)) << 4));
    const uint32_t e = ((q < 4 ? sc.x : sc.y) >> (8 * (q & 3))) & 0xFFu;
    const uint32_t d = (((q < 4 ? mx0 : mx1) >> (8 * (q & 3))) & 0xFFu) - e;
    const uint2 tb = __ldg(reinterpret_cast<const uint2*>(g_lut_col.v[d]));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int hw = 0; hw < 2; ++hw) {
        const uint32_t f4 = lut_lookup4_nosign(w[j] >> (16 * hw), tb.x, tb.y);
        const int n = q * 32 + j * 8 + hw * 4;
        *reinterpret_cast<uint32_t*>(trl + n * kColPitch) = transpose4x4(f4, sel1, sel2);
      }
    }
  }
  __syncthreads();
  // scales: [M/128, 2*Kb], each block scale repeated over its 32 columns
  {
    const int q = t >> 5;
    const uint32_t wa = ((((q < 4 ? mx0 : mx1) >> (8 * (q & 3))) & 0xFFu) - 6u) & 0xFFu;
    scales_out[(row0 / 128) * (2 * Kb) + 2 * cb0 + t] = __uint_as_float(wa << 23);
  }
  // output rows n = 2*cb0 + 0..255: 128 FP8 bytes each at columns row0..row0+127
  uint8_t* ob = out + 2 * cb0 * M + row0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = k * kThreads + t;
    const int n = i >> 3, part = i & 7;
    const uint4 o = *reinterpret_cast<const uint4*>(&tr[n * kColPitch + part * 16]);
    st_stream_v4(ob + n * M + part * 16, o);
  }
}

// ------------------------------------------------------- colT / colT-split
// Tile: 128 rows x 128 elements.  Phase 1 decodes the tile to BF16 (code x
// E8M0 scale, exact) in shared memory, phase 2 finds each column's amax,
// phase 3 scales, clamps and converts column pairs to FP8 into a transposed
// staging tile (128-byte rows, 16-byte chunks XOR-swizzled by row / 2), and
// phase 4 writes that tile out as 128-byte row runs.
constexpr int kTPitch = 272;  // bytes per BF16 row in shared memory (256 + 16)

struct SplitArgs {
  const int32_t* m_splits;
  const int32_t* split_offsets;
  const int32_t* scale_offsets;
};

__device__ __forceinline__ int out_swz(int n, int chunk) { return n * 128 + ((chunk ^ ((n >> 1) & 7)) << 4); }

template <bool kSplit>
__global__ void __launch_bounds__(kThreads) fp8_colT_kernel(const __grid_constant__ CUtensorMap tmap,
                                                            const uint8_t* __restrict__ scales,
                                                            int64_t M, int64_t N, float eps,
                                                            uint8_t* __restrict__ out,
                                                            float* __restrict__ scales_out,
                                                            SplitArgs sa) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ctile = smem;                                // 8 KiB codes (64-byte swizzle)
  uint8_t* tile = smem + kCodeTileBytes;                // 128 x 272 B BF16
  uint8_t* otile = tile + 128 * kTPitch;                // 128 x 128 B FP8 (swizzled)
  uint32_t* part_max = reinterpret_cast<uint32_t*>(otile + 128 * 128);  // [4][128]
  float* col_qs = reinterpret_cast<float*>(part_max + 4 * 128);         // [128]
  uint32_t* col_clamp = reinterpret_cast<uint32_t*>(col_qs + 128);       // [128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(col_clamp + 128);
  int* has_special = reinterpret_cast<int*>(bar + 1);
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
  const int64_t S = N / 32;
  if (t == 0) *has_special = 0;

  // this thread's row (phase 1): lane = row within a 32-row block, warp pair = half
  const int rb = warp >> 1, hh = warp & 1, r = rb * 32 + lane;
  uint32_t sc = 0;
  if (r < rows) {
    const uint8_t* sp = scales + (row_start + r) * S + col0 / 32;
    if (cols == 128 && (reinterpret_cast<uintptr_t>(sp) & 3) == 0) {
      sc = ld_stream_u32(sp);  // the tile's four E8M0 bytes of this row at once
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (q * 32 < cols) sc |= (uint32_t)ld_stream_u8(sp + q) << (8 * q);
    }
  }
  if (!load_code_tile(ctile, bar, &tmap, (int32_t)(col0 / 2), (int32_t)row_start)) return;

  // ---- phase 1: decode two 32-element blocks of row r
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const int q = 2 * hh + cc;
    uint32_t o[16];
    if (r < rows && q * 32 < cols) {
      const uint4 c = ld_code_chunk(ctile, r, q);
      const uint32_t e = (sc >> (8 * q)) & 0xFFu;
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
        if (e == 255u) *has_special = 1;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = 0u;
    }
    uint4* dst = reinterpret_cast<uint4*>(tile + r * kTPitch + q * 64);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
  }
  __syncthreads();

  // ---- phase 2: column amax (thread = column pair x 32-row quarter)
  {
    const int cp = ((warp & 1) << 5) | lane, rq = warp >> 1;
    const uint32_t* col = reinterpret_cast<const uint32_t*>(tile + rq * 32 * kTPitch) + cp;
    if (*has_special == 0) {
      uint32_t w[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) w[i] = col[i * (kTPitch / 4)];
      const uint32_t m = absmax_tree<32>(w) & 0x7FFF7FFFu;
      part_max[rq * 128 + 2 * cp] = (m & 0xFFFFu) << 16;
      part_max[rq * 128 + 2 * cp + 1] = m & 0xFFFF0000u;
    } else {
      float a0 = 0.0f, a1 = 0.0f;  // fmaxf ignores NaN, as the reference's loop does
      for (int i = 0; i < 32; ++i) {
        const uint32_t w = col[i * (kTPitch / 4)];
        a0 = fmaxf(a0, fabsf(bf16lo_to_f(w)));
        a1 = fmaxf(a1, fabsf(bf16hi_to_f(w)));
      }
      part_max[rq * 128 + 2 * cp] = __float_as_uint(a0);
      part_max[rq * 128 + 2 * cp + 1] = __float_as_uint(a1);
    }
  }
  __syncthreads();
  if (t < 128) {
    // magnitudes are non-negative floats, so integer order is float order
    const uint32_t mb = max(max(part_max[t], part_max[128 + t]),
                            max(part_max[256 + t], part_max[384 + t]));
    const float mxv = __uint_as_float(mb);
    float qs;
    if (!kSplit) {
      const float amax = fmaxf(eps, mxv);
      if (t < cols) scales_out[scale_row * N + col0 + t] = amax / 448.0f;
      qs = (amax > 1e-9f) ? (448.0f / amax) : 0.0f;
    } else {
      const float amax = mxv;  // initialised to 0 on the split path
      float s;
      if (amax <= eps) {
        s = 1.0f;
      } else {
        const uint32_t rbits = __float_as_uint(amax / 448.0f);
        uint32_t ex = (rbits >> 23) & 0xFFu;
        if (rbits & 0x7FFFFFu) ex += 1u;
        s = (float)(1.0 / (double)__uint_as_float(ex << 23));
      }
      if (t < cols) scales_out[scale_row * N + col0 + t] = 1.0f / s;
      qs = s;
    }
    col_qs[t] = qs;
    // NaN products are possible only with an Inf amax or an E8M0 byte of 255
    col_clamp[t] = (mb >= 0x7F800000u || *has_special) ? 1u : 0u;
  }
  __syncthreads();

  // ---- phase 3: column pair x 16-row chunk -> two 16-byte runs of the staging tile.
  // With a finite amax every |v * qs| is at most 448 (1 + 2^-23), which the
  // saturating conversion maps exactly as clamp-then-convert does (true for
  // every finite value), so the clamp is applied only where a NaN can occur:
  // columns with an Inf amax (v * 0) and tiles holding an E8M0 byte of 255
  // (0 * Inf); the reference clamps NaN to -448.
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int cp = ((warp & 1) << 5) | lane;
    const int chunk = (warp >> 1) + 4 * k;  // 0..7
    const uint32_t* col = reinterpret_cast<const uint32_t*>(tile + chunk * 16 * kTPitch) + cp;
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = col[i * (kTPitch / 4)];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float qs = col_qs[2 * cp + h];
      const bool clamp = col_clamp[2 * cp + h] != 0;
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t word = 0;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint32_t b0 = w[4 * j + 2 * u], b1 = w[4 * j + 2 * u + 1];
          float q0, q1;
          mul2_f32(h ? (b0 & 0xFFFF0000u) : (b0 << 16), h ? (b1 & 0xFFFF0000u) : (b1 << 16), qs,
                   q0, q1);
          if (clamp) {
            q0 = fminf(fmaxf(q0, -448.0f), 448.0f);
            q1 = fminf(fmaxf(q1, -448.0f), 448.0f);
          }
          word |= cvt_e4m3x2(q0, q1) << (16 * u);
        }
        o[j] = word;
      }
      *reinterpret_cast<uint4*>(otile + out_swz(2 * cp + h, chunk)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();

  // ---- phase 4: output rows n (128 FP8 bytes each), eight lanes per row
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = k * kThreads + t;
    const int n = i >> 3, part = i & 7;
    if (n >= cols || part * 16 >= rows) continue;
    const uint4 o = *reinterpret_cast<const uint4*>(otile + out_swz(n, part));
    uint8_t* dst = out + out_base + (col0 + n) * out_pitch + part * 16;
    const int valid = (int)min((int64_t)16, rows - part * 16);
    if (valid == 16 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
      st_stream_v4(dst, o);
    } else {
      const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
      for (int j = 0; j < valid; ++j) dst[j] = (uint8_t)(ow[j >> 2] >> (8 * (j & 3)));
    }
  }
}

constexpr size_t kColTSmem = 1024 + kCodeTileBytes + 128 * kTPitch + 128 * 128 + 4 * 128 * 4 +
                             2 * 128 * 4 + 16;

bool colT_attr() {
  static const bool ok =
      cudaFuncSetAttribute((const void*)fp8_colT_kernel<false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kColTSmem) ==
          cudaSuccess &&
      cudaFuncSetAttribute((const void*)fp8_colT_kernel<true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kColTSmem) ==
          cudaSuccess;
  return ok;
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
  MXB_REQUIRE(aligned(input, 16) && aligned(input_s, 8) && aligned(output_q, 16),
              MXB_ERR_MISALIGNED, "mxfp4_to_fp8_col: misaligned pointer");
  CUtensorMap tmap;
  if (!make_tensor_map_2d(&tmap, input, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, Kb, Kb, 128, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return MXB_ERR_CUDA;
  static const bool attr_ok =
      cudaFuncSetAttribute((const void*)fp8_col_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kColSmem) == cudaSuccess;
  MXB_REQUIRE(attr_ok, MXB_ERR_CUDA, "mxfp4_to_fp8_col: cannot reserve shared memory");
  const dim3 grid((unsigned)(Kb / 128), (unsigned)(M / 128));
  fp8_col_kernel<<<grid, kThreads, kColSmem, to_cuda(stream)>>>(tmap, (const uint8_t*)input_s, M,
                                                                Kb, (uint8_t*)output_q,
                                                                (float*)output_s);
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
  MXB_REQUIRE(colT_attr(), MXB_ERR_CUDA, "mxfp4_to_fp8_colT: cannot reserve shared memory");
  CUtensorMap tmap;
  if (!make_tensor_map_2d(&tmap, input, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, N / 2, N / 2, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_64B))
    return MXB_ERR_CUDA;
  const dim3 grid((unsigned)cdiv(M, 128), 1, (unsigned)cdiv(N, 128));
  fp8_colT_kernel<false><<<grid, kThreads, kColTSmem, to_cuda(stream)>>>(
      tmap, (const uint8_t*)input_s, M, N, eps, (uint8_t*)output_q, (float*)output_s,
      SplitArgs{nullptr, nullptr, nullptr});
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
  MXB_REQUIRE(colT_attr(), MXB_ERR_CUDA, "mxfp4_to_fp8_colT_msplit: cannot reserve shared memory");
  CUtensorMap tmap;
  if (!make_tensor_map_2d(&tmap, input, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, total_M, N / 2, N / 2,
                          64, 128, CU_TENSOR_MAP_SWIZZLE_64B))
    return MXB_ERR_CUDA;
  const dim3 grid((unsigned)num_splits, (unsigned)cdiv(max_split_len, 128), (unsigned)cdiv(N, 128));
  fp8_colT_kernel<true><<<grid, kThreads, kColTSmem, to_cuda(stream)>>>(
      tmap, (const uint8_t*)input_s, total_M, N, eps, (uint8_t*)output_q, (float*)output_s,
      SplitArgs{m_splits, split_offsets, scale_offsets});
  return launch_status("mxfp4_to_fp8_colT_msplit");
}
