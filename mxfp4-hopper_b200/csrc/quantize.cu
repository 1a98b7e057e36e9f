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
// Fast path (fp4_max = 6, fp4_min = -6, 0 <= eps <= 6e-10: the reference API's
// only configuration).  For a finite BF16 amax = 1.m * 2^e the exponent of
// y_s is exactly
//     k = max(e - 2 + [1.m > 1.5], -33)
// because amax/6 = (1.m / 1.5) * 2^(e-2) and 1.m / 1.5 lies in [2/3, 4/3): it
// is a power of two only at 1.m = 1.5 and otherwise at least 0.5% away from
// one, so neither the rounding of the division nor log2f can move the ceiling;
// -33 = ceil(log2(1e-10)) is the clamp, and eps <= 6e-10 never raises amax/6
// above it.  The block amax is an integer max over BF16 magnitude patterns,
// x * 2^-k is one fma.rn.f32.bf16 per value (see encode8_pairs), and the codes come from
// Blackwell's cvt.rn.satfinite.e2m1x2.f32, whose round-to-nearest-even with
// the sign kept on zero equals the reference's integer rounding for every
// such product (both are checked exhaustively against the reference kernel).
// Blocks holding Inf/NaN, and every block when the parameters differ from the
// defaults, take the generic path, which evaluates the reference formula
// literally and encodes with the reference's integer rounding.
#include <cuda_bf16.h>

#include "capi_util.h"
#include "common.cuh"
#include "fp8_lut.cuh"
#include "qrow.cuh"
#include "tma.cuh"

namespace mxb {
namespace {

__device__ __forceinline__ int64_t swizzle_offset(int64_t r, int64_t c, int64_t sp4) {
  return ((r >> 7) * sp4 + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3);
}

// ------------------------------------------------------------------ Q-row
// Two lanes per 32-element block, 16 elements (two 16-byte loads) per lane.
// A warp covers 16 consecutive blocks: 1 KiB of contiguous input per step.
//
// With kFp8 the same pass also writes the rowwise FP8 conversion of the codes
// it has just produced (the reference op omo_per_token_group_quant_fp4_fused_ToFp8,
// bound at code/kernel/ops.cu:34 with no source shipped), bit-identical to
// running the rowwise FP8 converter (per_token_Mxfp4ToFp8.cu:157-233) on this
// kernel's output: a lane's 8 code bytes are exactly one lane of that
// converter, the 8 lanes of a 1x128 group are adjacent in the warp (K % 128 ==
// 0), so the group max of the four E8M0 bytes is two shuffles, and each lane
// maps its nibbles through the table row for d = max - e (fp8_lut.cuh).  The
// codes are never re-read from HBM.
__device__ const Fp8Lut g_lut_fused = make_fp8_lut(false);

template <bool kFast, bool kFp8, bool kOcp = false>
__global__ void __launch_bounds__(256) quant_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                         int64_t M, int64_t K, int64_t ldx,
                                                         uint8_t* __restrict__ codes,
                                                         uint8_t* __restrict__ scales,
                                                         QuantParams p, uint8_t* __restrict__ fp8,
                                                         float* __restrict__ fp8_s) {
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
    uint32_t mb = max_abs_pairs(w);
    mb = max(mb, __shfl_xor_sync(pair_mask, mb, 1));
    uint32_t byte, out[2];
    if (kFast && mb < 0x7F80u) {
      uint32_t inv;
      scale_fast_rule<kOcp>(mb, byte, inv);
      out[0] = encode8_pairs(&w[0], inv);
      out[1] = encode8_pairs(&w[4], inv);
    } else {
      uint32_t f0[8], f1[8];
      unpack8(&w[0], f0);
      unpack8(&w[4], f1);
      float am = fmaxf(amax_generic(f0, p.eps), amax_generic(f1, p.eps));
      am = fmaxf(am, __shfl_xor_sync(pair_mask, am, 1));
      float inv;
      scale_generic_rule<kOcp>(am, p, inv, byte);
      out[0] = encode8_generic(f0, inv, p);
      out[1] = encode8_generic(f1, inv, p);
    }
    st_stream_v2(codes + r * (K >> 1) + g * 16 + half * 8, make_uint2(out[0], out[1]));
    if (half == 0) scales[r * G + g] = (uint8_t)byte;
    if (kFp8) {
      const unsigned group_mask = 0xFFu << (lane & ~7);
      uint32_t mx = max(byte, __shfl_xor_sync(group_mask, byte, 2));
      mx = max(mx, __shfl_xor_sync(group_mask, mx, 4));
      const uint4 t = __ldg(reinterpret_cast<const uint4*>(g_lut_fused.v[mx - byte]));
      const uint4 o = make_uint4(lut_lookup4(out[0], t.x, t.y, t.z, t.w),
                                 lut_lookup4(out[0] >> 16, t.x, t.y, t.z, t.w),
                                 lut_lookup4(out[1], t.x, t.y, t.z, t.w),
                                 lut_lookup4(out[1] >> 16, t.x, t.y, t.z, t.w));
      st_stream_v4(fp8 + r * K + g * 32 + half * 16, o);
      if ((h & 7) == 0) fp8_s[(g >> 2) * M + r] = __uint_as_float(((mx - 6u) & 0xFFu) << 23);
    }
  }
}

// ------------------------------------------------------- fused Q-row + Q-col
// Persistent, warp-specialised kernel, two CTAs per SM.  Each CTA walks
// 128x128 BF16 tiles (tile = blockIdx.x + i * gridDim.x):
//   * a producer warp streams tiles into a ring of kStages shared-memory
//     buffers with TMA (one 32 KiB cp.async.bulk.tensor per tile, completion on
//     full[s]); eight consumer warps release a buffer on empty[s];
//   * row pass: a thread quantizes two 1x32 row blocks (64 contiguous bytes);
//     col pass: a thread quantizes a column pair over one 32-row block;
//   * both passes write their codes into a double-buffered shared-memory
//     staging area (two 128 x 64-byte boxes, 64-byte TMA swizzle) and their
//     E8M0 bytes into 128 x 4-byte scale boxes; after one consumer barrier a
//     single thread writes the two code boxes with TMA stores and every
//     consumer thread writes one 4-byte scale word.
// Staging keeps the SM's load/store unit out of the transpose: written
// directly, the column pass would issue 16-byte stores to 32 rows 8 KiB apart
// and single-byte scale stores, which bound the kernel well below HBM speed.
// The input tile is stored densely (256-byte rows); the row pass rotates the
// order in which a thread reads its four 16-byte chunks by (row % 4) so that
// the eight lanes of each shared-memory phase hit eight different bank groups.
// HBM sees every input byte once and every output byte once.
constexpr int kTile = 128;
constexpr int kStages = 2;
constexpr uint32_t kTileBytes = kTile * kTile * 2;  // 32 KiB of BF16
constexpr uint32_t kCodeBox = kTile * 64;           // 8 KiB: 128 rows x 64 code bytes
constexpr uint32_t kScaleBox = kTile * 4;           // 128 rows x 4 scale bytes
constexpr uint32_t kStageOut = 2 * kCodeBox + 2 * kScaleBox;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kRowColThreads = kConsumers + 32;
constexpr size_t kRowColSmem = kStages * kTileBytes + 2 * kStageOut + 2 * kStages * 8 + 1024;

// Rotates four words right by r (o[(j + r) & 3] = in[j]) without local memory.
__device__ __forceinline__ void rotate4(uint32_t (&o)[4], uint32_t r) {
  uint32_t a[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) a[j] = (r & 1) ? o[(j + 3) & 3] : o[j];
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = (r & 2) ? a[(j + 2) & 3] : a[j];
}

// Byte offset of 16-byte chunk `c` of row `r` in a 128 x 64-byte box laid out
// with the TMA 64-byte swizzle (chunk index XOR bits 7..8 of the offset).
__device__ __forceinline__ uint32_t sw64(uint32_t r, uint32_t c) {
  return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
}

template <bool kFast, bool kRows, bool kOcp = false>
__global__ void __launch_bounds__(kRowColThreads, 2) quant_rowcol_kernel(
    const __grid_constant__ CUtensorMap tmap_in, const __grid_constant__ CUtensorMap tmap_row,
    const __grid_constant__ CUtensorMap tmap_col, int64_t M, int64_t K,
    uint8_t* __restrict__ scales_row, uint8_t* __restrict__ scales_col,
    uint8_t* __restrict__ scales_swz, QuantParams p, int col_tiles, int tiles) {
  extern __shared__ uint8_t smem_raw[];
  // 1 KiB alignment for the swizzled staging boxes
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* out_base = smem + kStages * kTileBytes;  // 2 x kStageOut
  uint64_t* full = reinterpret_cast<uint64_t*>(out_base + 2 * kStageOut);
  uint64_t* empty = full + kStages;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int my_tiles =
      (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int64_t G = K >> 5, Gc = M >> 5, sp4 = (G + 3) >> 2;

  if (t == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------ producer warp
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&empty[s], (uint32_t)(i / kStages - 1) & 1u)) break;
        fence_proxy_async_smem();
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        const int rt = tile / col_tiles, ct = tile - rt * col_tiles;
        mbar_arrive_expect_tx(&full[s], kTileBytes);
        tma_load_2d(smem + s * kTileBytes, &tmap_in, ct * kTile, rt * kTile, &full[s]);
        issued = i + 1;
      }
      // do not leave while copies of this CTA are still landing
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
        mbar_wait(&full[i % kStages], (uint32_t)(i / kStages) & 1u);
    }
    return;
  }

  // -------------------------------------------------- consumer warps
  bool alive = true;
  for (int i = 0; i < my_tiles; ++i) {
    const int s = i % kStages;
    alive = alive && mbar_wait(&full[s], (uint32_t)(i / kStages) & 1u);
    const uint8_t* ts = smem + s * kTileBytes;
    uint8_t* ob = out_base + (i & 1) * kStageOut;
    uint8_t* o_row = ob;                       // row codes box   [128 rows][64 B]
    uint8_t* o_col = ob + kCodeBox;            // col codes box   [128 cols][64 B]
    uint8_t* s_row = ob + 2 * kCodeBox;        // row scales      [128 rows][4]
    uint8_t* s_col = s_row + kScaleBox;        // col scales      [128 cols][4]
    const int tile = (int)blockIdx.x + i * (int)gridDim.x;
    const int rt = tile / col_tiles, ct = tile - rt * col_tiles;
    const int64_t row0 = (int64_t)rt * kTile, col0 = (int64_t)ct * kTile;

    if (kRows && alive) {
      const uint32_t rsub = lane & 3, gsel = (lane >> 2) & 1, rhi = lane >> 3;
      const int r = warp * 16 + (int)(rhi * 4 + rsub);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int g = 2 * k + (int)gsel;
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t c = (j + rsub) & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(ts + r * 256 + g * 64 + c * 16);
          w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
        }
        uint32_t out[4], byte;
        quant_block32<kFast, kOcp>(w, p, out, byte);  // out[j] encodes chunk (j + rsub) & 3
        rotate4(out, rsub);
        *reinterpret_cast<uint4*>(o_row + sw64(r, g)) = make_uint4(out[0], out[1], out[2], out[3]);
        s_row[r * 4 + g] = (uint8_t)byte;
        if (scales_swz) {
          const int64_t gr = row0 + r, gg = (col0 >> 5) + g;
          if (gr < M && gg < G) scales_swz[swizzle_offset(gr, gg, sp4)] = (uint8_t)byte;
        }
      }
    }

    if (alive) {
      const int cp = ((warp & 1) << 5) | lane;  // column pair within the tile
      const int rb = warp >> 1;                 // 32-row block within the tile
      uint32_t w[32];  // rows rb*32 .. +31, columns (2cp, 2cp + 1) as BF16 pairs
#pragma unroll
      for (int r = 0; r < 32; ++r)
        w[r] = *reinterpret_cast<const uint32_t*>(ts + (rb * 32 + r) * 256 + cp * 4);
      const uint32_t m = absmax_tree<32>(w) & 0x7FFF7FFFu;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t mb = h ? (m >> 16) : (m & 0xFFFFu);
        uint32_t out[4], byte;
        if (kFast && mb < 0x7F80u) {
          uint32_t inv;
          scale_fast_rule<kOcp>(mb, byte, inv);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            out[q] = h ? encode8_half<true>(&w[8 * q], inv) : encode8_half<false>(&w[8 * q], inv);
        } else {
          uint32_t fa[32];
#pragma unroll
          for (int r = 0; r < 32; ++r) fa[r] = h ? (w[r] & 0xFFFF0000u) : (w[r] << 16);
          float inv;
          scale_generic_rule<kOcp>(amax_generic(fa, p.eps), p, inv, byte);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t f[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = fa[8 * q + j];
            out[q] = encode8_generic(f, inv, p);
          }
        }
        const int c = 2 * cp + h;
        *reinterpret_cast<uint4*>(o_col + sw64(c, rb)) = make_uint4(out[0], out[1], out[2], out[3]);
        s_col[c * 4 + rb] = (uint8_t)byte;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with input stage s
    fence_proxy_async_smem();               // staging writes -> visible to the TMA store
    if (t == 0) bulk_wait_read_all();       // the previous tile's stores have read their box
    if (named_sync_or(1, kConsumers, !alive)) break;  // a tile never arrived: stop together
    if (t == 0) {
      if (kRows) tma_store_2d(&tmap_row, (int32_t)(col0 >> 1), (int32_t)row0, o_row);
      tma_store_2d(&tmap_col, (int32_t)(row0 >> 1), (int32_t)col0, o_col);
      bulk_commit();
    }
    // scale words: thread t < 128 -> row scales of row t; t >= 128 -> col scales of column t-128
    {
      const bool is_row = t < kTile;
      if (is_row && !kRows) continue;
      const int idx = is_row ? t : t - kTile;
      const int64_t lim_outer = is_row ? M : K, lim_inner = is_row ? G : Gc;
      const int64_t outer = (is_row ? row0 : col0) + idx;
      const int64_t inner0 = (is_row ? col0 : row0) >> 5;
      uint8_t* dst_base = is_row ? scales_row : scales_col;
      const uint32_t word = *reinterpret_cast<const uint32_t*>((is_row ? s_row : s_col) + idx * 4);
      if (outer < lim_outer) {
        uint8_t* dst = dst_base + outer * lim_inner + inner0;
        const int64_t n = min((int64_t)4, lim_inner - inner0);
        if (n == 4 && (reinterpret_cast<uintptr_t>(dst) & 3) == 0) {
          *reinterpret_cast<uint32_t*>(dst) = word;
        } else {
          for (int j = 0; j < n; ++j) dst[j] = (uint8_t)(word >> (8 * j));
        }
      }
    }
  }
  if (t == 0) bulk_wait_all();
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

// Hardware approximate reciprocal (about 1 ulp), subnormal results kept.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// ------------------------------------------------- SwiGLU fused with Q-row
// Megatron's SwiGLU with fp4_input_store (megatron-0.15.0rc7.diff:164-193)
// returns swiglu(x) = silu(x1) * x2 (x1, x2 the two halves of the last
// dimension) and keeps the MXFP4 quantization of x itself for the backward
// pass.  One pass reads x once and writes both: lane pairs own the gate block
// j (elements 32j..32j+31) and the up block j (H + 32j ..) of a row, quantize
// both exactly as Q-row does, and form 16 outputs each.  silu(g) * u is
// evaluated in f32 and rounded to BF16 once.
template <bool kFast>
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                           int64_t M, int64_t H,
                                                           __nv_bfloat16* __restrict__ y,
                                                           uint8_t* __restrict__ codes,
                                                           uint8_t* __restrict__ scales,
                                                           QuantParams p) {
  const int64_t J = H >> 5;        // block pairs per row
  const int64_t halves = M * J * 2;
  const int lane = threadIdx.x & 31;
  const unsigned pair_mask = 3u << (lane & ~1);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t K = 2 * H;         // row length of x
  // the 2 x 32 input bytes of work item h (gate and up half-blocks), loaded one
  // item ahead so that the loads overlap the previous item's arithmetic
  auto load_item = [&](int64_t h, uint32_t (&w)[2][8]) {
    const int64_t pr = h >> 1, r = pr / J, j = pr - r * J;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const uint8_t* src =
          reinterpret_cast<const uint8_t*>(x + r * K + s * H + j * 32 + (h & 1) * 16);
      const uint4 a = ld_stream_v4(src), b = ld_stream_v4(src + 16);
      w[s][0] = a.x; w[s][1] = a.y; w[s][2] = a.z; w[s][3] = a.w;
      w[s][4] = b.x; w[s][5] = b.y; w[s][6] = b.z; w[s][7] = b.w;
    }
  };
  int64_t base = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);
  uint32_t nxt[2][8];
  if (base + lane < halves) load_item(base + lane, nxt);
  for (; base < halves; base += stride) {
    const int64_t h = base + lane;
    uint32_t wv[2][8];  // [gate, up][16 elements as BF16 pairs]
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int i = 0; i < 8; ++i) wv[s][i] = nxt[s][i];
    if (base + stride + lane < halves) load_item(base + stride + lane, nxt);
    if (h >= halves) continue;  // pairs are both in or both out (halves is even)
    const int64_t pr = h >> 1;
    const int half = (int)(h & 1);
    const int64_t r = pr / J, j = pr - r * J;
    // ---- MXFP4 of both blocks (bit-exact Q-row)
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const uint32_t (&w)[8] = wv[s];
      uint32_t mb = max_abs_pairs(w);
      mb = max(mb, __shfl_xor_sync(pair_mask, mb, 1));
      uint32_t byte, out[2];
      if (kFast && mb < 0x7F80u) {
        uint32_t inv;
        scale_fast(mb, byte, inv);
        out[0] = encode8_pairs(&w[0], inv);
        out[1] = encode8_pairs(&w[4], inv);
      } else {
        uint32_t f0[8], f1[8];
        unpack8(&w[0], f0);
        unpack8(&w[4], f1);
        float am = fmaxf(amax_generic(f0, p.eps), amax_generic(f1, p.eps));
        am = fmaxf(am, __shfl_xor_sync(pair_mask, am, 1));
        float inv;
        scale_generic(am, p, inv, byte);
        out[0] = encode8_generic(f0, inv, p);
        out[1] = encode8_generic(f1, inv, p);
      }
      const int64_t blk = s * J + j;  // block index within the row of x
      st_stream_v2(codes + r * H + blk * 16 + half * 8, make_uint2(out[0], out[1]));
      if (half == 0) scales[r * (2 * J) + blk] = (uint8_t)byte;
    }
    // ---- swiglu of the 16 (gate, up) pairs
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float g = e ? bf16hi_to_f(wv[0][i]) : bf16lo_to_f(wv[0][i]);
        const float u = e ? bf16hi_to_f(wv[1][i]) : bf16lo_to_f(wv[1][i]);
        // g * u * (1 / (1 + e^-g)): the hardware exponential and reciprocal
        // (rcp.approx.f32, subnormal results kept) keep the relative error
        // near 1e-6, far inside one BF16 ulp; e^-g = Inf gives (g * u) * +0,
        // keeping the sign of zero
        v[e] = (g * u) * rcp_approx(1.0f + __expf(-g));
      }
      o[i] = cvt_bf16x2(v[0], v[1]);
    }
    uint8_t* dst = reinterpret_cast<uint8_t*>(y + r * H + j * 32 + half * 16);
    st_stream_v4(dst, make_uint4(o[0], o[1], o[2], o[3]));
    st_stream_v4(dst + 16, make_uint4(o[4], o[5], o[6], o[7]));
  }
}

template <bool kFp8>
void launch_quant_rows(bool fast, const void* input, int64_t M, int64_t K, int64_t ldx,
                       void* output_q, void* output_s, const QuantParams& p, void* fp8, void* fp8_s,
                       mxb_stream_t stream, bool ocp = false) {
  const void* kern = fast ? (const void*)quant_rows_kernel<true, kFp8>
                          : (const void*)quant_rows_kernel<false, kFp8>;
  if (ocp) kern = (const void*)quant_rows_kernel<true, kFp8, true>;
  const int64_t halves = M * (K / 32) * 2;
  const int64_t want = cdiv(halves, 256);
  const int64_t cap = (int64_t)persistent_ctas(kern, 256, 0) * 4;
  const int grid = (int)(want < cap ? want : cap);
  if (ocp)
    quant_rows_kernel<true, kFp8, true><<<grid, 256, 0, to_cuda(stream)>>>(
        (const __nv_bfloat16*)input, M, K, ldx, (uint8_t*)output_q, (uint8_t*)output_s, p,
        (uint8_t*)fp8, (float*)fp8_s);
  else if (fast)
    quant_rows_kernel<true, kFp8><<<grid, 256, 0, to_cuda(stream)>>>(
        (const __nv_bfloat16*)input, M, K, ldx, (uint8_t*)output_q, (uint8_t*)output_s, p,
        (uint8_t*)fp8, (float*)fp8_s);
  else
    quant_rows_kernel<false, kFp8><<<grid, 256, 0, to_cuda(stream)>>>(
        (const __nv_bfloat16*)input, M, K, ldx, (uint8_t*)output_q, (uint8_t*)output_s, p,
        (uint8_t*)fp8, (float*)fp8_s);
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
  launch_quant_rows<false>(fast, input, M, K, ldx, output_q, output_s, p, nullptr, nullptr, stream);
  return launch_status("quant_fp4");
}

extern "C" mxb_status mxb_per_token_group_quant_fp4_fused_ToFp8(
    const void* input, int64_t M, int64_t K, int64_t ldx, void* output_q, void* output_s,
    void* output_fp8, void* output_fp8_s, int group_size, float eps, float fp4_min, float fp4_max,
    int scale_ue8m0, mxb_stream_t stream) {
  MXB_REQUIRE(group_size == 32, MXB_ERR_UNSUPPORTED,
              "quant_fp4_fused_fp8: group_size must be 32 (got %d)", group_size);
  MXB_REQUIRE(!scale_ue8m0, MXB_ERR_UNSUPPORTED,
              "quant_fp4_fused_fp8: scale_ue8m0=True is rejected, as by the reference host assert");
  MXB_REQUIRE(M >= 0 && K >= 0 && K % 128 == 0, MXB_ERR_INVALID_ARGUMENT,
              "quant_fp4_fused_fp8: need K %% 128 == 0 (1x128 FP8 groups), got M=%lld K=%lld",
              (long long)M, (long long)K);
  MXB_REQUIRE(ldx >= K && ldx % 8 == 0, MXB_ERR_MISALIGNED,
              "quant_fp4_fused_fp8: row pitch must be >= K and a multiple of 8 elements");
  if (M == 0 || K == 0) return MXB_OK;
  MXB_REQUIRE(input && output_q && output_s && output_fp8 && output_fp8_s, MXB_ERR_INVALID_ARGUMENT,
              "quant_fp4_fused_fp8: null pointer");
  MXB_REQUIRE(aligned(input, 16) && aligned(output_q, 8) && aligned(output_fp8, 16) &&
                  aligned(output_fp8_s, 4),
              MXB_ERR_MISALIGNED,
              "quant_fp4_fused_fp8: input and output_fp8 must be 16-byte, output_q 8-byte and "
              "output_fp8_s 4-byte aligned");
  const QuantParams p{eps, fp4_min, fp4_max};
  launch_quant_rows<true>(fast_params(eps, fp4_min, fp4_max), input, M, K, ldx, output_q, output_s,
                          p, output_fp8, output_fp8_s, stream);
  return launch_status("quant_fp4_fused_fp8");
}

extern "C" mxb_status mxb_swiglu_quant_mxfp4(const void* input, int64_t M, int64_t H, void* output,
                                             void* codes, void* scales, float eps, float fp4_min,
                                             float fp4_max, mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && H >= 0 && H % 32 == 0, MXB_ERR_INVALID_ARGUMENT,
              "swiglu_quant: need H %% 32 == 0 (M=%lld H=%lld)", (long long)M, (long long)H);
  if (M == 0 || H == 0) return MXB_OK;
  MXB_REQUIRE(input && output && codes && scales, MXB_ERR_INVALID_ARGUMENT,
              "swiglu_quant: null pointer");
  MXB_REQUIRE(aligned(input, 16) && aligned(output, 16) && aligned(codes, 8), MXB_ERR_MISALIGNED,
              "swiglu_quant: input and output must be 16-byte and codes 8-byte aligned");
  const QuantParams p{eps, fp4_min, fp4_max};
  const bool fast = fast_params(eps, fp4_min, fp4_max);
  const void* kern = fast ? (const void*)swiglu_quant_kernel<true> : (const void*)swiglu_quant_kernel<false>;
  const int64_t halves = M * (H / 32) * 2;
  const int64_t want = cdiv(halves, 256);
  const int64_t cap = (int64_t)persistent_ctas(kern, 256, 0) * 4;
  const int grid = (int)(want < cap ? want : cap);
  if (fast)
    swiglu_quant_kernel<true><<<grid, 256, 0, to_cuda(stream)>>>(
        (const __nv_bfloat16*)input, M, H, (__nv_bfloat16*)output, (uint8_t*)codes,
        (uint8_t*)scales, p);
  else
    swiglu_quant_kernel<false><<<grid, 256, 0, to_cuda(stream)>>>(
        (const __nv_bfloat16*)input, M, H, (__nv_bfloat16*)output, (uint8_t*)codes,
        (uint8_t*)scales, p);
  return launch_status("swiglu_quant");
}

// The fused row + column quantize behind mxb_quant_mxfp4_rowcol and
// mxb_quantize_mxfp4 (ocp: the OCP scale rule, default parameters only).
static mxb_status quant_rowcol_impl(const void* input, int64_t M, int64_t K, int64_t ldx,
                                    void* codes_row, void* scales_row, void* codes_col,
                                    void* scales_col, void* scales_row_swizzled, float eps,
                                    float fp4_min, float fp4_max, bool ocp, mxb_stream_t stream) {
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
  MXB_REQUIRE(aligned(input, 16) && aligned(codes_col, 16) && (!codes_row || aligned(codes_row, 16)),
              MXB_ERR_MISALIGNED, "quant_rowcol: input and code outputs must be 16-byte aligned");
  cudaStream_t s = to_cuda(stream);
  if (scales_row_swizzled) {
    const int64_t bytes = (M + 127) / 128 * 128 * ((K / 32 + 3) / 4 * 4);
    cudaError_t e = cudaMemsetAsync(scales_row_swizzled, 0, (size_t)bytes, s);
    MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "quant_rowcol: memset failed: %s",
                cudaGetErrorString(e));
  }
  const QuantParams p{eps, fp4_min, fp4_max};
  const bool fast = fast_params(eps, fp4_min, fp4_max);
  CUtensorMap tm_in, tm_row, tm_col;
  if (!make_tensor_map_2d(&tm_in, input, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, ldx, kTile,
                          kTile))
    return MXB_ERR_CUDA;
  // code outputs: uint8 [M, K/2] and [K, M/2], 64-byte x 128-row boxes, 64-byte swizzle
  if (codes_row && !make_tensor_map_2d(&tm_row, codes_row, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M,
                                       K / 2, K / 2, 64, kTile, CU_TENSOR_MAP_SWIZZLE_64B))
    return MXB_ERR_CUDA;
  if (!codes_row) tm_row = tm_in;  // unused when the row outputs are skipped
  if (!make_tensor_map_2d(&tm_col, codes_col, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M / 2, M / 2,
                          64, kTile, CU_TENSOR_MAP_SWIZZLE_64B))
    return MXB_ERR_CUDA;
  const int64_t col_tiles = cdiv(K, kTile), tiles = col_tiles * cdiv(M, kTile);
  MXB_REQUIRE(tiles < (1LL << 31), MXB_ERR_INVALID_ARGUMENT, "quant_rowcol: tensor too large");
  auto* sr = (uint8_t*)scales_row;
  auto* sc = (uint8_t*)scales_col;
  auto* sw = (uint8_t*)scales_row_swizzled;
  using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, int64_t, int64_t,
                        uint8_t*, uint8_t*, uint8_t*, QuantParams, int, int);
  Kern kern = codes_row ? (fast ? quant_rowcol_kernel<true, true> : quant_rowcol_kernel<false, true>)
                        : (fast ? quant_rowcol_kernel<true, false> : quant_rowcol_kernel<false, false>);
  if (ocp) kern = codes_row ? quant_rowcol_kernel<true, true, true> : quant_rowcol_kernel<true, false, true>;
  static const bool attr_ok = [] {
    bool ok = true;
    for (Kern k : {quant_rowcol_kernel<true, true>, quant_rowcol_kernel<false, true>,
                   quant_rowcol_kernel<true, false>, quant_rowcol_kernel<false, false>,
                   quant_rowcol_kernel<true, true, true>, quant_rowcol_kernel<true, false, true>})
      ok &= cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kRowColSmem) == cudaSuccess;
    return ok;
  }();
  MXB_REQUIRE(attr_ok, MXB_ERR_CUDA, "quant_rowcol: cannot reserve %zu bytes of shared memory",
              kRowColSmem);
  const int64_t cap = (int64_t)persistent_ctas((const void*)kern, kRowColThreads, kRowColSmem);
  const int grid = (int)(tiles < cap ? tiles : cap);
  kern<<<grid, kRowColThreads, kRowColSmem, s>>>(tm_in, tm_row, tm_col, M, K, sr, sc, sw, p,
                                                 (int)col_tiles, (int)tiles);
  return launch_status("quant_rowcol");
}

extern "C" mxb_status mxb_quant_mxfp4_rowcol(const void* input, int64_t M, int64_t K, int64_t ldx,
                                             void* codes_row, void* scales_row, void* codes_col,
                                             void* scales_col, void* scales_row_swizzled,
                                             float eps, float fp4_min, float fp4_max,
                                             mxb_stream_t stream) {
  return quant_rowcol_impl(input, M, K, ldx, codes_row, scales_row, codes_col, scales_col,
                           scales_row_swizzled, eps, fp4_min, fp4_max, false, stream);
}

extern "C" mxb_status mxb_quantize_mxfp4(const void* input, int64_t M, int64_t K, int64_t ldx,
                                         void* codes_row, void* scales_row, void* codes_col,
                                         void* scales_col, void* scales_row_swizzled,
                                         int scale_rule, mxb_stream_t stream) {
  MXB_REQUIRE(scale_rule == MXB_SCALE_REFERENCE || scale_rule == MXB_SCALE_OCP,
              MXB_ERR_INVALID_ARGUMENT, "quantize_mxfp4: unknown scale rule %d", scale_rule);
  const bool ocp = scale_rule == MXB_SCALE_OCP;
  const float eps = 1e-10f, lo = -6.0f, hi = 6.0f;
  if (codes_col || scales_col)
    return quant_rowcol_impl(input, M, K, ldx, codes_row, scales_row, codes_col, scales_col,
                             scales_row_swizzled, eps, lo, hi, ocp, stream);
  // rowwise only
  MXB_REQUIRE(M >= 0 && K >= 0 && K % 32 == 0, MXB_ERR_INVALID_ARGUMENT,
              "quantize_mxfp4: need M >= 0 and K %% 32 == 0 (M=%lld K=%lld)", (long long)M,
              (long long)K);
  MXB_REQUIRE(ldx >= K && ldx % 8 == 0, MXB_ERR_MISALIGNED,
              "quantize_mxfp4: row pitch must be >= K and a multiple of 8 elements");
  if (M == 0 || K == 0) return MXB_OK;
  MXB_REQUIRE(input && codes_row && scales_row, MXB_ERR_INVALID_ARGUMENT,
              "quantize_mxfp4: null pointer (a rowwise call needs codes_row and scales_row)");
  MXB_REQUIRE(aligned(input, 16) && aligned(codes_row, 8), MXB_ERR_MISALIGNED,
              "quantize_mxfp4: input must be 16-byte and codes_row 8-byte aligned");
  const QuantParams p{eps, lo, hi};
  launch_quant_rows<false>(true, input, M, K, ldx, codes_row, scales_row, p, nullptr, nullptr,
                           stream, ocp);
  mxb_status st = launch_status("quantize_mxfp4");
  if (st != MXB_OK || !scales_row_swizzled) return st;
  return mxb_swizzle_scales(scales_row, M, K / 32, scales_row_swizzled, stream);
}

extern "C" unsigned int mxb_wait_timeouts(void) { return sum_wait_timeouts(false); }
extern "C" unsigned int mxb_reset_wait_timeouts(void) { return sum_wait_timeouts(true); }

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
