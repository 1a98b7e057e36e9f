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
#include <mutex>
#include <type_traits>

#include "capi_util.h"
#include "common.cuh"
#include "fp8_lut.cuh"
#include "tma.cuh"

namespace mxb {
namespace {

constexpr int kThreads = 256;

__device__ const Fp8Lut g_lut_col = make_fp8_lut(true);

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
// The transposed tile has 128-byte element rows whose 16-byte chunks are
// XOR-swizzled by (element & 3) << 1: the four lanes that write four element
// rows of the same 4-byte column, and the two half-warps, land in eight
// different chunks (no bank conflicts), and the 8 lanes that read one element
// row read a permutation of its chunks.
constexpr int kColPitch = 128;                 // bytes per element row of the transposed tile
constexpr uint32_t kColCodeBytes = 128 * 128;  // 16 KiB

// 4x4 byte transpose across lanes 4m..4m+3: in, lane i holds row i's bytes for
// elements 0..3; out, lane i holds element i's bytes for rows 0..3.
__device__ __forceinline__ uint32_t transpose4x4(uint32_t w, uint32_t sel1, uint32_t sel2) {
  const uint32_t t = prmt(w, __shfl_xor_sync(0xffffffffu, w, 2), sel1);
  return prmt(t, __shfl_xor_sync(0xffffffffu, t, 1), sel2);
}

// The tile's 256 output rows leave in four phases of 64 (each warp converts
// one of its four 32-column blocks per phase) through a staging tile of 64
// element rows (~26 KB of shared memory per CTA).  Measured on config 3:
// whole-tile staging (4 CTAs per SM): 120 us; two phases: 115 us; four phases:
// 89 us with the compiler's 40 registers (6 CTAs per SM), but 117 us when held
// to 32 registers for 8 CTAs per SM: the gain is the loads the compiler keeps
// in flight within a phase, not the occupancy.
constexpr int kColPhases = 4;                  // output phases per tile (2 or 4)
static_assert(kColPhases == 2 || kColPhases == 4, "each warp converts whole 32-column blocks");
constexpr int kColPhaseRows = 256 / kColPhases;  // output rows staged per phase
constexpr size_t kColSmem = 1024 + kColCodeBytes + kColPhaseRows * kColPitch + 4 * 8 + 16;

__global__ void __launch_bounds__(kThreads) fp8_col_kernel(const __grid_constant__ CUtensorMap tmap,
                                                           const uint8_t* __restrict__ scales,
                                                           int64_t M, int64_t Kb,
                                                           uint8_t* __restrict__ out,
                                                           float* __restrict__ scales_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ctile = smem;                                      // 128 x 128 B (128-byte swizzle)
  uint8_t* tr = smem + kColCodeBytes;                         // [element][row] FP8, one phase
  uint32_t* red = reinterpret_cast<uint32_t*>(tr + kColPhaseRows * kColPitch);  // [4 row blocks][2 words]
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + 8);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int rb = warp >> 1, hh = warp & 1;  // 32-row block, 64-byte half of the tile
  // row blocks fastest: CTAs running together extend the same 256 output rows
  // (adjacent 128-byte runs), so the transposed writes merge into long runs
  const int64_t row0 = (int64_t)blockIdx.x * 128;
  const int64_t cb0 = (int64_t)blockIdx.y * 128;  // first code byte of the tile
  const int64_t S = Kb / 16;
  const int r = rb * 32 + lane;

  // the tile's copy goes out first, so that it lands while the scale loads
  // and their reduction run
  if (t == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar, kColCodeBytes);
    tma_load_2d(ctile, &tmap, (int32_t)cb0, (int32_t)row0, bar);
  }
  // this row's eight E8M0 bytes (one per 32-column block of the tile)
  // (evict-last: the three column tiles beside this one read the same sector)
  const uint2 sc = ld_keep_v2(scales + (row0 + r) * S + cb0 / 16, l2_keep_policy());
  if (hh == 0) {
    uint32_t m0 = sc.x, m1 = sc.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      m0 = max_u8x4(m0, __shfl_xor_sync(0xffffffffu, m0, o));
      m1 = max_u8x4(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    if (lane == 0) {
      red[rb * 2] = m0;
      red[rb * 2 + 1] = m1;
    }
  }
  __syncthreads();  // the barrier's initialisation and red[] are visible
  if (__syncthreads_or(!mbar_wait(bar, 0))) return;  // the copy never completed
  const uint32_t mx0 = max_u8x4(max_u8x4(red[0], red[2]), max_u8x4(red[4], red[6]));
  const uint32_t mx1 = max_u8x4(max_u8x4(red[1], red[3]), max_u8x4(red[5], red[7]));
  // lane-dependent byte selectors of the two transpose rounds
  const uint32_t sel1 = (lane & 2) ? 0x3276u : 0x5410u;
  const uint32_t sel2 = (lane & 1) ? 0x3715u : 0x6240u;
  // this lane stores element (4k + (lane & 3)) for rows (lane & ~3) .. +3: byte
  // column rb * 32 + (lane & ~3), chunk rb * 2 + lane / 16 swizzled by (lane & 3) << 1
  uint8_t* trl = tr + (lane & 3) * kColPitch +
                 ((((rb * 2 + (lane >> 4)) ^ ((lane & 3) << 1))) << 4) + ((lane >> 2) & 3) * 4;
  // scales: [M/128, 2*Kb], each block scale repeated over its 32 columns
  {
    const int q = t >> 5;
    const uint32_t wa = ((((q < 4 ? mx0 : mx1) >> (8 * (q & 3))) & 0xFFu) - 6u) & 0xFFu;
    scales_out[(row0 / 128) * (2 * Kb) + 2 * cb0 + t] = __uint_as_float(wa << 23);
  }
#pragma unroll
  for (int p = 0; p < kColPhases; ++p) {
    constexpr int kQ = 8 / kColPhases;  // 32-column blocks per phase
#pragma unroll
    for (int cc = 0; cc < kQ / 2; ++cc) {
      const int q = kQ * p + (kQ / 2) * hh + cc;  // phase p covers blocks kQ*p .. kQ*p + kQ - 1
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
          const int n = (q - kQ * p) * 32 + j * 8 + hw * 4;  // element row within the phase
          *reinterpret_cast<uint32_t*>(trl + n * kColPitch) = transpose4x4(f4, sel1, sel2);
        }
      }
    }
    __syncthreads();
    // output rows 2*cb0 + kColPhaseRows * p + 0..: 128 FP8 bytes each at columns row0..row0+127
    uint8_t* ob = out + (2 * cb0 + kColPhaseRows * p) * M + row0;
#pragma unroll
    for (int k = 0; k < kColPhaseRows * 8 / kThreads; ++k) {
      const int i = k * kThreads + t;
      const int n = i >> 3, part = i & 7;
      const uint4 o =
          *reinterpret_cast<const uint4*>(&tr[n * kColPitch + ((part ^ ((n & 3) << 1)) << 4)]);
      st_stream_v4(ob + n * M + part * 16, o);
    }
    if (p + 1 < kColPhases) __syncthreads();  // the staging tile is refilled by the next phase
  }
}

// ------------------------------------------------------- colT / colT-split
// Persistent: each CTA walks tiles of 128 rows x 128 elements (tile = blockIdx.x
// + i * gridDim.x, row blocks fastest so that neighbouring CTAs extend the same
// output rows).  While it converts tile i, the TMA copy of tile i+1's codes
// lands in the other half of a two-stage ring and tile i+1's E8M0 bytes are in
// flight to registers, so neither load's latency is exposed.
//
// Thread (wc = t % 16, rg = t / 16) owns the 8 x 8 block of rows 8rg..8rg+7 and
// columns 8wc..8wc+7 and keeps it in registers, as f32, from decode to FP8:
//   1. one 32-bit code word per row (lanes 16..31 read their rows in the order
//      k ^ 1 so that the two half-warps hit different bank halves), decoded and
//      scaled by the row's E8M0 factor (decode8_scaled: exact);
//   2. column amax over the 8 rows (three-input max of magnitudes), then across
//      the warp's two row groups with one shuffle, then across the 8 warps
//      through shared memory;
//   3. per column, row pairs are scaled and converted to E4M3 (the 8 bytes of
//      the column's 8 rows) and stored as one 8-byte chunk of the transposed
//      staging tile, whose 8-byte chunk index is XOR-swizzled by column / 8 so
//      that the 16 lanes of a half-warp hit 16 different bank pairs;
//   4. the staging tile leaves as 128-byte runs of output rows.
// The instruction mix is chosen for the SM's pipes: decoding runs on the
// conversion unit, widening and scaling on the FMA pipe, leaving the integer
// pipe the amax, the E4M3 conversion and the transpose.
struct SplitArgs {
  const int32_t* m_splits;
  const int32_t* split_offsets;
  const int32_t* scale_offsets;
};

// Position of a CTA in its tile walk: tile = (z * ns + s) * nb + b, where z is
// the 128-column block, s the segment (always 0 without splits) and b the
// 128-row block within it.  Advancing by gridDim.x tiles is a carry-add of the
// step's own (z, s, b) digits, so the walk needs no division after the start.
struct ColTWalk {
  int64_t z;
  int s, b;
};

__device__ __forceinline__ ColTWalk colT_digits(int64_t idx, int ns, int nb) {
  ColTWalk w;
  const int64_t sb = (int64_t)ns * nb;
  w.z = idx / sb;
  const int64_t r = idx - w.z * sb;
  w.s = (int)(r / nb);
  w.b = (int)(r - (int64_t)w.s * nb);
  return w;
}

__device__ __forceinline__ void colT_advance(ColTWalk& w, const ColTWalk& step, int ns, int nb) {
  w.z += step.z;
  w.s += step.s;
  w.b += step.b;
  if (w.b >= nb) {
    w.b -= nb;
    ++w.s;
  }
  if (w.s >= ns) {
    w.s -= ns;
    ++w.z;
  }
}

// Where one 128 x 128 tile reads and writes.
struct ColTTile {
  int64_t row_start, out_base, out_pitch, scale_row, col0;
  int rows, cols;
  bool merge_in, carry_out;  // split path: partial chunks shared with the previous / next tile
};

// Tile at walk position w; false if it lies past the end of its segment.
template <bool kSplit>
__device__ __forceinline__ bool colT_tile(const ColTWalk& w, int64_t M, int64_t N,
                                          const SplitArgs& sa, ColTTile& g) {
  g.col0 = w.z * 128;
  g.cols = (int)min((int64_t)128, N - g.col0);
  g.merge_in = g.carry_out = false;
  if (kSplit) {
    const int64_t mi = sa.m_splits[w.s];
    if ((int64_t)w.b * 128 >= mi) return false;
    const int64_t o = sa.split_offsets[w.s];
    g.row_start = o + (int64_t)w.b * 128;
    g.rows = (int)min((int64_t)128, mi - (int64_t)w.b * 128);
    g.out_base = o * N + (int64_t)w.b * 128;  // + n * mi + local row
    g.out_pitch = mi;
    g.scale_row = sa.scale_offsets[w.s] + w.b;
  } else {
    g.row_start = (int64_t)w.b * 128;
    g.rows = (int)min((int64_t)128, M - g.row_start);
    g.out_base = g.row_start;
    g.out_pitch = M;
    g.scale_row = w.b;
  }
  return true;
}

// Advances w to this CTA's next non-empty tile; false when the walk is over.
template <bool kSplit>
__device__ __forceinline__ bool colT_next(ColTWalk& w, const ColTWalk& step, int64_t zt, int ns,
                                          int nb, int64_t M, int64_t N, const SplitArgs& sa,
                                          ColTTile& g) {
  for (;;) {
    colT_advance(w, step, ns, nb);
    if (w.z >= zt) return false;
    if (colT_tile<kSplit>(w, M, N, sa, g)) return true;
  }
}

// Split path walk.  A segment's output [N, m_i] is one contiguous block, so
// its row segments start at n * m_i and are rarely 16-byte aligned; the
// 16-byte memory chunk a row segment shares with the next 128-row block is
// written once, whole, when the same CTA converts that block next.  So the
// split path walks units of up to kUnitTiles consecutive row blocks of one
// (segment, 128-column block): unit = (s * SS + ss) * ZT + z with z fastest
// (neighbouring CTAs convert neighbouring columns of the same rows), ss the
// unit's index along the segment, SS = ceil(nb / kUnitTiles) for the longest
// segment (units past a segment's end are empty).  Partial chunks remain only
// at unit ends.  Digits (z, ss, s) advance by the step's digits without
// division, as in the tile walk.
constexpr int kUnitTiles = 2;

struct SplitWalk {
  int64_t z;
  int s, ss, bi;  // bi: tile within the unit
};

__device__ __forceinline__ SplitWalk split_digits(int64_t idx, int SS, int64_t ZT) {
  SplitWalk w;
  const int64_t r = idx / ZT;
  w.z = idx - r * ZT;
  w.s = (int)(r / SS);
  w.ss = (int)(r - (int64_t)w.s * SS);
  w.bi = 0;
  return w;
}

// Tile (s, z, b = kUnitTiles * ss + bi) of the split path; false past the segment's end.
__device__ __forceinline__ bool split_tile(const SplitWalk& w, int64_t N, const SplitArgs& sa,
                                           ColTTile& g) {
  const int64_t mi = sa.m_splits[w.s];
  const int64_t b = (int64_t)w.ss * kUnitTiles + w.bi;
  if (b * 128 >= mi) return false;
  const int64_t o = sa.split_offsets[w.s];
  g.col0 = w.z * 128;
  g.cols = (int)min((int64_t)128, N - g.col0);
  g.row_start = o + b * 128;
  g.rows = (int)min((int64_t)128, mi - b * 128);
  g.out_base = o * N + b * 128;  // + n * mi + local row
  g.out_pitch = mi;
  g.scale_row = sa.scale_offsets[w.s] + b;
  g.merge_in = w.bi > 0;
  g.carry_out = w.bi + 1 < kUnitTiles && (b + 1) * 128 < mi;
  return true;
}

// The CTA's next tile: the next block of the unit, else the first tile of its
// next non-empty unit; false when the walk is over.
__device__ __forceinline__ bool split_next(SplitWalk& w, const SplitWalk& step, int ns, int SS,
                                           int64_t ZT, int64_t N, const SplitArgs& sa,
                                           ColTTile& g) {
  if (g.carry_out) {
    ++w.bi;
    return split_tile(w, N, sa, g);
  }
  for (;;) {
    w.bi = 0;
    w.z += step.z;
    w.ss += step.ss;
    w.s += step.s;
    if (w.z >= ZT) {
      w.z -= ZT;
      ++w.ss;
    }
    if (w.ss >= SS) {
      w.ss -= SS;
      ++w.s;
    }
    if (w.s >= ns) return false;
    if (split_tile(w, N, sa, g)) return true;
  }
}

// Row r's four E8M0 bytes of a tile, loaded raw so that the load's latency
// stays hidden until colT_factors consumes them at the end of the tile.
__device__ __forceinline__ uint32_t colT_scale_word(const uint8_t* scales, int64_t S,
                                                    const ColTTile& g, int r) {
  uint32_t sc = 0;
  if (r < g.rows) {
    const uint8_t* sp = scales + (g.row_start + r) * S + g.col0 / 32;
    if (g.cols == 128 && (reinterpret_cast<uintptr_t>(sp) & 3) == 0) {
      // the seven other 128-column tiles of these rows that share the 32-byte
      // sector read it again (evict-last keeps it in L2 until they do)
      sc = ld_keep_u32(sp, l2_keep_policy());
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (q * 32 < g.cols) sc |= (uint32_t)ld_stream_u8(sp + q) << (8 * q);
    }
  }
  return sc;
}

// Stores row r's four E8M0 factors of a tile as float bit patterns (e << 23:
// e = 0 reads 0, e = 255 reads Inf, as the reference's BF16 reading does)
// into fac[q * 128 + r]; true if a factor is Inf.  colT_scale_word leaves the
// bytes past the tile's edges 0, whose factor 0 meets only zero codes there
// (the copy's zero fill, or the split path's masked rows), so the tile's
// shape is not needed here.
__device__ __forceinline__ bool colT_factors(uint32_t sc, int r, uint32_t* fac) {
  bool special = false;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t e = (sc >> (8 * q)) & 0xFFu;
    fac[q * 128 + r] = e << 23;
    special = special || e == 255u;
  }
  return special;
}

// max(|a|, |b|, |c|), NaN inputs ignored (sm_100 three-input max).
__device__ __forceinline__ float max3_abs(float a, float b, float c) {
  float r;
  asm("max.abs.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

constexpr int kColTStages = 2;
constexpr uint32_t kColTCodeBytes = 128 * 64;  // 128 rows x 64 code bytes, unswizzled

// Stores bytes [lo, hi) of the 16-byte value v at the 16-byte aligned address
// b, as naturally aligned pieces: pieces of 1, 2, 4, 8 bytes bring the start
// up to 16-byte alignment, then pieces of 8, 4, 2, 1 bytes cover the rest.
__device__ __forceinline__ void st_piece(uint8_t* b, uint64_t w0, uint64_t w1, int pos, int sz) {
  const uint64_t piece = pos < 8 ? (w0 >> (8 * pos)) : (w1 >> (8 * (pos - 8)));
  if (sz == 8) {
    asm volatile("st.global.cs.u64 [%0], %1;" ::"l"(b + pos), "l"(piece) : "memory");
  } else if (sz == 4) {
    st_stream_u32(b + pos, (uint32_t)piece);
  } else if (sz == 2) {
    asm volatile("st.global.cs.u16 [%0], %1;" ::"l"(b + pos), "h"((uint16_t)piece) : "memory");
  } else {
    st_stream_u8(b + pos, (uint32_t)piece & 0xFFu);
  }
}

__device__ __forceinline__ void store_bytes16(uint8_t* b, uint4 v, int lo, int hi) {
  const uint64_t w0 = ((uint64_t)v.y << 32) | v.x, w1 = ((uint64_t)v.w << 32) | v.z;
  int pos = lo;
#pragma unroll
  for (int sz = 1; sz <= 8; sz <<= 1) {
    if ((pos & sz) && pos + sz <= hi) {
      st_piece(b, w0, w1, pos, sz);
      pos += sz;
    }
  }
#pragma unroll
  for (int sz = 8; sz >= 1; sz >>= 1) {
    if (pos + sz <= hi) {
      st_piece(b, w0, w1, pos, sz);
      pos += sz;
    }
  }
}

// Bytes 0 .. a-1 from c, bytes a .. 15 from o.
__device__ __forceinline__ uint4 blend16(uint4 c, uint4 o, int a) {
  const uint32_t cw[4] = {c.x, c.y, c.z, c.w}, ow[4] = {o.x, o.y, o.z, o.w};
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = a - 4 * i;  // bytes of word i taken from c
    const uint32_t m = k >= 4 ? 0xFFFFFFFFu : (k <= 0 ? 0u : (1u << (8 * k)) - 1u);
    r[i] = (cw[i] & m) | (ow[i] & ~m);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Output row segments of the split path start at n * m_i and are rarely 16-byte
// aligned.  A row segment of `len` bytes starting at `row` (a = row % 16) is
// written as the 16-byte aligned chunks of memory it covers: memory chunk m
// holds data bytes 16m - a .. 16m - a + 15, i.e. the top a bytes of data chunk
// m-1 followed by the low 16 - a bytes of data chunk m (shift_window).  Chunks
// 1-7 (the body) are written by lane m of the row's eight lanes from its own
// and its neighbour's data chunk; the two edge chunks, 0 and 8, by one thread
// per row in a second pass (store_row_edges), so that their heavier code does
// not run serialised beside the body lanes.  Memory chunk 8 is memory chunk 0
// of the next 128-row block: with carry_out it is kept in carry[n] instead of
// stored, and with merge_in this block's chunk 0 is completed from carry[n]
// and stored whole.  Other partial chunks are written in naturally aligned
// pieces, so neighbouring segments' bytes are never touched.
__device__ __forceinline__ uint4 shift_window(uint4 prev, uint4 d, int a) {
  if (a == 0) return d;
  // out word i = bytes 16 - a + 4i .. + 3 of W = (prev, d): words W[qs + i],
  // W[qs + i + 1] funnel-shifted by rs bytes, qs = (16 - a) / 4, rs = (16 - a) % 4
  const int sft = 16 - a, qs = sft >> 2, rs = sft & 3;
  const uint32_t W[8] = {prev.x, prev.y, prev.z, prev.w, d.x, d.y, d.z, d.w};
  uint32_t X[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const uint32_t lo2 = (qs & 1) ? W[k + 1] : W[k];
    const uint32_t hi2 = (qs & 1) ? W[k + 3] : W[k + 2];
    X[k] = (qs & 2) ? hi2 : lo2;
  }
  return make_uint4(__funnelshift_r(X[0], X[1], 8 * rs), __funnelshift_r(X[1], X[2], 8 * rs),
                    __funnelshift_r(X[2], X[3], 8 * rs), __funnelshift_r(X[3], X[4], 8 * rs));
}

// Body chunk p (1..7) of a row segment; d and prev are data chunks p and p-1.
__device__ __forceinline__ void store_row_body(uint8_t* row, int p, uint4 d, uint4 prev, int len) {
  const int a = (int)(reinterpret_cast<uintptr_t>(row) & 15);
  uint8_t* base = row - a;  // 16-byte aligned
  // memory chunk p covers data bytes [16p - a, 16p - a + 16) clipped to [0, len)
  const int hi = min(16, len + a - 16 * p);
  if (hi <= 0) return;
  const uint4 o = shift_window(prev, d, a);
  if (hi == 16) {
    st_stream_v4(base + 16 * p, o);
  } else {
    store_bytes16(base + 16 * p, o, 0, hi);
  }
}

// Edge chunks 0 and 8 of a row segment; c7 and c0 are data chunks 7 and 0.
__device__ __forceinline__ void store_row_edges(uint8_t* row, uint4 c7, uint4 c0, int len,
                                                bool merge_in, bool carry_out, uint4* carry) {
  const int a = (int)(reinterpret_cast<uintptr_t>(row) & 15);
  uint8_t* base = row - a;  // 16-byte aligned
  // the low a bytes: data 128 - a .. 127 (chunk 8); the rest: data 0 .. 15 - a (chunk 0)
  const uint4 o = shift_window(c7, c0, a);
  {  // memory chunk 0: bytes [a, min(16, len + a)) of this block
    const int hi = min(16, len + a);
    const uint4 v = (merge_in && a != 0) ? blend16(*carry, o, a) : o;
    const int lo = (merge_in || a == 0) ? 0 : a;
    if (lo == 0 && hi == 16) {
      st_stream_v4(base, v);
    } else {
      store_bytes16(base, v, lo, hi);
    }
  }
  // memory chunk 8: bytes [0, min(a, len + a - 128)) (data 128 - a .. len - 1),
  // present when the segment reaches past memory chunk 7
  if (a != 0 && len + a > 128) {
    if (carry_out) {  // implies len == 128
      *carry = o;
    } else {
      store_bytes16(base + 128, o, 0, min(a, len + a - 128));
    }
  }
}

template <bool kSplit>
__global__ void __launch_bounds__(kThreads) fp8_colT_kernel(const __grid_constant__ CUtensorMap tmap,
                                                            const uint8_t* __restrict__ scales,
                                                            int64_t M, int64_t N, float eps,
                                                            uint8_t* __restrict__ out,
                                                            float* __restrict__ scales_out,
                                                            SplitArgs sa, int ns, int nb,
                                                            int64_t zt) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~uintptr_t(127));
  uint8_t* ctiles = smem;                                  // 2 x [128 rows][64 B] codes
  uint8_t* otile = ctiles + kColTStages * kColTCodeBytes;  // [128 cols][16 x 8 B] FP8, swizzled
  uint32_t* part = reinterpret_cast<uint32_t*>(otile + 128 * 128);  // [8 warps][128 cols]
  float* col_qs = reinterpret_cast<float*>(part + 8 * 128);         // [128]
  uint8_t* col_clamp = reinterpret_cast<uint8_t*>(col_qs + 128);    // [128]
  uint32_t* fac = reinterpret_cast<uint32_t*>(col_clamp + 128);     // 2 x [4 blocks][128 rows]
  uint64_t* full = reinterpret_cast<uint64_t*>(fac + 2 * 512);      // [2]
  int* timeout_flag = reinterpret_cast<int*>(full + 2);
  uint4* carry = reinterpret_cast<uint4*>(full + 4);                 // [128 output rows]
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int wc = t & 15, rg = t >> 4;
  const uint32_t up = (uint32_t)(t >> 4) & 1u;
  const int64_t S = N / 32;

  // walk: tiles of the column/row-block grid, or units of a segment on the
  // split path (nb is then the number of units along the longest segment)
  using Walk = std::conditional_t<kSplit, SplitWalk, ColTWalk>;
  Walk step, w;
  ColTTile g;
  if constexpr (kSplit) {
    step = split_digits(gridDim.x, nb, zt);
    w = split_digits(blockIdx.x, nb, zt);
    if (w.s >= ns) return;
    if (!split_tile(w, N, sa, g)) {
      g.carry_out = false;
      if (!split_next(w, step, ns, nb, zt, N, sa, g)) return;
    }
  } else {
    step = colT_digits(gridDim.x, ns, nb);
    w = colT_digits(blockIdx.x, ns, nb);
    if (w.z >= zt) return;
    if (!colT_tile<false>(w, M, N, sa, g) && !colT_next<false>(w, step, zt, ns, nb, M, N, sa, g))
      return;
  }
  bool special_next = false;  // an Inf factor in the tile whose factors this thread loaded
  if (t == 0) {
    *timeout_flag = 0;
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&full[0], kColTCodeBytes);
    tma_load_2d(ctiles, &tmap, (int32_t)(g.col0 / 2), (int32_t)g.row_start, &full[0]);
  }
  if (t < 128) special_next = colT_factors(colT_scale_word(scales, S, g, t), t, fac);
  __syncthreads();

  int issued = 1;  // code tiles requested so far (tile i uses stage i & 1)
  for (int i = 0;; ++i) {
    const bool special_cur = special_next;
    // ---- prefetch tile i+1: its codes into the other stage, its factors into registers
    Walk wn = w;
    ColTTile gn = g;
    bool has_next;
    if constexpr (kSplit) {
      has_next = split_next(wn, step, ns, nb, zt, N, sa, gn);
    } else {
      has_next = colT_next<false>(wn, step, zt, ns, nb, M, N, sa, gn);
    }
    if (has_next) {
      // the other stage was last read in tile i-1's step 1, which every thread has left
      if (t == 0) {
        uint64_t* bar = &full[(i + 1) & 1];
        mbar_arrive_expect_tx(bar, kColTCodeBytes);
        tma_load_2d(ctiles + ((i + 1) & 1) * kColTCodeBytes, &tmap, (int32_t)(gn.col0 / 2),
                    (int32_t)gn.row_start, bar);
      }
      ++issued;
    }
    const uint32_t sc_next = (has_next && t < 128) ? colT_scale_word(scales, S, gn, t) : 0u;
    // A copy that never arrives is reported at the next barrier (the tile's
    // values are then garbage and never stored).
    const bool ok = mbar_wait(&full[i & 1], (uint32_t)(i >> 1) & 1u);
    if (!ok) *timeout_flag = 1;

    // ---- 1. codes and factors of this thread's 8 x 8 block -> f32 values
    const int row_base = rg * 8;
    uint32_t cw[8];
    {
      const uint32_t* ct = reinterpret_cast<const uint32_t*>(ctiles + (i & 1) * kColTCodeBytes) +
                           row_base * 16 + wc;
#pragma unroll
      for (int k = 0; k < 8; ++k) cw[k] = ct[(k ^ (int)up) * 16];
#pragma unroll
      for (int k = 0; k < 8; k += 2) {  // undo the k ^ 1 read order
        const uint32_t a = cw[k], b = cw[k + 1];
        cw[k] = up ? b : a;
        cw[k + 1] = up ? a : b;
      }
    }
    const uint4* fp = reinterpret_cast<const uint4*>(fac + (i & 1) * 512 + (wc >> 2) * 128 + row_base);
    const uint4 fa = fp[0], fb = fp[1];
    const uint32_t fr[8] = {fa.x, fa.y, fa.z, fa.w, fb.x, fb.y, fb.z, fb.w};
    float v[8][8];  // [row][column]
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      // rows of the next segment that share this tile read as zeros (past the
      // tensor's last row the copy itself fills zeros)
      const uint32_t c = (kSplit && row_base + k >= g.rows) ? 0u : cw[k];
      decode8_scaled(c, __uint_as_float(fr[k]), v[k]);
    }

    // ---- 2. column amax, starting from 0 so that all-NaN columns read 0, as
    // the reference's fmaxf loop does
    uint32_t am[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float m = max3_abs(0.0f, v[0][c], v[1][c]);
      m = max3_abs(m, v[2][c], v[3][c]);
      m = max3_abs(m, v[4][c], v[5][c]);
      m = max3_abs(m, v[6][c], v[7][c]);
      am[c] = __float_as_uint(m);  // a magnitude: integer order is float order
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) am[c] = max(am[c], __shfl_xor_sync(0xffffffffu, am[c], 16));
    if (lane < 16) {
      uint4* pw = reinterpret_cast<uint4*>(part + warp * 128 + wc * 8);
      pw[0] = make_uint4(am[0], am[1], am[2], am[3]);
      pw[1] = make_uint4(am[4], am[5], am[6], am[7]);
    }
    const bool tile_special = __syncthreads_or(special_cur || !ok);
    if (tile_special && *timeout_flag) break;  // a tile never arrived: stop together
    if (t < 128) {
      uint32_t mb = part[t];
#pragma unroll
      for (int j = 1; j < 8; ++j) mb = max(mb, part[j * 128 + t]);
      const float mxv = __uint_as_float(mb);
      float qs;
      if (!kSplit) {
        const float amax = fmaxf(eps, mxv);
        if (t < g.cols) scales_out[g.scale_row * N + g.col0 + t] = amax / 448.0f;
        qs = (amax > 1e-9f) ? (448.0f / amax) : 0.0f;
      } else {
        const float amax = mxv;  // initialised to 0 on the split path
        // s = (float)(1 / (double)x) with x = 2^ceil(log2(amax / 448)) as the
        // float with biased exponent ex (0 or Inf at the ends), and the stored
        // scale 1 / s, which is x again; both from exponent bits, no division
        float s, inv_s;
        if (amax <= eps) {
          s = 1.0f;
          inv_s = 1.0f;
        } else {
          const uint32_t rbits = __float_as_uint(amax / 448.0f);
          uint32_t ex = (rbits >> 23) & 0xFFu;
          if (rbits & 0x7FFFFFu) ex += 1u;
          inv_s = __uint_as_float(ex << 23);  // x: 0 for ex = 0, Inf for ex = 255
          const uint32_t sb = ex == 0u     ? 0x7F800000u             // 1 / 0
                              : ex <= 253u ? (254u - ex) << 23       // 2^(127 - ex), normal
                              : ex == 254u ? 0x00400000u             // 2^-127, subnormal
                                           : 0u;                     // 1 / Inf
          s = __uint_as_float(sb);
        }
        if (t < g.cols) scales_out[g.scale_row * N + g.col0 + t] = inv_s;
        qs = s;
      }
      col_qs[t] = qs;
      // NaN products are possible only with an Inf amax or an E8M0 byte of 255
      col_clamp[t] = (mb >= 0x7F800000u || tile_special) ? 1 : 0;
    }
    __syncthreads();

    // ---- 3. scale, convert row pairs to E4M3, one 8-byte chunk per column.
    // With a finite amax every |v * qs| is at most 448 (1 + 2^-23), which the
    // saturating conversion maps exactly as clamp-then-convert does (true for
    // every finite value), so the clamp is needed only where a NaN can occur:
    // columns with an Inf amax (v * 0) and tiles holding an E8M0 byte of 255
    // (0 * Inf); the reference clamps NaN to -448.
    {
      const float4 qa = *reinterpret_cast<const float4*>(col_qs + wc * 8);
      const float4 qb = *reinterpret_cast<const float4*>(col_qs + wc * 8 + 4);
      const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      const uint2 cl = *reinterpret_cast<const uint2*>(col_clamp + wc * 8);
      const bool clamp = (cl.x | cl.y) != 0u;
      uint8_t* orow = otile + (wc * 8) * 128 + ((rg ^ wc) << 3);
      // column pairs (2j, 2j + 1) of a row are neighbouring decode outputs, so
      // each mul.rn.f32x2 takes them with the pair of column scales as is
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float q[8][2];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mul2_f32_pairs(v[k][2 * j], v[k][2 * j + 1], qv[2 * j], qv[2 * j + 1], q[k][0], q[k][1]);
        if (clamp) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            q[k][0] = fminf(fmaxf(q[k][0], -448.0f), 448.0f);
            q[k][1] = fminf(fmaxf(q[k][1], -448.0f), 448.0f);
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
          *reinterpret_cast<uint2*>(orow + (2 * j + h) * 128) =
              make_uint2(cvt_e4m3x4(q[0][h], q[1][h], q[2][h], q[3][h]),
                         cvt_e4m3x4(q[4][h], q[5][h], q[6][h], q[7][h]));
      }
    }
    // tile i+1's factors into the other buffer (last read in tile i-1's step
    // 1); the barrier below orders these stores before tile i+1's step 1, and
    // steps 1-3 of this tile have covered the scale load's latency
    if (t < 128 && has_next) special_next = colT_factors(sc_next, t, fac + ((i + 1) & 1) * 512);
    __syncthreads();

    // ---- 4. output rows n (128 FP8 bytes each), eight lanes per row: thread t
    // writes chunk p = t % 8 of rows n = 32k + t / 8 (k = 0..3), whose
    // column swizzle x = n / 8 has x & 1 = (t / 64) & 1 and x / 2 = 2k + t / 128
    {
      const int p = t & 7, n0 = t >> 3;
      uint8_t* dst = out + g.out_base + (g.col0 + n0) * g.out_pitch + p * 16;
      const int64_t stride = 32 * g.out_pitch;
      const bool swap = (t >> 6) & 1;
      // block-uniform: full tile, tile origin and row pitch 16-byte aligned (the
      // other path shuffles across lanes and must be taken by whole warps)
      const uintptr_t origin = reinterpret_cast<uintptr_t>(out + g.out_base + g.col0 * g.out_pitch);
      if (g.rows == 128 && g.cols == 128 && ((origin | (uintptr_t)g.out_pitch) & 15) == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int n = 32 * k + n0;
          uint4 o = *reinterpret_cast<const uint4*>(otile + n * 128 + ((p ^ ((2 * k + (t >> 7)) & 7)) << 4));
          if (swap) o = make_uint4(o.z, o.w, o.x, o.y);
          st_stream_v4(dst + k * stride, o);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int n = 32 * k + n0;
          uint4 o = *reinterpret_cast<const uint4*>(otile + n * 128 + ((p ^ ((2 * k + (t >> 7)) & 7)) << 4));
          if (swap) o = make_uint4(o.z, o.w, o.x, o.y);
          const int src = (t & ~7) | ((p + 7) & 7);  // chunk (p-1) mod 8 of the same row
          const uint4 prev = make_uint4(__shfl_sync(0xffffffffu, o.x, src & 31),
                                        __shfl_sync(0xffffffffu, o.y, src & 31),
                                        __shfl_sync(0xffffffffu, o.z, src & 31),
                                        __shfl_sync(0xffffffffu, o.w, src & 31));
          if (n < g.cols && p != 0) store_row_body(dst - p * 16 + k * stride, p, o, prev, g.rows);
        }
        // edge chunks: one thread per output row
        if (t < g.cols) {
          const int n = t;
          auto chunk = [&](int q) {  // data chunk q of staged row n
            uint4 c = *reinterpret_cast<const uint4*>(otile + n * 128 + ((q ^ ((n >> 4) & 7)) << 4));
            if ((n >> 3) & 1) c = make_uint4(c.z, c.w, c.x, c.y);
            return c;
          };
          store_row_edges(out + g.out_base + (g.col0 + n) * g.out_pitch, chunk(7), chunk(0),
                          g.rows, g.merge_in, g.carry_out, carry + n);
        }
      }
    }
    if (!has_next) return;
    // tile i+1 (on the split path rebuilt from its walk position, so that its
    // descriptor is not kept live through the tile: 128 registers with no
    // spills)
    w = wn;
    if constexpr (kSplit) {
      split_tile(w, N, sa, g);
    } else {
      g = gn;
    }
  }
  // Left early (tile `issued - 2` or `issued - 1` never arrived): do not exit
  // while a requested copy may still land in this CTA's memory.
  if (t == 0)
    for (int j = issued >= 2 ? issued - 2 : 0; j < issued; ++j)
      mbar_wait(&full[j & 1], (uint32_t)(j >> 1) & 1u);
}

constexpr size_t kColTSmem = 128 + kColTStages * kColTCodeBytes + 128 * 128 + 8 * 128 * 4 +
                             128 * 4 + 128 + 2 * 512 * 4 + 2 * 8 + 16 + 16 + 128 * 16;

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

// ------------------------------------------------ msplit without allocation
// Scratch of the allocation-free split entry point: split_offsets in words
// [0, kMaxSeg), scale_offsets in [kMaxSeg, 2 kMaxSeg).  32 KiB per device.
constexpr int kMaxSeg = MXB_MSPLIT_MAX_SEGMENTS;
static __device__ __align__(256) int32_t g_msplit_scratch[2 * kMaxSeg];

// One block of 1024 threads: exclusive scans of m_i (row offsets) and of
// ceil(m_i / 128) (scale-row offsets); thread t owns segments 4t .. 4t+3.
__global__ void __launch_bounds__(1024) msplit_offsets_kernel(const int32_t* __restrict__ m_splits,
                                                             int ns, int32_t* __restrict__ so,
                                                             int32_t* __restrict__ sco) {
  __shared__ int32_t warp_rows[32], warp_blocks[32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  int32_t m[4], rows = 0, blocks = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * t + j;
    m[j] = i < ns ? m_splits[i] : 0;
    rows += m[j];
    blocks += (m[j] + 127) / 128;
  }
  // inclusive warp scans, then the warp totals
  int32_t ir = rows, ib = blocks;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t r = __shfl_up_sync(0xffffffffu, ir, o), b = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ir += r;
      ib += b;
    }
  }
  if (lane == 31) {
    warp_rows[warp] = ir;
    warp_blocks[warp] = ib;
  }
  __syncthreads();
  if (warp == 0) {
    int32_t wr = warp_rows[lane], wb = warp_blocks[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t r = __shfl_up_sync(0xffffffffu, wr, o), b = __shfl_up_sync(0xffffffffu, wb, o);
      if (lane >= o) {
        wr += r;
        wb += b;
      }
    }
    warp_rows[lane] = wr - warp_rows[lane];  // exclusive prefix of the warp totals
    warp_blocks[lane] = wb - warp_blocks[lane];
  }
  __syncthreads();
  int32_t r0 = warp_rows[warp] + ir - rows, b0 = warp_blocks[warp] + ib - blocks;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * t + j;
    if (i < ns) {
      so[i] = r0;
      sco[i] = b0;
    }
    r0 += m[j];
    b0 += (m[j] + 127) / 128;
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
  const dim3 grid((unsigned)(M / 128), (unsigned)(Kb / 128));
  fp8_col_kernel<<<grid, kThreads, kColSmem, to_cuda(stream)>>>(
      tmap, (const uint8_t*)input_s, M, Kb, (uint8_t*)output_q, (float*)output_s);
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
  if (!make_tensor_map_2d(&tmap, input, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, N / 2, N / 2, 64, 128))
    return MXB_ERR_CUDA;
  MXB_REQUIRE(cdiv(M, 128) <= INT32_MAX, MXB_ERR_INVALID_ARGUMENT, "mxfp4_to_fp8_colT: M too large");
  const int nb = (int)cdiv(M, 128);
  const int64_t zt = cdiv(N, 128), tiles = zt * nb;
  const int ctas = persistent_ctas((const void*)fp8_colT_kernel<false>, kThreads, kColTSmem);
  fp8_colT_kernel<false><<<(unsigned)min((int64_t)ctas, tiles), kThreads, kColTSmem,
                           to_cuda(stream)>>>(tmap, (const uint8_t*)input_s, M, N, eps,
                                              (uint8_t*)output_q, (float*)output_s,
                                              SplitArgs{nullptr, nullptr, nullptr}, 1, nb, zt);
  return launch_status("mxfp4_to_fp8_colT");
}

// Argument checks shared by both split entry points, so that the no-alloc
// variant rejects a bad call before it touches its shared scratch.  Sets
// *empty when there is nothing to convert (then MXB_OK and no launch).
static mxb_status colT_msplit_check(const void* input, const void* input_s, int64_t total_M,
                                    int64_t N, const void* output_q, const void* output_s,
                                    const int32_t* m_splits, int64_t num_splits,
                                    int64_t max_split_len, bool* empty) {
  *empty = false;
  MXB_REQUIRE(total_M >= 0 && N >= 0 && N % 32 == 0 && num_splits >= 0 && max_split_len >= 0,
              MXB_ERR_INVALID_ARGUMENT, "mxfp4_to_fp8_colT_msplit: need N %% 32 == 0, got %lld",
              (long long)N);
  MXB_REQUIRE(num_splits <= 65535 && cdiv(max_split_len, 128) <= 65535, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT_msplit: too many splits or rows per split");
  if (total_M == 0 || N == 0 || num_splits == 0 || max_split_len == 0) {
    *empty = true;
    return MXB_OK;
  }
  MXB_REQUIRE(input && input_s && output_q && output_s && m_splits, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT_msplit: null pointer");
  MXB_REQUIRE(aligned(input, 16), MXB_ERR_MISALIGNED,
              "mxfp4_to_fp8_colT_msplit: input not 16-byte aligned");
  return MXB_OK;
}

extern "C" mxb_status mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit(
    const void* input, const void* input_s, int64_t total_M, int64_t N, void* output_q,
    void* output_s, const int32_t* m_splits, const int32_t* split_offsets,
    const int32_t* scale_offsets, int64_t num_splits, int64_t max_split_len, float eps,
    mxb_stream_t stream) {
  bool empty = false;
  const mxb_status chk = colT_msplit_check(input, input_s, total_M, N, output_q, output_s, m_splits,
                                           num_splits, max_split_len, &empty);
  if (chk != MXB_OK || empty) return chk;
  MXB_REQUIRE(split_offsets && scale_offsets, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT_msplit: null pointer");
  MXB_REQUIRE(colT_attr(), MXB_ERR_CUDA, "mxfp4_to_fp8_colT_msplit: cannot reserve shared memory");
  CUtensorMap tmap;
  if (!make_tensor_map_2d(&tmap, input, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, total_M, N / 2, N / 2,
                          64, 128))
    return MXB_ERR_CUDA;
  // units of up to kUnitTiles row blocks along each segment
  const int nb = (int)cdiv(cdiv(max_split_len, 128), kUnitTiles);
  const int64_t zt = cdiv(N, 128), tiles = zt * num_splits * nb;
  const int ctas = persistent_ctas((const void*)fp8_colT_kernel<true>, kThreads, kColTSmem);
  fp8_colT_kernel<true><<<(unsigned)min((int64_t)ctas, tiles), kThreads, kColTSmem,
                          to_cuda(stream)>>>(tmap, (const uint8_t*)input_s, total_M, N, eps,
                                             (uint8_t*)output_q, (float*)output_s,
                                             SplitArgs{m_splits, split_offsets, scale_offsets},
                                             (int)num_splits, nb, zt);
  return launch_status("mxfp4_to_fp8_colT_msplit");
}

// Device address of g_msplit_scratch, looked up once per device with that
// device current (a module's __device__ arrays exist once per device).
static int32_t* msplit_scratch() {
  static std::mutex mu;
  static int32_t* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_msplit_scratch) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<int32_t*>(p);
  }
  return addr[dev];
}

extern "C" mxb_status mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit_noalloc(
    const void* input, const void* input_s, int64_t total_M, int64_t N, void* output_q,
    void* output_s, const int32_t* m_splits, int64_t num_splits, int64_t max_split_len, float eps,
    mxb_stream_t stream) {
  MXB_REQUIRE(num_splits >= 0 && num_splits <= kMaxSeg, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT_msplit_noalloc: num_splits = %lld exceeds the %d segments of "
              "the static scratch (use mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit)",
              (long long)num_splits, kMaxSeg);
  MXB_REQUIRE(total_M >= 0 && total_M <= INT32_MAX && max_split_len >= 0, MXB_ERR_INVALID_ARGUMENT,
              "mxfp4_to_fp8_colT_msplit_noalloc: need 0 <= total_M <= 2^31-1 and max_split_len >= 0");
  bool empty = false;
  const mxb_status chk = colT_msplit_check(input, input_s, total_M, N, output_q, output_s, m_splits,
                                           num_splits, max_split_len, &empty);
  if (chk != MXB_OK || empty) return chk;
  int32_t* scratch = msplit_scratch();
  MXB_REQUIRE(scratch, MXB_ERR_CUDA,
              "mxfp4_to_fp8_colT_msplit_noalloc: cannot look up the static scratch (%s)",
              cudaGetErrorString(cudaGetLastError()));
  msplit_offsets_kernel<<<1, 1024, 0, to_cuda(stream)>>>(m_splits, (int)num_splits, scratch,
                                                         scratch + kMaxSeg);
  const mxb_status st = launch_status("mxfp4_to_fp8_colT_msplit_noalloc (offsets)");
  if (st != MXB_OK) return st;
  return mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit(input, input_s, total_M, N, output_q, output_s,
                                                     m_splits, scratch, scratch + kMaxSeg,
                                                     num_splits, max_split_len, eps, stream);
}
