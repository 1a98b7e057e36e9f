// Fused MoE dispatch / combine over NVLink peer memory (sm_100a, one process
// per GPU, buffers mapped with CUDA IPC).  The quantize of a token and its
// transfer are one kernel: each CTA quantizes a token row once and stores the
// wire row straight into the receive buffer of every destination GPU, so the
// NVLink traffic overlaps the math token by token.  The expert stage writes
// each output row straight back into its source GPU's combine buffer, and the
// combine sums a token's returned rows locally.
//
// Every rank allocates one buffer with the layout of mxb_ep_layout (offsets in
// bytes, all 256-byte aligned):
//   sig   uint32 [G]            epoch flags written by the peers
//   cnt   int32  [2][G][G]      cnt[p][s][g] = rows rank s sends to rank g in a
//                               step of parity p (double buffered across steps)
//   wire  uint8  [G*Tcap][RB]   received wire rows codes[H/2] || scales[H/32],
//                               grouped by source rank, token order within
//   meta  int32  [G*Tcap][2k]   per received row: destination-local expert ids
//                               (-1 if the expert is elsewhere) and weights
//   back  bf16   [G*Tcap][H]    expert rows returned to this rank, indexed by
//                               this rank's send slot
// Peer access is plain ld/st to addresses from cudaIpcOpenMemHandle (no
// multicast object, no TMA on peer memory).  Cross-GPU waits are bounded: a
// wait that gives up counts a timeout (mxb_ep_wait_timeouts) and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "capi_util.h"
#include "common.cuh"
#include "qrow.cuh"

namespace mxb {
namespace {

static __device__ unsigned int g_ep_timeouts;
constexpr uint32_t kPeerSpins = 1u << 22;  // default polls of ~64 ns sleep each
// Polls a cross-GPU wait makes before it gives up (mxb_ep_set_wait_polls).
static __device__ uint32_t g_ep_wait_polls = kPeerSpins;
constexpr int kP2PThreads = 256;
constexpr int kMaxScaleBytes = 2048;  // H / 32 for H <= 65536
constexpr int kMaxMetaInts = 512;     // 2 * world * topk for world * topk <= 256

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint8_t* peer(const uint64_t* bases, int p) {
  return reinterpret_cast<uint8_t*>(bases[p]);
}

__device__ __forceinline__ const int32_t* cnt_of(const uint64_t* bases, const mxb_ep_layout& L,
                                                 int parity) {
  return reinterpret_cast<const int32_t*>(peer(bases, L.rank) + L.cnt_off) +
         (int64_t)parity * L.world * L.world;
}

// Signals every peer that this rank reached `epoch`, then waits until every
// peer has signalled it.  Called by one full warp; lane p handles peer p.
__device__ void barrier_warp(const uint64_t* bases, const mxb_ep_layout& L, uint32_t epoch) {
  const int p = threadIdx.x & 31;
  __threadfence_system();
  __syncwarp();
  for (int q = p; q < L.world; q += 32)
    st_release_sys(reinterpret_cast<uint32_t*>(peer(bases, q) + L.sig_off) + L.rank, epoch);
  for (int q = p; q < L.world; q += 32) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(peer(bases, L.rank) + L.sig_off) + q;
    const uint32_t limit = g_ep_wait_polls;
    uint32_t i = 0;
    while (ld_acquire_sys(mine) < epoch) {
      if (++i >= limit) {
        atomicAdd(&g_ep_timeouts, 1u);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
}

__global__ void ep_counts_kernel(const uint64_t* __restrict__ bases, mxb_ep_layout L,
                                 const int32_t* __restrict__ send_counts, int parity,
                                 uint32_t epoch) {
  // this rank's row of the count matrix -> every rank's copy
  for (int i = threadIdx.x; i < L.world * L.world; i += blockDim.x) {
    const int p = i / L.world, g = i - p * L.world;
    int32_t* c = reinterpret_cast<int32_t*>(peer(bases, p) + L.cnt_off) +
                 ((int64_t)parity * L.world + L.rank) * L.world + g;
    *c = send_counts[g];
  }
  __syncthreads();
  if (threadIdx.x < 32) barrier_warp(bases, L, epoch);
}

__global__ void ep_barrier_kernel(const uint64_t* __restrict__ bases, mxb_ep_layout L,
                                  uint32_t epoch) {
  if (threadIdx.x < 32) barrier_warp(bases, L, epoch);
}

// Q-row of one 32-element block held by 4 consecutive lanes, 8 elements each,
// with the quantizers' scale rule and rounding (qrow.cuh): fast path, or the
// literal reference formula for blocks with Inf/NaN.  Returns this lane's 8
// codes; `byte` is the block's E8M0 scale (same in the 4 lanes).  The 4 lanes
// take the same branch, so the shuffles name only their quad.
__device__ __forceinline__ uint32_t p2p_quant_quad(const uint4 a, uint32_t& byte) {
  const unsigned qmask = 0xFu << (threadIdx.x & 28);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) m = vmax_u16x2(m, w[i] & 0x7FFF7FFFu);
  m = vmax_u16x2(m, __shfl_xor_sync(qmask, m, 1));
  m = vmax_u16x2(m, __shfl_xor_sync(qmask, m, 2));
  const uint32_t mb = max(m & 0xFFFFu, m >> 16);
  if (mb < 0x7F80u) {
    uint32_t inv;
    scale_fast(mb, byte, inv);
    return encode8_pairs(w, inv);
  }
  const QuantParams p{1e-10f, -6.0f, 6.0f};
  uint32_t f[8];
  unpack8(w, f);
  float am = amax_generic(f, p.eps);
  am = fmaxf(am, __shfl_xor_sync(qmask, am, 1));
  am = fmaxf(am, __shfl_xor_sync(qmask, am, 2));
  float inv;
  scale_generic(am, p, inv, byte);
  return encode8_generic(f, inv, p);
}

constexpr int kP2PWarps = kP2PThreads / 32;
constexpr int kDispatchBatch = 4;  // 256-element steps per batch: 4 loads in flight per lane

// One warp per token (grid-stride): quantize the row once, store its wire row
// and routing metadata into every destination's receive buffer.  A step of
// 256 elements is 8 blocks, 4 lanes per block; a batch of 4 steps gives 512
// bytes of codes, staged in shared memory so that every lane stores 16 bytes
// per destination.
__global__ void __launch_bounds__(kP2PThreads) ep_dispatch_p2p_kernel(
    const uint8_t* __restrict__ x, int64_t T, const int32_t* __restrict__ within,
    const int64_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
    const uint64_t* __restrict__ bases, mxb_ep_layout L, int parity) {
  __shared__ __align__(16) uint8_t scale_bytes[kP2PWarps][kMaxScaleBytes];
  __shared__ __align__(16) uint32_t stage[kP2PWarps][32 * kDispatchBatch];
  __shared__ int64_t dst_row[kP2PWarps][32];
  __shared__ __align__(16) int32_t meta_rows[kP2PWarps][kMaxMetaInts];
  const int G = L.world, H = L.hidden, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t rb = H / 2 + H / 32;
  const int steps = H / 256;  // H is a multiple of 512
  const int32_t* cnt = cnt_of(bases, L, parity);
  int64_t off = 0;  // lane g < G: rows that lower ranks send to g come first
  if (lane < G)
    for (int s = 0; s < L.rank; ++s) off += cnt[s * G + lane];
  uint8_t* sb = scale_bytes[warp];
  uint32_t* st = stage[warp];
  int64_t* dr = dst_row[warp];
  for (int64_t t = (int64_t)blockIdx.x * kP2PWarps + warp; t < T;
       t += (int64_t)gridDim.x * kP2PWarps) {
    const uint8_t* xr = x + t * H * 2;
    if (lane < G) {
      const int32_t wi = within[t * G + lane];
      dr[lane] = wi < 0 ? -1 : off + wi;
    }
    __syncwarp();
    for (int s0 = 0; s0 < steps; s0 += kDispatchBatch) {
      uint4 a[kDispatchBatch];
#pragma unroll
      for (int u = 0; u < kDispatchBatch; ++u)
        if (s0 + u < steps) a[u] = ld_stream_v4(xr + ((int64_t)(s0 + u) * 256 + lane * 8) * 2);
#pragma unroll
      for (int u = 0; u < kDispatchBatch; ++u) {
        if (s0 + u >= steps) continue;
        uint32_t byte;
        st[u * 32 + lane] = p2p_quant_quad(a[u], byte);
        if ((lane & 3) == 0) sb[(s0 + u) * 8 + (lane >> 2)] = (uint8_t)byte;
      }
      __syncwarp();
      const int nbytes = min(kDispatchBatch, steps - s0) * 128;
      if (lane * 16 < nbytes) {
        const uint4 v = reinterpret_cast<const uint4*>(st)[lane];
        for (int g = 0; g < G; ++g) {
          const int64_t r = dr[g];
          if (r < 0) continue;
          uint8_t* row = peer(bases, g) + L.wire_off + r * rb;
          *reinterpret_cast<uint4*>(row + (int64_t)s0 * 128 + lane * 16) = v;
        }
      }
      __syncwarp();
    }
    // the row's scale bytes as 16-byte stores (H / 32 is a multiple of 16)
    const int nv = H / 512;
    for (int i = lane; i < G * nv; i += 32) {
      const int g = i / nv, q = i - g * nv;
      const int64_t r = dr[g];
      if (r < 0) continue;
      uint8_t* row = peer(bases, g) + L.wire_off + r * rb;
      *reinterpret_cast<uint4*>(row + H / 2 + q * 16) =
          *reinterpret_cast<const uint4*>(sb + q * 16);
    }
    // routing metadata, one row of 2 * topk words per destination: expert ids
    // local to the destination (or -1), then weights (or 0).  Rows are built in
    // shared memory and leave as 16-byte stores when 2 * topk is a multiple of
    // 4 (word stores otherwise), so that NVLink carries few small writes.
    const int mrow = 2 * L.topk;
    int32_t* mr = meta_rows[warp];
    for (int i = lane; i < G * L.topk; i += 32) {
      const int g = i / L.topk, j = i - g * L.topk;
      if (dr[g] < 0) continue;
      const int64_t e = topk_idx[t * L.topk + j];
      // e / experts_per_rank == g (C division) without a 64-bit division
      const int64_t lo = (int64_t)g * L.experts_per_rank;
      const bool here = e >= 0 ? (e >= lo && e < lo + L.experts_per_rank)
                               : (g == 0 && e > -(int64_t)L.experts_per_rank);
      mr[g * mrow + j] = here ? (int32_t)(e - lo) : -1;
      mr[g * mrow + L.topk + j] = __float_as_int(here ? topk_w[t * L.topk + j] : 0.0f);
    }
    __syncwarp();
    const int wpp = (mrow & 3) == 0 ? 4 : 1;  // words per store
    const int pieces = mrow / wpp;
    for (int i = lane; i < G * pieces; i += 32) {
      const int g = i / pieces, q = i - g * pieces;
      const int64_t r = dr[g];
      if (r < 0) continue;
      int32_t* m = reinterpret_cast<int32_t*>(peer(bases, g) + L.meta_off) + r * mrow + q * wpp;
      if (wpp == 4)
        *reinterpret_cast<int4*>(m) = *reinterpret_cast<const int4*>(mr + g * mrow + q * 4);
      else
        *m = mr[g * mrow + q];
    }
    __syncwarp();
  }
  __threadfence_system();
}

constexpr int kReturnBatch = 4;  // chunks per lane with their loads issued together

// Expert stage + return: for every received row r (source s, i-th row from s),
// y = user row y_in[r] if given, else the routing-weighted identity expert
// bf16(bf16(dequant(wire[r])) * sum_j weight[r][j]); the row is stored into
// source s's `back` buffer at s's send slot sum_{g < rank} cnt[s][g] + i.
// One warp per row; lane l handles the 8-element chunks l, l + 32, ...
// Rows are visited source-minor (i -> j = i / G, s = i % G) so that at any
// moment the warps write to every source, local HBM and NVLink together.
__global__ void __launch_bounds__(kP2PThreads) ep_return_p2p_kernel(
    const uint8_t* __restrict__ y_in, const uint64_t* __restrict__ bases, mxb_ep_layout L,
    int parity) {
  __shared__ int32_t col[64];       // cnt[s][rank]
  __shared__ int64_t start[64];     // sum_{q < s} cnt[q][rank]
  __shared__ int64_t back_off[64];  // sum_{g < rank} cnt[s][g]
  const int G = L.world, H = L.hidden, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t rb = H / 2 + H / 32;
  const int32_t* cnt = cnt_of(bases, L, parity);
  if (threadIdx.x < G) {
    const int s = threadIdx.x;
    col[s] = cnt[s * G + L.rank];
    int64_t o = 0, st = 0;
    for (int g = 0; g < L.rank; ++g) o += cnt[s * G + g];
    for (int q = 0; q < s; ++q) st += cnt[q * G + L.rank];
    back_off[s] = o;
    start[s] = st;
  }
  __syncthreads();
  int64_t cmax = 0;
  for (int s = 0; s < G; ++s) cmax = max(cmax, (int64_t)col[s]);
  const uint8_t* wire = peer(bases, L.rank) + L.wire_off;
  const int32_t* meta = reinterpret_cast<const int32_t*>(peer(bases, L.rank) + L.meta_off);
  const int chunks = H / 8;  // a multiple of 64
  for (int64_t i = (int64_t)blockIdx.x * kP2PWarps + warp; i < cmax * G;
       i += (int64_t)gridDim.x * kP2PWarps) {
    const int s = (int)(i % G);
    const int64_t j = i / G;
    if (j >= col[s]) continue;
    const int64_t r = start[s] + j;
    uint8_t* out = peer(bases, s) + L.back_off + (back_off[s] + j) * H * 2;
    if (y_in) {
      const uint8_t* yr = y_in + r * H * 2;
      for (int c0 = lane; c0 < chunks; c0 += 32 * kReturnBatch) {
        uint4 v[kReturnBatch];
#pragma unroll
        for (int u = 0; u < kReturnBatch; ++u)
          if (c0 + 32 * u < chunks) v[u] = *reinterpret_cast<const uint4*>(yr + (c0 + 32 * u) * 16);
#pragma unroll
        for (int u = 0; u < kReturnBatch; ++u)
          if (c0 + 32 * u < chunks) *reinterpret_cast<uint4*>(out + (c0 + 32 * u) * 16) = v[u];
      }
      continue;
    }
    // lane j loads weight j; the sum keeps the order j = 0, 1, ...
    const int32_t* m = meta + r * 2 * L.topk;
    const float wj = lane < L.topk ? __int_as_float(m[L.topk + lane]) : 0.0f;
    float wsum = __shfl_sync(0xffffffffu, wj, 0);
    for (int q = 1; q < L.topk; ++q) wsum += __shfl_sync(0xffffffffu, wj, q);
    const uint8_t* row = wire + r * rb;
    for (int c0 = lane; c0 < chunks; c0 += 32 * kReturnBatch) {
      uint32_t wv[kReturnBatch], ev[kReturnBatch];
#pragma unroll
      for (int u = 0; u < kReturnBatch; ++u) {
        const int c = c0 + 32 * u;
        if (c < chunks) {
          wv[u] = *reinterpret_cast<const uint32_t*>(row + c * 4);
          ev[u] = row[H / 2 + (c >> 2)];
        }
      }
#pragma unroll
      for (int u = 0; u < kReturnBatch; ++u) {
        const int c = c0 + 32 * u;
        if (c >= chunks) continue;
        const uint32_t w = wv[u], e = ev[u];
        uint32_t o[4];
        e2m1x4_to_bf16x4(w, o[0], o[1]);
        e2m1x4_to_bf16x4(w >> 16, o[2], o[3]);
        if (e - 2u <= 252u) {
          const uint32_t s2 = (e << 7) | (e << 23);
#pragma unroll
          for (int q = 0; q < 4; ++q) o[q] = mul_bf16x2(o[q], s2);
        } else {
          const float sc = e8m0_to_f(e);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            o[q] = cvt_bf16x2(bf16lo_to_f(o[q]) * sc, bf16hi_to_f(o[q]) * sc);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          o[q] = cvt_bf16x2(bf16lo_to_f(o[q]) * wsum, bf16hi_to_f(o[q]) * wsum);
        *reinterpret_cast<uint4*>(out + c * 16) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  __threadfence_system();
}

// Destination rank of expert id e, or -1 when e / experts_per_rank (C
// division) lies outside [0, G).
__device__ __forceinline__ int route_rank(int64_t e, int experts_per_rank, int G) {
  const int64_t q = (e >= 0 && e <= 0x7FFFFFFFLL)
                        ? (int64_t)((uint32_t)e / (uint32_t)experts_per_rank)
                        : e / experts_per_rank;
  return q >= 0 && q < G ? (int)q : -1;
}

// Mask of the destination ranks of token t (bit g set if any of its k experts
// lives on rank g), with 8 id loads in flight.
__device__ __forceinline__ uint64_t route_mask(const int64_t* __restrict__ topk_idx, int64_t t,
                                               int k, int experts_per_rank, int G) {
  const int64_t* p = topk_idx + t * k;
  uint64_t mask = 0;
  for (int j0 = 0; j0 < k; j0 += 8) {
    int64_t e[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) e[u] = j0 + u < k ? p[j0 + u] : -1;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = j0 + u < k ? route_rank(e[u], experts_per_rank, G) : -1;
      if (q >= 0) mask |= 1ull << q;
    }
  }
  return mask;
}

// Routing without host synchronisation, in two launches over tiles of
// kRouteTile tokens (one token per thread).
//   ep_route_tile_kernel: within[t, g] = token t's index among the tokens of
//     its tile routed to rank g (ballot per rank, then a scan over the tile's
//     warps), -1 if t does not go to g.  The tile's last token carries the
//     tile's count c for every rank it does not go to, as -(c + 2), so the
//     count of every tile can be read back from that one row (c = w + 1 for
//     w >= 0, -w - 2 otherwise).
//   ep_route_prefix_kernel (one CTA): reads every tile's counts, turns them
//     into per-rank prefixes, adds each tile's prefix to its entries, restores
//     -1 and writes send_counts[g] = number of tokens routed to g.  T * G
//     entries are small next to the expert ids the first launch reads.
// The result: within[t, g] is t's index among all tokens routed to g, in
// token order.
constexpr int kRouteTile = 256;
constexpr int kRouteThreads = 1024;
constexpr int kRouteMaxEntries = 16384;  // tiles * G held in shared memory (64 KB)
constexpr int kRouteUnroll = 8;          // 16-byte groups per thread in flight (prefix pass)

__global__ void __launch_bounds__(kRouteTile) ep_route_tile_kernel(
    const int64_t* __restrict__ topk_idx, int64_t T, int k, int experts_per_rank, int G,
    int32_t* __restrict__ within) {
  __shared__ int32_t warp_base[kRouteTile / 32][64];
  const int t0 = threadIdx.x, lane = t0 & 31, warp = t0 >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int64_t base = (int64_t)blockIdx.x * kRouteTile, t = base + t0;
  const int64_t last = min(T, base + kRouteTile) - 1;
  const uint64_t mask = t < T ? route_mask(topk_idx, t, k, experts_per_rank, G) : 0;
  for (int g = 0; g < G; ++g) {
    const uint32_t b = __ballot_sync(0xffffffffu, (mask >> g) & 1);
    if (lane == 0) warp_base[warp][g] = __popc(b);
  }
  __syncthreads();
  if (t0 < G) {  // exclusive scan over the warps, per rank
    int32_t acc = 0;
    for (int w = 0; w < kRouteTile / 32; ++w) {
      const int32_t v = warp_base[w][t0];
      warp_base[w][t0] = acc;
      acc += v;
    }
  }
  __syncthreads();
  for (int g = 0; g < G; ++g) {
    const uint32_t b = __ballot_sync(0xffffffffu, (mask >> g) & 1);
    if (t > last) continue;
    const bool hit = (mask >> g) & 1;
    const int32_t idx = warp_base[warp][g] + __popc(b & lt_mask);
    // for the last token, idx + hit is the tile's count for g
    within[t * G + g] = hit ? idx : (t == last ? -(idx + 2) : -1);
  }
}

__global__ void __launch_bounds__(kRouteThreads) ep_route_prefix_kernel(
    int64_t T, int G, int tiles, int32_t* __restrict__ within, int32_t* __restrict__ send_counts) {
  extern __shared__ int32_t pref[];  // [tiles][G]: counts, then exclusive prefixes
  for (int i = threadIdx.x; i < tiles * G; i += kRouteThreads) {
    const int q = i / G, g = i - q * G;
    const int64_t last = min(T, (int64_t)(q + 1) * kRouteTile) - 1;
    const int32_t w = within[last * G + g];
    pref[i] = w >= 0 ? w + 1 : -w - 2;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    int32_t acc = 0;
    for (int q = 0; q < tiles; ++q) {
      const int32_t c = pref[q * G + g];
      pref[q * G + g] = acc;
      acc += c;
    }
    send_counts[g] = acc;
  }
  __syncthreads();
  // Rewrite as 16-byte groups of 4 entries, kRouteUnroll groups per thread in
  // flight (a tile's 256 * G entries are a multiple of 4, so a group never
  // straddles two tiles); the ragged end, or a within[] that is not 16-byte
  // aligned, entry by entry.
  const uint32_t n = (uint32_t)(T * G), row_elems = (uint32_t)(kRouteTile * G);
  const uint32_t n4 = (reinterpret_cast<uintptr_t>(within) & 15) == 0 ? n / 4 : 0;
  int4* w4 = reinterpret_cast<int4*>(within);
  for (uint32_t j0 = threadIdx.x; j0 < n4; j0 += kRouteUnroll * kRouteThreads) {
    int4 v[kRouteUnroll];
#pragma unroll
    for (int u = 0; u < kRouteUnroll; ++u) {
      const uint32_t j = j0 + u * kRouteThreads;
      if (j < n4) v[u] = w4[j];
    }
#pragma unroll
    for (int u = 0; u < kRouteUnroll; ++u) {
      const uint32_t j = j0 + u * kRouteThreads;
      if (j < n4) {
        const uint32_t i = 4 * j;
        const int32_t* pq = pref + (i / row_elems) * G;
        const uint32_t g0 = i % (uint32_t)G, g1 = g0 + 1 == (uint32_t)G ? 0 : g0 + 1,
                       g2 = g1 + 1 == (uint32_t)G ? 0 : g1 + 1,
                       g3 = g2 + 1 == (uint32_t)G ? 0 : g2 + 1;
        w4[j] = make_int4(v[u].x >= 0 ? v[u].x + pq[g0] : -1, v[u].y >= 0 ? v[u].y + pq[g1] : -1,
                          v[u].z >= 0 ? v[u].z + pq[g2] : -1, v[u].w >= 0 ? v[u].w + pq[g3] : -1);
      }
    }
  }
  for (uint32_t i = 4 * n4 + threadIdx.x; i < n; i += kRouteThreads) {
    const uint32_t q = i / row_elems, g = i % (uint32_t)G;
    const int32_t w = within[i];
    within[i] = w >= 0 ? w + pref[q * G + g] : -1;
  }
}

// Fallback for more than kRouteMaxEntries tile counts: one CTA walks the
// tokens in order with a running per-rank count.

__global__ void __launch_bounds__(kRouteThreads) ep_route_serial_kernel(
    const int64_t* __restrict__ topk_idx, int64_t T, int k, int experts_per_rank, int G,
    int32_t* __restrict__ within, int32_t* __restrict__ send_counts) {
  __shared__ int32_t warp_base[kRouteThreads / 32][64];
  __shared__ int32_t run[64];
  const int t0 = threadIdx.x, lane = t0 & 31, warp = t0 >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  if (t0 < G) run[t0] = 0;
  for (int64_t base = 0; base < T; base += kRouteThreads) {
    const int64_t t = base + t0;
    const uint64_t mask = t < T ? route_mask(topk_idx, t, k, experts_per_rank, G) : 0;
    for (int g = 0; g < G; ++g) {
      const uint32_t b = __ballot_sync(0xffffffffu, (mask >> g) & 1);
      if (lane == 0) warp_base[warp][g] = __popc(b);
    }
    __syncthreads();
    if (t0 < G) {
      int32_t acc = run[t0];
      for (int w = 0; w < kRouteThreads / 32; ++w) {
        const int32_t v = warp_base[w][t0];
        warp_base[w][t0] = acc;
        acc += v;
      }
      run[t0] = acc;
    }
    __syncthreads();
    for (int g = 0; g < G; ++g) {
      const uint32_t b = __ballot_sync(0xffffffffu, (mask >> g) & 1);
      if (t < T)
        within[t * G + g] = ((mask >> g) & 1) ? warp_base[warp][g] + __popc(b & lt_mask) : -1;
    }
    __syncthreads();
  }
  if (t0 < G) send_counts[t0] = run[t0];
}

// Local combine of the rows returned to this rank: out[t] = bf16(sum over g of
// float(back[slot(t, g)])), slot(t, g) = sum_{g' < g} send_counts[g'] + within[t, g],
// the sum in the order g = 0, 1, ...  One warp per (token, segment of 128
// 8-element chunks); lane l handles the chunks l, l + 32, l + 64, l + 96 of
// the segment, with their 4 loads of a source issued together.  Sources that
// sent the token nothing are skipped (a warp-uniform test).
constexpr int kCombineBatch = 4;

__global__ void __launch_bounds__(kP2PThreads, 4) ep_p2p_combine_kernel(
    const uint8_t* __restrict__ back, int64_t T, int64_t H, const int32_t* __restrict__ within,
    const int32_t* __restrict__ send_counts, int G, uint8_t* __restrict__ out) {
  __shared__ int64_t off[64];
  if (threadIdx.x == 0) {
    int64_t o = 0;
    for (int g = 0; g < G; ++g) {
      off[g] = o;
      o += send_counts[g];
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t chunks = H / 8, segs = (chunks + 32 * kCombineBatch - 1) / (32 * kCombineBatch);
  for (int64_t i = (int64_t)blockIdx.x * kP2PWarps + warp; i < T * segs;
       i += (int64_t)gridDim.x * kP2PWarps) {
    const int64_t t = i / segs, c0 = (i - t * segs) * 32 * kCombineBatch + lane;
    auto slot = [&](int g) -> int64_t {  // the row of source g, or -1
      const int32_t wi = within[t * G + g];
      return wi < 0 ? -1 : off[g] + wi;
    };
    const int64_t my_slot = lane < G ? slot(lane) : -1;
    float acc[kCombineBatch][8];
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u)
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[u][q] = 0.0f;
    for (int g = 0; g < G; ++g) {
      const int64_t sl = g < 32 ? __shfl_sync(0xffffffffu, my_slot, g) : slot(g);
      if (sl < 0) continue;
      const uint8_t* src = back + sl * H * 2;
      uint4 v[kCombineBatch];
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u)
        if (c0 + 32 * u < chunks) v[u] = *reinterpret_cast<const uint4*>(src + (c0 + 32 * u) * 16);
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        if (c0 + 32 * u >= chunks) continue;
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[u][2 * q] += bf16lo_to_f(w[q]);
          acc[u][2 * q + 1] += bf16hi_to_f(w[q]);
        }
      }
    }
    uint8_t* o = out + t * H * 2;
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      if (c0 + 32 * u >= chunks) continue;
      *reinterpret_cast<uint4*>(o + (c0 + 32 * u) * 16) =
          make_uint4(cvt_bf16x2(acc[u][0], acc[u][1]), cvt_bf16x2(acc[u][2], acc[u][3]),
                     cvt_bf16x2(acc[u][4], acc[u][5]), cvt_bf16x2(acc[u][6], acc[u][7]));
    }
  }
}

using PFN_getAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_getAddressRange address_range_fn() {
  static PFN_getAddressRange fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_getAddressRange>(p);
  }();
  return fn;
}

// CTAs for `items` warp-sized work items: one per item up to 8 CTAs per SM.
int p2p_grid(int64_t items) {
  const int64_t ctas = (items + kP2PWarps - 1) / kP2PWarps;
  return (int)(ctas < 148LL * 8 ? (ctas > 0 ? ctas : 1) : 148LL * 8);
}

mxb_status check_layout(const mxb_ep_layout* L, const char* what) {
  MXB_REQUIRE(L && L->world >= 1 && L->world <= 32 && L->rank >= 0 && L->rank < L->world &&
                  L->topk >= 1 && L->topk <= 32 && L->world * L->topk <= 256 &&
                  L->hidden % 512 == 0 && L->hidden > 0 && L->hidden <= 32 * kMaxScaleBytes &&
                  L->experts_per_rank >= 1,
              MXB_ERR_INVALID_ARGUMENT, "%s: invalid layout", what);
  return MXB_OK;
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_ep_layout_init(int32_t world, int32_t rank, int64_t tcap, int32_t hidden,
                                         int32_t topk, int32_t experts_per_rank,
                                         mxb_ep_layout* L, int64_t* total_bytes) {
  MXB_REQUIRE(L && total_bytes && tcap > 0, MXB_ERR_INVALID_ARGUMENT, "ep_layout_init: bad args");
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  L->world = world;
  L->rank = rank;
  L->topk = topk;
  L->hidden = hidden;
  L->experts_per_rank = experts_per_rank;
  L->tcap = tcap;
  const int64_t rows = (int64_t)world * tcap;
  int64_t o = 0;
  L->sig_off = o;
  o = up(o + 4LL * world);
  L->cnt_off = o;
  o = up(o + 4LL * 2 * world * world);
  L->wire_off = o;
  o = up(o + rows * (hidden / 2 + hidden / 32));
  L->meta_off = o;
  o = up(o + rows * 2 * topk * 4);
  L->back_off = o;
  o = up(o + rows * hidden * 2);
  *total_bytes = o;
  return check_layout(L, "ep_layout_init");
}

extern "C" mxb_status mxb_ipc_export(const void* ptr, void* handle64, int64_t* offset) {
  MXB_REQUIRE(ptr && handle64 && offset, MXB_ERR_INVALID_ARGUMENT, "ipc_export: null pointer");
  auto fn = address_range_fn();
  MXB_REQUIRE(fn, MXB_ERR_CUDA, "ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  MXB_REQUIRE(fn(&base, &size, (CUdeviceptr)ptr) == CUDA_SUCCESS, MXB_ERR_CUDA,
              "ipc_export: cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "ipc_export: %s", cudaGetErrorString(e));
  memcpy(handle64, &h, sizeof(h));
  *offset = (int64_t)((CUdeviceptr)ptr - base);
  return MXB_OK;
}

extern "C" mxb_status mxb_ipc_import(const void* handle64, int64_t offset, void** ptr) {
  MXB_REQUIRE(handle64 && ptr, MXB_ERR_INVALID_ARGUMENT, "ipc_import: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "ipc_import: %s", cudaGetErrorString(e));
  *ptr = static_cast<uint8_t*>(base) + offset;
  return MXB_OK;
}

extern "C" mxb_status mxb_ipc_close(void* ptr, int64_t offset) {
  MXB_REQUIRE(ptr, MXB_ERR_INVALID_ARGUMENT, "ipc_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(e));
  return MXB_OK;
}

extern "C" mxb_status mxb_ep_p2p_counts(const uint64_t* bases, const mxb_ep_layout* L,
                                        const int32_t* send_counts, int parity, uint32_t epoch,
                                        mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_p2p_counts");
  mxb_status st = check_layout(L, "ep_p2p_counts");
  if (st != MXB_OK) return st;
  MXB_REQUIRE(bases && send_counts, MXB_ERR_INVALID_ARGUMENT, "ep_p2p_counts: null pointer");
  ep_counts_kernel<<<1, 128, 0, to_cuda(stream)>>>(bases, *L, send_counts, parity & 1, epoch);
  return launch_status("ep_p2p_counts");
}

extern "C" mxb_status mxb_ep_p2p_dispatch(const void* x, int64_t T, const int32_t* within,
                                          const int64_t* topk_idx, const float* topk_w,
                                          const uint64_t* bases, const mxb_ep_layout* L,
                                          int parity, mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_p2p_dispatch");
  mxb_status st = check_layout(L, "ep_p2p_dispatch");
  if (st != MXB_OK) return st;
  MXB_REQUIRE(T >= 0 && T <= L->tcap, MXB_ERR_INVALID_ARGUMENT,
              "ep_p2p_dispatch: T=%lld exceeds the buffer capacity %lld", (long long)T,
              (long long)L->tcap);
  if (T == 0) return MXB_OK;
  MXB_REQUIRE(x && within && topk_idx && topk_w && bases, MXB_ERR_INVALID_ARGUMENT,
              "ep_p2p_dispatch: null pointer");
  MXB_REQUIRE(aligned(x, 16), MXB_ERR_MISALIGNED, "ep_p2p_dispatch: x not 16-byte aligned");
  ep_dispatch_p2p_kernel<<<p2p_grid(T), kP2PThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)x, T, within, topk_idx, topk_w, bases, *L, parity & 1);
  return launch_status("ep_p2p_dispatch");
}

extern "C" mxb_status mxb_ep_p2p_barrier(const uint64_t* bases, const mxb_ep_layout* L,
                                         uint32_t epoch, mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_p2p_barrier");
  mxb_status st = check_layout(L, "ep_p2p_barrier");
  if (st != MXB_OK) return st;
  MXB_REQUIRE(bases, MXB_ERR_INVALID_ARGUMENT, "ep_p2p_barrier: null pointer");
  ep_barrier_kernel<<<1, 32, 0, to_cuda(stream)>>>(bases, *L, epoch);
  return launch_status("ep_p2p_barrier");
}

extern "C" mxb_status mxb_ep_p2p_return(const void* y, const uint64_t* bases,
                                        const mxb_ep_layout* L, int parity, mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_p2p_return");
  mxb_status st = check_layout(L, "ep_p2p_return");
  if (st != MXB_OK) return st;
  MXB_REQUIRE(bases, MXB_ERR_INVALID_ARGUMENT, "ep_p2p_return: null pointer");
  MXB_REQUIRE(!y || aligned(y, 16), MXB_ERR_MISALIGNED, "ep_p2p_return: y not 16-byte aligned");
  ep_return_p2p_kernel<<<p2p_grid((int64_t)L->world * L->tcap), kP2PThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)y, bases, *L, parity & 1);
  return launch_status("ep_p2p_return");
}

extern "C" mxb_status mxb_ep_route(const int64_t* topk_idx, int64_t T, int32_t topk,
                                   int32_t experts_per_rank, int32_t world, int32_t* within,
                                   int32_t* send_counts, mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_route");
  MXB_REQUIRE(T >= 0 && topk >= 1 && topk <= 1024 && experts_per_rank >= 1 && world >= 1 &&
                  world <= 64,
              MXB_ERR_INVALID_ARGUMENT, "ep_route: bad arguments");
  MXB_REQUIRE(topk_idx && within && send_counts, MXB_ERR_INVALID_ARGUMENT,
              "ep_route: null pointer");
  if (T == 0) {
    const cudaError_t e = cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world, to_cuda(stream));
    MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "ep_route: memset failed: %s",
                cudaGetErrorString(e));
    return MXB_OK;
  }
  const int64_t tiles = (T + kRouteTile - 1) / kRouteTile;
  if (tiles * world > kRouteMaxEntries || T * world > 0x7FFFFFFFLL) {
    ep_route_serial_kernel<<<1, kRouteThreads, 0, to_cuda(stream)>>>(
        topk_idx, T, topk, experts_per_rank, world, within, send_counts);
  } else {
    ep_route_tile_kernel<<<(int)tiles, kRouteTile, 0, to_cuda(stream)>>>(
        topk_idx, T, topk, experts_per_rank, world, within);
    const size_t smem = sizeof(int32_t) * tiles * world;
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(
          ep_route_prefix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "ep_route: %s", cudaGetErrorString(e));
    }
    ep_route_prefix_kernel<<<1, kRouteThreads, smem, to_cuda(stream)>>>(T, world, (int)tiles,
                                                                        within, send_counts);
  }
  return launch_status("ep_route");
}

extern "C" mxb_status mxb_ep_p2p_combine(const void* back, int64_t T, int64_t H,
                                         const int32_t* within, const int32_t* send_counts,
                                         int32_t world, void* out, mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_p2p_combine");
  MXB_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && world >= 1 && world <= 64,
              MXB_ERR_INVALID_ARGUMENT, "ep_p2p_combine: bad arguments");
  if (T == 0) return MXB_OK;
  MXB_REQUIRE(back && within && send_counts && out, MXB_ERR_INVALID_ARGUMENT,
              "ep_p2p_combine: null pointer");
  MXB_REQUIRE(aligned(back, 16) && aligned(out, 16), MXB_ERR_MISALIGNED,
              "ep_p2p_combine: back and out must be 16-byte aligned");
  const int64_t segs = (H / 8 + 127) / 128;
  ep_p2p_combine_kernel<<<p2p_grid(T * segs), kP2PThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)back, T, H, within, send_counts, world, (uint8_t*)out);
  return launch_status("ep_p2p_combine");
}

extern "C" unsigned int mxb_ep_wait_timeouts(void) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ep_timeouts, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  return v;
}

extern "C" unsigned int mxb_ep_reset_wait_timeouts(void) {
  const unsigned int v = mxb_ep_wait_timeouts();
  const unsigned int z = 0;
  if (cudaMemcpyToSymbol(g_ep_timeouts, &z, sizeof(z)) != cudaSuccess) return 0xFFFFFFFFu;
  return v;
}

extern "C" mxb_status mxb_ep_set_wait_polls(uint32_t polls) {
  const uint32_t v = polls ? polls : kPeerSpins;
  const cudaError_t e = cudaMemcpyToSymbol(g_ep_wait_polls, &v, sizeof(v));
  MXB_REQUIRE(e == cudaSuccess, MXB_ERR_CUDA, "ep_set_wait_polls: %s", cudaGetErrorString(e));
  return MXB_OK;
}
