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

namespace mxb {
namespace {

static __device__ unsigned int g_ep_timeouts;
constexpr uint32_t kPeerSpins = 1u << 22;  // polls of ~64 ns sleep each
constexpr int kP2PThreads = 256;
constexpr int kMaxScaleBytes = 2048;  // H / 32 for H <= 65536

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
    uint32_t i = 0;
    while (ld_acquire_sys(mine) < epoch) {
      if (++i == kPeerSpins) {
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

// Q-row of one 32-element block (fast path; literal fallback for Inf/NaN).
__device__ __forceinline__ void p2p_quant_block(const uint32_t (&w)[16], uint32_t (&out)[4],
                                                uint32_t& byte) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) m = vmax_u16x2(m, w[i] & 0x7FFF7FFFu);
  const uint32_t mb = max(m & 0xFFFFu, m >> 16);
  if (mb < 0x7F80u) {
    int k = (int)(mb >> 7) - 129 + ((mb & 0x7Fu) > 0x40u ? 1 : 0);
    k = k < -33 ? -33 : k;
    byte = (uint32_t)(k + 127);
    const float inv = __uint_as_float((uint32_t)(127 - k) << 23);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = bf16lo_to_f(w[4 * i + j]) * inv;
        v[2 * j + 1] = bf16hi_to_f(w[4 * i + j]) * inv;
      }
      out[i] = cvt_e2m1x8(v);
    }
  } else {
    float a = 1e-10f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      a = fmaxf(a, fmaxf(fabsf(bf16lo_to_f(w[i])), fabsf(bf16hi_to_f(w[i]))));
    const float y = exp2f(ceilf(log2f(fmaxf(a / 6.0f, 1e-10f))));
    byte = ((uint32_t)(int)log2f(y) + 127u) & 0xFFu;
    const float inv = 1.0f / y;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t r = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t wj = w[4 * i + j / 2];
        float q = (j & 1) ? bf16hi_to_f(wj) : bf16lo_to_f(wj);
        q = fminf(fmaxf(q * inv, -6.0f), 6.0f);
        const uint32_t b = __float_as_uint(q);
        const uint32_t sign = b >> 28 & 0x8u;
        uint32_t ex = (b >> 23) & 0xFFu, man = b & 0x7FFFFFu;
        if (ex < 127u) {
          const uint32_t sh = 126u - ex;
          man = sh >= 32u ? 0u : ((0x400000u | (man >> 1)) >> sh);
        }
        ex = (ex > 126u ? ex : 126u) - 126u;
        const uint32_t m2 = man >> 21;
        const uint32_t inc = (m2 & 1u) & (((man & 0x1FFFFFu) != 0u) | ((m2 >> 1) & 1u));
        uint32_t c = (((ex << 2) | m2) + inc) >> 1;
        c = c > 7u ? 7u : c;
        r |= (sign | c) << (4 * j);
      }
      out[i] = r;
    }
  }
}

// One CTA per token (grid-stride): quantize the row once, store its wire row
// and routing metadata into every destination's receive buffer.
__global__ void __launch_bounds__(kP2PThreads) ep_dispatch_p2p_kernel(
    const uint8_t* __restrict__ x, int64_t T, const int32_t* __restrict__ within,
    const int64_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
    const uint64_t* __restrict__ bases, mxb_ep_layout L, int parity) {
  __shared__ int64_t dst_row[64];
  __shared__ __align__(16) uint8_t scale_bytes[kMaxScaleBytes];
  const int G = L.world, H = L.hidden;
  const int64_t nb = H / 32, rb = H / 2 + H / 32;
  const int32_t* cnt = cnt_of(bases, L, parity);
  int64_t off = 0;  // thread g < G: rows that lower ranks send to g come first
  if (threadIdx.x < G)
    for (int s = 0; s < L.rank; ++s) off += cnt[s * G + threadIdx.x];
  const int64_t b0 = threadIdx.x;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const uint8_t* xr = x + t * H * 2;
    uint4 a[4];
    if (b0 < nb) {  // the first block's loads go out before the barrier
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = ld_stream_v4(xr + b0 * 64 + i * 16);
    }
    if (threadIdx.x < G) {
      const int32_t wi = within[t * G + threadIdx.x];
      dst_row[threadIdx.x] = wi < 0 ? -1 : off + wi;
    }
    __syncthreads();
    for (int64_t b = b0; b < nb; b += kP2PThreads) {
      if (b != b0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = ld_stream_v4(xr + b * 64 + i * 16);
      }
      const uint32_t w[16] = {a[0].x, a[0].y, a[0].z, a[0].w, a[1].x, a[1].y, a[1].z, a[1].w,
                              a[2].x, a[2].y, a[2].z, a[2].w, a[3].x, a[3].y, a[3].z, a[3].w};
      uint32_t out[4], byte;
      p2p_quant_block(w, out, byte);
      scale_bytes[b] = (uint8_t)byte;
      for (int g = 0; g < G; ++g) {
        const int64_t r = dst_row[g];
        if (r < 0) continue;
        uint8_t* row = peer(bases, g) + L.wire_off + r * rb;
        *reinterpret_cast<uint4*>(row + b * 16) = make_uint4(out[0], out[1], out[2], out[3]);
      }
    }
    __syncthreads();
    // the row's scale bytes go out as 16-byte stores (H / 32 is a multiple of 16)
    const int nv = (int)(nb / 16);
    for (int i = threadIdx.x; i < G * nv; i += kP2PThreads) {
      const int g = i / nv, q = i - g * nv;
      const int64_t r = dst_row[g];
      if (r < 0) continue;
      uint8_t* row = peer(bases, g) + L.wire_off + r * rb;
      *reinterpret_cast<uint4*>(row + H / 2 + q * 16) =
          *reinterpret_cast<const uint4*>(scale_bytes + q * 16);
    }
    // routing metadata: expert id local to the destination (or -1), weight (or 0)
    for (int i = threadIdx.x; i < G * L.topk; i += kP2PThreads) {
      const int g = i / L.topk, j = i - g * L.topk;
      const int64_t r = dst_row[g];
      if (r < 0) continue;
      const int64_t e = topk_idx[t * L.topk + j];
      const bool here = e / L.experts_per_rank == g;
      int32_t* m = reinterpret_cast<int32_t*>(peer(bases, g) + L.meta_off) + r * 2 * L.topk;
      m[j] = here ? (int32_t)(e - (int64_t)g * L.experts_per_rank) : -1;
      m[L.topk + j] = __float_as_int(here ? topk_w[t * L.topk + j] : 0.0f);
    }
    __syncthreads();
  }
  __threadfence_system();
}

// Expert stage + return: for every received row r (source s, i-th row from s),
// y = user row y_in[r] if given, else the routing-weighted identity expert
// bf16(bf16(dequant(wire[r])) * sum_j weight[r][j]); the row is stored into
// source s's `back` buffer at s's send slot sum_{g < rank} cnt[s][g] + i.
__global__ void __launch_bounds__(kP2PThreads) ep_return_p2p_kernel(
    const uint8_t* __restrict__ y_in, const uint64_t* __restrict__ bases, mxb_ep_layout L,
    int parity) {
  __shared__ int32_t col[64];     // cnt[s][rank]
  __shared__ int64_t back_off[64];  // sum_{g < rank} cnt[s][g]
  const int G = L.world, H = L.hidden;
  const int64_t rb = H / 2 + H / 32;
  const int32_t* cnt = cnt_of(bases, L, parity);
  if (threadIdx.x < G) {
    const int s = threadIdx.x;
    col[s] = cnt[s * G + L.rank];
    int64_t o = 0;
    for (int g = 0; g < L.rank; ++g) o += cnt[s * G + g];
    back_off[s] = o;
  }
  __syncthreads();
  // Rows are visited source-minor (i -> j = i / G, s = i % G) so that at any
  // moment the CTAs write to every source, local HBM and NVLink together.
  int64_t cmax = 0;
  for (int s = 0; s < G; ++s) cmax = max(cmax, (int64_t)col[s]);
  const uint8_t* wire = peer(bases, L.rank) + L.wire_off;
  const int32_t* meta = reinterpret_cast<const int32_t*>(peer(bases, L.rank) + L.meta_off);
  const int64_t chunks = H / 8;
  for (int64_t i = blockIdx.x; i < cmax * G; i += gridDim.x) {
    const int s = (int)(i % G);
    const int64_t j = i / G;
    if (j >= col[s]) continue;
    int64_t start = 0;
    for (int q = 0; q < s; ++q) start += col[q];
    const int64_t r = start + j;
    const int64_t dst = back_off[s] + j;
    uint8_t* out = peer(bases, s) + L.back_off + dst * H * 2;
    float wsum = 0.0f;
    if (!y_in) {  // lane j loads weight j; the sum keeps the order j = 0, 1, ...
      const int32_t* m = meta + r * 2 * L.topk;
      const int lane = threadIdx.x & 31;
      const float wj = lane < L.topk ? __int_as_float(m[L.topk + lane]) : 0.0f;
      wsum = __shfl_sync(0xffffffffu, wj, 0);
      for (int j = 1; j < L.topk; ++j) wsum += __shfl_sync(0xffffffffu, wj, j);
    }
    const uint8_t* row = wire + r * rb;
    constexpr int kU = 4;  // chunks per thread with their loads issued together
    for (int64_t c0 = threadIdx.x; c0 < chunks; c0 += kP2PThreads * kU) {
      if (y_in) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int64_t c = c0 + u * kP2PThreads;
          if (c < chunks) v[u] = *reinterpret_cast<const uint4*>(y_in + (r * H + c * 8) * 2);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int64_t c = c0 + u * kP2PThreads;
          if (c < chunks) *reinterpret_cast<uint4*>(out + c * 16) = v[u];
        }
        continue;
      }
      uint32_t wv[kU], ev[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t c = c0 + u * kP2PThreads;
        if (c < chunks) {
          wv[u] = *reinterpret_cast<const uint32_t*>(row + c * 4);
          ev[u] = row[H / 2 + (c >> 2)];
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t c = c0 + u * kP2PThreads;
        if (c >= chunks) continue;
        const uint32_t w = wv[u], e = ev[u];
        uint32_t o[4];
        e2m1x4_to_bf16x4(w, o[0], o[1]);
        e2m1x4_to_bf16x4(w >> 16, o[2], o[3]);
        if (e - 2u <= 252u) {
          const uint32_t s2 = (e << 7) | (e << 23);
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i] = mul_bf16x2(o[i], s2);
        } else {
          const float sc = e8m0_to_f(e);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[i] = cvt_bf16x2(bf16lo_to_f(o[i]) * sc, bf16hi_to_f(o[i]) * sc);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          o[i] = cvt_bf16x2(bf16lo_to_f(o[i]) * wsum, bf16hi_to_f(o[i]) * wsum);
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
  const uint32_t n = (uint32_t)(T * G), row_elems = (uint32_t)(kRouteTile * G);
  for (uint32_t i = threadIdx.x; i < n; i += kRouteThreads) {
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
// float(back[slot(t, g)])), slot(t, g) = sum_{g' < g} send_counts[g'] + within[t, g].
// Work items are (token, 8-element chunk) pairs over a grid-stride loop with
// no barrier inside; the slot offsets sit in shared memory and the loads of up
// to 4 sources are issued before their sums.
__global__ void __launch_bounds__(kP2PThreads) ep_p2p_combine_kernel(
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
  const int64_t chunks = H / 8, n = T * chunks;
  const bool small = n <= 0x7FFFFFFFLL;
  for (int64_t i = (int64_t)blockIdx.x * kP2PThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kP2PThreads) {
    const int64_t t = small ? (int64_t)((uint32_t)i / (uint32_t)chunks) : i / chunks;
    const int64_t c = i - t * chunks;
    const int32_t* wt = within + t * G;
    // A source that sent nothing adds +0, which leaves the sum unchanged: it
    // starts at +0 and so is never -0.
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int g0 = 0; g0 < G; g0 += 4) {
      int32_t wi[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) wi[u] = g0 + u < G ? wt[g0 + u] : -1;
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = wi[u] < 0 ? make_uint4(0, 0, 0, 0)
                         : *reinterpret_cast<const uint4*>(
                               back + ((off[g0 + u] + wi[u]) * H + c * 8) * 2);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] += bf16lo_to_f(w[q]);
          acc[2 * q + 1] += bf16hi_to_f(w[q]);
        }
      }
    }
    *reinterpret_cast<uint4*>(out + (t * H + c * 8) * 2) =
        make_uint4(cvt_bf16x2(acc[0], acc[1]), cvt_bf16x2(acc[2], acc[3]),
                   cvt_bf16x2(acc[4], acc[5]), cvt_bf16x2(acc[6], acc[7]));
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

int p2p_grid(int64_t rows) {
  return (int)(rows < 148LL * 8 ? (rows > 0 ? rows : 1) : 148LL * 8);
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
  mxb_status st = check_layout(L, "ep_p2p_barrier");
  if (st != MXB_OK) return st;
  MXB_REQUIRE(bases, MXB_ERR_INVALID_ARGUMENT, "ep_p2p_barrier: null pointer");
  ep_barrier_kernel<<<1, 32, 0, to_cuda(stream)>>>(bases, *L, epoch);
  return launch_status("ep_p2p_barrier");
}

extern "C" mxb_status mxb_ep_p2p_return(const void* y, const uint64_t* bases,
                                        const mxb_ep_layout* L, int parity, mxb_stream_t stream) {
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
  MXB_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && world >= 1 && world <= 64,
              MXB_ERR_INVALID_ARGUMENT, "ep_p2p_combine: bad arguments");
  if (T == 0) return MXB_OK;
  MXB_REQUIRE(back && within && send_counts && out, MXB_ERR_INVALID_ARGUMENT,
              "ep_p2p_combine: null pointer");
  MXB_REQUIRE(aligned(back, 16) && aligned(out, 16), MXB_ERR_MISALIGNED,
              "ep_p2p_combine: back and out must be 16-byte aligned");
  ep_p2p_combine_kernel<<<p2p_grid(T), kP2PThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)back, T, H, within, send_counts, world, (uint8_t*)out);
  return launch_status("ep_p2p_combine");
}

extern "C" unsigned int mxb_ep_wait_timeouts(void) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ep_timeouts, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  return v;
}
