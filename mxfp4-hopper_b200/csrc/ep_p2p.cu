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
  const int G = L.world, H = L.hidden;
  const int64_t nb = H / 32, rb = H / 2 + H / 32;
  const int32_t* cnt = cnt_of(bases, L, parity);
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x < G) {
      const int g = threadIdx.x;
      const int32_t wi = within[t * G + g];
      int64_t off = 0;
      for (int s = 0; s < L.rank; ++s) off += cnt[s * G + g];  // rows from lower ranks first
      dst_row[g] = wi < 0 ? -1 : off + wi;
    }
    __syncthreads();
    const uint8_t* xr = x + t * H * 2;
    for (int64_t b = threadIdx.x; b < nb; b += kP2PThreads) {
      const uint4 a0 = ld_stream_v4(xr + b * 64), a1 = ld_stream_v4(xr + b * 64 + 16);
      const uint4 a2 = ld_stream_v4(xr + b * 64 + 32), a3 = ld_stream_v4(xr + b * 64 + 48);
      const uint32_t w[16] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w,
                              a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
      uint32_t out[4], byte;
      p2p_quant_block(w, out, byte);
      for (int g = 0; g < G; ++g) {
        const int64_t r = dst_row[g];
        if (r < 0) continue;
        uint8_t* row = peer(bases, g) + L.wire_off + r * rb;
        *reinterpret_cast<uint4*>(row + b * 16) = make_uint4(out[0], out[1], out[2], out[3]);
        row[H / 2 + b] = (uint8_t)byte;
      }
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
  int64_t R = 0;
  for (int s = 0; s < G; ++s) R += col[s];
  const uint8_t* wire = peer(bases, L.rank) + L.wire_off;
  const int32_t* meta = reinterpret_cast<const int32_t*>(peer(bases, L.rank) + L.meta_off);
  const int64_t chunks = H / 8;
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    int s = 0;
    int64_t start = 0;
    while (s < G - 1 && r >= start + col[s]) start += col[s++];
    const int64_t dst = back_off[s] + (r - start);
    uint8_t* out = peer(bases, s) + L.back_off + dst * H * 2;
    float wsum = 0.0f;
    if (!y_in) {
      const int32_t* m = meta + r * 2 * L.topk;
      wsum = __int_as_float(m[L.topk]);
      for (int j = 1; j < L.topk; ++j) wsum += __int_as_float(m[L.topk + j]);
    }
    const uint8_t* row = wire + r * rb;
    for (int64_t c = threadIdx.x; c < chunks; c += kP2PThreads) {
      uint4 v;
      if (y_in) {
        v = *reinterpret_cast<const uint4*>(y_in + (r * H + c * 8) * 2);
      } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(row + c * 4);
        const uint32_t e = row[H / 2 + (c >> 2)];
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
        v = make_uint4(o[0], o[1], o[2], o[3]);
      }
      *reinterpret_cast<uint4*>(out + c * 16) = v;
    }
  }
  __threadfence_system();
}

// Routing without host synchronisation.  CTA g scans the tokens in order and
// gives every token routed to rank g its index among them (within[t, g], -1 if
// the token does not go to g); send_counts[g] is the number of such tokens.
constexpr int kRouteThreads = 1024;

__global__ void __launch_bounds__(kRouteThreads) ep_route_kernel(
    const int64_t* __restrict__ topk_idx, int64_t T, int k, int experts_per_rank, int G,
    int32_t* __restrict__ within, int32_t* __restrict__ send_counts) {
  __shared__ int32_t warp_sums[kRouteThreads / 32];
  const int g = blockIdx.x, t0 = threadIdx.x, lane = t0 & 31, warp = t0 >> 5;
  const int64_t per = (T + kRouteThreads - 1) / kRouteThreads;  // tokens per thread
  const int64_t lo = t0 * per, hi = min(T, lo + per);
  auto hits = [&](int64_t t) {
    bool h = false;
    for (int j = 0; j < k; ++j) h |= (topk_idx[t * k + j] / experts_per_rank) == g;
    return h;
  };
  int32_t c = 0;
  for (int64_t t = lo; t < hi; ++t) c += hits(t) ? 1 : 0;
  // block-wide exclusive scan of c
  int32_t v = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int32_t ws = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t n = __shfl_up_sync(0xffffffffu, ws, o);
      if (lane >= o) ws += n;
    }
    warp_sums[lane] = ws;  // inclusive over warps
  }
  __syncthreads();
  int32_t base = v - c + (warp > 0 ? warp_sums[warp - 1] : 0);
  for (int64_t t = lo; t < hi; ++t) within[t * G + g] = hits(t) ? base++ : -1;
  if (t0 == kRouteThreads - 1) send_counts[g] = warp_sums[31];
}

// Local combine of the rows returned to this rank: out[t] = bf16(sum over g of
// float(back[slot(t, g)])), slot(t, g) = sum_{g' < g} send_counts[g'] + within[t, g].
__global__ void __launch_bounds__(kP2PThreads) ep_p2p_combine_kernel(
    const uint8_t* __restrict__ back, int64_t T, int64_t H, const int32_t* __restrict__ within,
    const int32_t* __restrict__ send_counts, int G, uint8_t* __restrict__ out) {
  __shared__ int64_t src[64];
  const int64_t chunks = H / 8;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x < G) {
      const int g = threadIdx.x;
      int64_t off = 0;
      for (int q = 0; q < g; ++q) off += send_counts[q];
      const int32_t wi = within[t * G + g];
      src[g] = wi < 0 ? -1 : off + wi;
    }
    __syncthreads();
    for (int64_t c = threadIdx.x; c < chunks; c += kP2PThreads) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int g = 0; g < G; ++g) {
        const int64_t sl = src[g];
        if (sl < 0) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(back + (sl * H + c * 8) * 2);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] += bf16lo_to_f(w[i]);
          acc[2 * i + 1] += bf16hi_to_f(w[i]);
        }
      }
      *reinterpret_cast<uint4*>(out + (t * H + c * 8) * 2) =
          make_uint4(cvt_bf16x2(acc[0], acc[1]), cvt_bf16x2(acc[2], acc[3]),
                     cvt_bf16x2(acc[4], acc[5]), cvt_bf16x2(acc[6], acc[7]));
    }
    __syncthreads();
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
                  L->hidden % 512 == 0 && L->hidden > 0 && L->experts_per_rank >= 1,
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
  MXB_REQUIRE(T >= 0 && topk >= 1 && experts_per_rank >= 1 && world >= 1 && world <= 64,
              MXB_ERR_INVALID_ARGUMENT, "ep_route: bad arguments");
  MXB_REQUIRE(topk_idx && within && send_counts, MXB_ERR_INVALID_ARGUMENT,
              "ep_route: null pointer");
  ep_route_kernel<<<world, kRouteThreads, 0, to_cuda(stream)>>>(topk_idx, T, topk,
                                                                experts_per_rank, world, within,
                                                                send_counts);
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
