// MoE expert-parallel dispatch / combine kernels with MXFP4 payloads (sm_100a).
//
// Wire row of one token (megatron-0.15.0rc7.diff:32-63, `_pack_rowwise_components`):
//     codes[H/2] || E8M0 scales[H/32]        (row_bytes = 17 H / 32; 3808 B at H = 7168)
// The reference quantizes the tokens (Q-row), concatenates codes and scales along
// the last dimension and hands the rows to DeepEP's dispatch; the receiver splits
// them at 16/17 and dequantizes (C2) (megatron-0.15.0rc7.diff:91-124,290-311).
//
//  * ep_pack: one CTA per token quantizes the row once (bit-exact Q-row) and
//    writes its wire row to every destination slot slots[t, g] >= 0, so a token
//    routed to several ranks is read from HBM once.
//  * ep_unpack: wire rows -> BF16 (bit-exact C2); optionally times a per-row
//    FP32 weight (the routing-weighted identity expert of the benchmark).
//  * ep_combine: out[t] = bf16(sum over g = 0..G-1 of float(recv[slots[t, g]])),
//    summed in rank order (deterministic).
#include <cuda_bf16.h>

#include <type_traits>

#include "capi_util.h"
#include "common.cuh"
#include "qrow.cuh"
#include "tma.cuh"

namespace mxb {
namespace {

constexpr int kEpThreads = 256;

// Q-row of one 32-element block held as 16 BF16 pairs (fp4_max = 6,
// eps <= 6e-10): the quantizers' own block routine (qrow.cuh).
__device__ __forceinline__ void ep_quant_block(const uint32_t (&w)[16], uint32_t (&out)[4],
                                               uint32_t& byte, float eps) {
  quant_block32<true>(w, QuantParams{eps, -6.0f, 6.0f}, out, byte);
}

__global__ void __launch_bounds__(kEpThreads) ep_pack_kernel(const uint8_t* __restrict__ x,
                                                             int64_t T, int64_t H,
                                                             const int32_t* __restrict__ slots,
                                                             int G, uint8_t* __restrict__ wire,
                                                             int64_t row_bytes, float eps) {
  __shared__ int32_t dst[64];
  const int64_t nb = H / 32;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x < G) dst[threadIdx.x] = slots[t * G + threadIdx.x];
    __syncthreads();
    const uint8_t* xr = x + t * H * 2;
    for (int64_t b = threadIdx.x; b < nb; b += kEpThreads) {
      const uint4 a0 = ld_stream_v4(xr + b * 64), a1 = ld_stream_v4(xr + b * 64 + 16);
      const uint4 a2 = ld_stream_v4(xr + b * 64 + 32), a3 = ld_stream_v4(xr + b * 64 + 48);
      const uint32_t w[16] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w,
                              a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
      uint32_t out[4], byte;
      ep_quant_block(w, out, byte, eps);
      for (int g = 0; g < G; ++g) {
        const int32_t s = dst[g];
        if (s < 0) continue;
        uint8_t* row = wire + (int64_t)s * row_bytes;
        uint32_t* c = reinterpret_cast<uint32_t*>(row + b * 16);
        c[0] = out[0]; c[1] = out[1]; c[2] = out[2]; c[3] = out[3];
        row[H / 2 + b] = (uint8_t)byte;
      }
    }
    __syncthreads();
  }
}

// wire rows -> BF16 (optionally x weight[row]); a thread handles 4 code bytes.
__global__ void __launch_bounds__(kEpThreads) ep_unpack_kernel(const uint8_t* __restrict__ wire,
                                                               int64_t R, int64_t H,
                                                               int64_t row_bytes,
                                                               const float* __restrict__ weight,
                                                               uint8_t* __restrict__ out) {
  const int64_t chunks = H / 8;  // 4 code bytes = 8 elements per chunk
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    const uint8_t* row = wire + r * row_bytes;
    const float wt = weight ? weight[r] : 1.0f;
    for (int64_t c = threadIdx.x; c < chunks; c += kEpThreads) {
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
        const float s = e8m0_to_f(e);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = cvt_bf16x2(bf16lo_to_f(o[i]) * s, bf16hi_to_f(o[i]) * s);
      }
      if (weight) {
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = cvt_bf16x2(bf16lo_to_f(o[i]) * wt, bf16hi_to_f(o[i]) * wt);
      }
      *reinterpret_cast<uint4*>(out + (r * H + c * 8) * 2) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// out[t] = bf16(sum_g float(recv[slots[t, g]])) in rank order.
__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(const uint8_t* __restrict__ recv,
                                                                int64_t T, int64_t H,
                                                                const int32_t* __restrict__ slots,
                                                                int G, uint8_t* __restrict__ out) {
  __shared__ int32_t src[64];
  const int64_t chunks = H / 8;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x < G) src[threadIdx.x] = slots[t * G + threadIdx.x];
    __syncthreads();
    for (int64_t c = threadIdx.x; c < chunks; c += kEpThreads) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int g = 0; g < G; ++g) {
        const int32_t s = src[g];
        if (s < 0) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(recv + ((int64_t)s * H + c * 8) * 2);
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

int ep_grid(int64_t rows) { return (int)(rows < 148LL * 16 ? (rows > 0 ? rows : 1) : 148LL * 16); }

// ------------------------------------------------------------ moe_permute
// The MXFP4 branch of Transformer Engine's moe_permute (transformer_engine-2.8.diff:
// 253-261,338-356): every source row goes, codes and E8M0 scales alike, to each
// expert slot it is routed to.  Here fused with the EP receive side: the source
// rows may be wire rows (codes || scales, megatron-0.15.0rc7.diff:32-63), which
// are split in the same pass.  One warp per source row reads the row once
// (16-byte chunks when every address and pitch allows, else 4-byte words, else
// bytes) and
// stores it to each destination dst[i * topk + k] in [0, n_out); other values
// (e.g. -1 for no slot) are skipped.
constexpr int kPermWarps = kEpThreads / 32;

template <int kVec>
__device__ __forceinline__ void permute_span(const uint8_t* src, int64_t bytes, uint8_t* out,
                                             int64_t out_pitch, const int32_t (&d)[32], int topk,
                                             int64_t n_out, int lane) {
  using V = typename std::conditional<
      kVec == 16, uint4, typename std::conditional<kVec == 4, uint32_t, uint8_t>::type>::type;
  constexpr int kBatch = 8;  // chunks per lane loaded before any is stored
  const int64_t n = bytes / kVec;
  for (int64_t c0 = 0; c0 < n; c0 += 32 * kBatch) {
    V v[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int64_t c = c0 + b * 32 + lane;
      if (c < n) v[b] = *reinterpret_cast<const V*>(src + c * kVec);
    }
    for (int k = 0; k < topk; ++k) {
      const int32_t dk = d[k];
      if (dk < 0 || dk >= n_out) continue;
      uint8_t* o = out + (int64_t)dk * out_pitch;
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int64_t c = c0 + b * 32 + lane;
        if (c < n) *reinterpret_cast<V*>(o + c * kVec) = v[b];
      }
    }
  }
}

// Where source row i goes: destinations dst[i * pitch + k] for k < n(i), with
// n(i) = topk, or dst[i * pitch + count_col] when count_col >= 0 (Transformer
// Engine's row_id_map keeps each row's count in its last column).
struct DstMap {
  const int32_t* dst;
  int64_t pitch;
  int count_col, topk;
  __device__ __forceinline__ int count(int64_t i) const {
    return count_col >= 0 ? dst[i * pitch + count_col] : topk;
  }
};

template <int kVec>
__global__ void __launch_bounds__(kEpThreads) moe_permute_kernel(
    const uint8_t* __restrict__ codes, int64_t cpitch, const uint8_t* __restrict__ scales,
    int64_t spitch, int64_t rows, int64_t H, DstMap map, uint8_t* __restrict__ out_codes,
    uint8_t* __restrict__ out_scales, int64_t n_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t)blockIdx.x * kPermWarps + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * kPermWarps;
  for (int64_t i = warp0; i < rows; i += nwarps) {
    const int n = map.count(i);
    for (int k0 = 0; k0 < n; k0 += 32) {  // destinations in groups of 32 (one row read each)
      const int cnt = min(32, n - k0);
      const int32_t mine = lane < cnt ? map.dst[i * map.pitch + k0 + lane] : -1;
      int32_t d[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) d[k] = __shfl_sync(0xffffffffu, mine, k);
      permute_span<kVec>(codes + i * cpitch, H / 2, out_codes, H / 2, d, cnt, n_out, lane);
      permute_span<kVec>(scales + i * spitch, H / 32, out_scales, H / 32, d, cnt, n_out, lane);
    }
  }
}

// The same permute with the SM's bulk-copy unit (16-byte aligned rows whose
// scale part is a multiple of 16 bytes, e.g. H = 7168: 3584 + 224 bytes): a
// one-warp CTA streams its rows through a ring of kPermStages shared-memory
// slots.  A row arrives by two 1-D bulk loads (codes, scales) issued by lane
// 0; lane k < topk reads destination k and issues that destination's two 1-D
// bulk stores, so no register or load/store-unit traffic carries the bytes
// and the destinations are stored in parallel.  A slot is refilled once every
// lane's stores of the row it held have read it (bulk wait_group.read), one
// row behind the current one.
constexpr int kPermStages = 4;

__global__ void __launch_bounds__(32) moe_permute_bulk_kernel(
    const uint8_t* __restrict__ codes, int64_t cpitch, const uint8_t* __restrict__ scales,
    int64_t spitch, int64_t rows, int64_t H, DstMap map, uint8_t* __restrict__ out_codes,
    uint8_t* __restrict__ out_scales, int64_t n_out, uint32_t slot_bytes) {
  extern __shared__ __align__(128) uint8_t psm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(psm + kPermStages * slot_bytes);
  const int lane = threadIdx.x;
  const uint32_t cb = (uint32_t)(H / 2), sb = (uint32_t)(H / 32);
  const int64_t first = blockIdx.x, step = gridDim.x;
  const int64_t my = first < rows ? (rows - 1 - first) / step + 1 : 0;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kPermStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto load = [&](int64_t j) {
    const int s = (int)(j % kPermStages);
    const int64_t i = first + j * step;
    uint8_t* slot = psm + s * slot_bytes;
    mbar_arrive_expect_tx(&full[s], cb + sb);
    bulk_load_1d(slot, codes + i * cpitch, cb, &full[s]);
    bulk_load_1d(slot + cb, scales + i * spitch, sb, &full[s]);
  };
  int64_t issued = my < kPermStages ? my : kPermStages;
  if (lane == 0)
    for (int64_t q = 0; q < issued; ++q) load(q);
  int64_t j = 0;
  for (; j < my; ++j) {
    const int s = (int)(j % kPermStages);
    const int64_t i = first + j * step;
    const int n = map.count(i);
    const int32_t d = lane < n ? map.dst[i * map.pitch + lane] : -1;
    const bool ok = mbar_wait(&full[s], (uint32_t)(j / kPermStages) & 1u);
    if (!__all_sync(0xffffffffu, ok)) break;
    const uint8_t* slot = psm + s * slot_bytes;
    if (d >= 0 && d < n_out) {
      bulk_store_1d(out_codes + (int64_t)d * cb, slot, cb);
      bulk_store_1d(out_scales + (int64_t)d * sb, slot + cb, sb);
    }
    for (int k = 32 + lane; k < n; k += 32) {  // more than 32 destinations
      const int32_t dk = map.dst[i * map.pitch + k];
      if (dk >= 0 && dk < n_out) {
        bulk_store_1d(out_codes + (int64_t)dk * cb, slot, cb);
        bulk_store_1d(out_scales + (int64_t)dk * sb, slot + cb, sb);
      }
    }
    bulk_commit();
    // refill the slot of row j-1 once every lane's stores have read it
    if (j >= 1 && issued < my) {
      bulk_wait_read_1();
      __syncwarp();
      if (lane == 0) load(issued);
      ++issued;
    }
  }
  // a row that never arrived: do not exit while requested copies may still land
  if (lane == 0)
    for (int64_t q = j; q < issued; ++q)
      mbar_wait(&full[q % kPermStages], (uint32_t)(q / kPermStages) & 1u);
  bulk_wait_all();
}

// ------------------------------------------------------------ row_id_map
// Transformer Engine's moe_permute with a mask routing map builds a row_id_map
// from routing_map (bool [T, E]) and moves each token row to its experts'
// slots with it.  The map restated here: row r of the permuted output holds
// the tokens routed to expert 0 in token order, then those routed to expert 1,
// ...; int32 [T, 2E + 1] per token t: columns 0 .. n-1 the destination rows of
// its n routed experts (ascending expert order), columns E .. E+n-1 those
// experts, column 2E the count n, the unused columns -1.
//   1. one CTA per expert ranks the expert's tokens (ballot scan down the
//      column) into column e and writes the expert's count;
//   2. one CTA turns the counts into exclusive offsets;
//   3. one thread per token compacts its columns in place.
constexpr int kRidThreads = 1024;

__global__ void __launch_bounds__(kRidThreads) row_id_rank_kernel(
    const uint8_t* __restrict__ routing_map, int64_t T, int E, int32_t* __restrict__ rid,
    int32_t* __restrict__ counts) {
  __shared__ int32_t warp_sum[kRidThreads / 32];
  const int e = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t P = 2LL * E + 1;
  int32_t carry = 0;
  for (int64_t t0 = 0; t0 < T; t0 += kRidThreads) {
    const int64_t t = t0 + threadIdx.x;
    const bool flag = t < T && routing_map[t * E + e] != 0;
    const uint32_t b = __ballot_sync(0xffffffffu, flag);
    const int32_t lane_rank = __popc(b & ((1u << lane) - 1u));
    if (lane == 0) warp_sum[warp] = __popc(b);
    __syncthreads();
    int32_t before = 0, total = 0;
    for (int w = 0; w < kRidThreads / 32; ++w) {  // tiny: 32 shared loads
      const int32_t v = warp_sum[w];
      before += w < warp ? v : 0;
      total += v;
    }
    if (t < T) rid[t * P + e] = flag ? carry + before + lane_rank : -1;
    carry += total;
    __syncthreads();  // warp_sum reused
  }
  if (threadIdx.x == 0) counts[e] = carry;
}

__global__ void row_id_offsets_kernel(int32_t* __restrict__ counts, int E) {
  if (threadIdx.x != 0) return;
  int32_t acc = 0;
  for (int e = 0; e < E; ++e) {
    const int32_t c = counts[e];
    counts[e] = acc;
    acc += c;
  }
}

__global__ void row_id_compact_kernel(int32_t* __restrict__ rid, const int32_t* __restrict__ offsets,
                                      int64_t T, int E) {
  const int64_t P = 2LL * E + 1;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T;
       t += (int64_t)gridDim.x * blockDim.x) {
    int32_t* row = rid + t * P;
    int j = 0;
    for (int e = 0; e < E; ++e) {  // column j <= e: never overwrites an unread rank
      const int32_t r = row[e];
      if (r >= 0) {
        row[j] = offsets[e] + r;
        row[E + j] = e;
        ++j;
      }
    }
    for (int k = j; k < E; ++k) {
      row[k] = -1;
      row[E + k] = -1;
    }
    row[2 * E] = j;
  }
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_ep_pack(const void* x, int64_t T, int64_t H, const int32_t* slots,
                                  int G, void* wire, float eps, mxb_stream_t stream) {
  MXB_REQUIRE(T >= 0 && H > 0 && H % 128 == 0 && G >= 1 && G <= 64, MXB_ERR_INVALID_ARGUMENT,
              "ep_pack: need H %% 128 == 0 and 1 <= G <= 64 (H=%lld G=%d)", (long long)H, G);
  MXB_REQUIRE(eps >= 0.0f && eps <= 6e-10f, MXB_ERR_UNSUPPORTED,
              "ep_pack: eps must be in [0, 6e-10] (the dispatch quantizer's configuration)");
  if (T == 0) return MXB_OK;
  MXB_REQUIRE(x && slots && wire, MXB_ERR_INVALID_ARGUMENT, "ep_pack: null pointer");
  const int64_t row_bytes = H / 2 + H / 32;
  MXB_REQUIRE(aligned(x, 16) && aligned(wire, 4) && row_bytes % 4 == 0, MXB_ERR_MISALIGNED,
              "ep_pack: x must be 16-byte and wire rows 4-byte aligned");
  ep_pack_kernel<<<ep_grid(T), kEpThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)x, T, H, slots, G, (uint8_t*)wire, row_bytes, eps);
  return launch_status("ep_pack");
}

extern "C" mxb_status mxb_ep_unpack(const void* wire, int64_t R, int64_t H, const float* weight,
                                    void* out, mxb_stream_t stream) {
  MXB_REQUIRE(R >= 0 && H > 0 && H % 128 == 0, MXB_ERR_INVALID_ARGUMENT,
              "ep_unpack: need H %% 128 == 0 (H=%lld)", (long long)H);
  if (R == 0) return MXB_OK;
  MXB_REQUIRE(wire && out, MXB_ERR_INVALID_ARGUMENT, "ep_unpack: null pointer");
  const int64_t row_bytes = H / 2 + H / 32;
  MXB_REQUIRE(aligned(wire, 4) && row_bytes % 4 == 0 && aligned(out, 16), MXB_ERR_MISALIGNED,
              "ep_unpack: wire rows must be 4-byte and out 16-byte aligned");
  ep_unpack_kernel<<<ep_grid(R), kEpThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)wire, R, H, row_bytes, weight, (uint8_t*)out);
  return launch_status("ep_unpack");
}

extern "C" mxb_status mxb_ep_combine(const void* recv, int64_t T, int64_t H, const int32_t* slots,
                                     int G, void* out, mxb_stream_t stream) {
  MXB_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && G >= 1 && G <= 64, MXB_ERR_INVALID_ARGUMENT,
              "ep_combine: need H %% 8 == 0 and 1 <= G <= 64");
  if (T == 0) return MXB_OK;
  MXB_REQUIRE(recv && slots && out, MXB_ERR_INVALID_ARGUMENT, "ep_combine: null pointer");
  MXB_REQUIRE(aligned(recv, 16) && aligned(out, 16), MXB_ERR_MISALIGNED,
              "ep_combine: recv and out must be 16-byte aligned");
  ep_combine_kernel<<<ep_grid(T), kEpThreads, 0, to_cuda(stream)>>>(
      (const uint8_t*)recv, T, H, slots, G, (uint8_t*)out);
  return launch_status("ep_combine");
}

static mxb_status moe_permute_impl(const void* codes, int64_t codes_pitch, const void* scales,
                                   int64_t scales_pitch, int64_t rows, int64_t H, DstMap map,
                                   void* out_codes, void* out_scales, int64_t n_out,
                                   mxb_stream_t stream) {
  const uintptr_t any = reinterpret_cast<uintptr_t>(codes) | reinterpret_cast<uintptr_t>(scales) |
                        reinterpret_cast<uintptr_t>(out_codes) |
                        reinterpret_cast<uintptr_t>(out_scales) | (uintptr_t)codes_pitch |
                        (uintptr_t)scales_pitch | (uintptr_t)(H / 2) | (uintptr_t)(H / 32);
  const uint32_t slot = (uint32_t)((H / 2 + H / 32 + 127) / 128 * 128);
  if ((any & 15) == 0 && (H / 32) % 16 == 0 && (size_t)slot * kPermStages <= 96 * 1024) {
    const size_t smem = (size_t)slot * kPermStages + kPermStages * 8;
    static const bool attr = cudaFuncSetAttribute((const void*)moe_permute_bulk_kernel,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  96 * 1024 + 64) == cudaSuccess;
    MXB_REQUIRE(attr, MXB_ERR_CUDA, "moe_permute_mxfp4: cannot reserve shared memory");
    const int per_sm = (int)max((size_t)1, min((size_t)32, (size_t)(200 * 1024) / (smem + 1024)));
    const int g = (int)min((int64_t)148 * per_sm, rows);
    moe_permute_bulk_kernel<<<g, 32, smem, to_cuda(stream)>>>(
        (const uint8_t*)codes, codes_pitch, (const uint8_t*)scales, scales_pitch, rows, H, map,
        (uint8_t*)out_codes, (uint8_t*)out_scales, n_out, slot);
    return launch_status("moe_permute_mxfp4");
  }
  const int grid = (int)min((int64_t)148 * 8, cdiv(rows, kPermWarps));
  auto* c = (const uint8_t*)codes;
  auto* sc = (const uint8_t*)scales;
  auto* oc = (uint8_t*)out_codes;
  auto* os = (uint8_t*)out_scales;
  if ((any & 15) == 0)
    moe_permute_kernel<16><<<grid, kEpThreads, 0, to_cuda(stream)>>>(c, codes_pitch, sc, scales_pitch,
                                                                     rows, H, map, oc, os, n_out);
  else if ((any & 3) == 0)
    moe_permute_kernel<4><<<grid, kEpThreads, 0, to_cuda(stream)>>>(c, codes_pitch, sc, scales_pitch,
                                                                    rows, H, map, oc, os, n_out);
  else
    moe_permute_kernel<1><<<grid, kEpThreads, 0, to_cuda(stream)>>>(c, codes_pitch, sc, scales_pitch,
                                                                    rows, H, map, oc, os, n_out);
  return launch_status("moe_permute_mxfp4");
}

extern "C" mxb_status mxb_moe_permute_mxfp4(const void* codes, int64_t codes_pitch,
                                            const void* scales, int64_t scales_pitch, int64_t rows,
                                            int64_t H, const int32_t* dst, int topk,
                                            void* out_codes, void* out_scales, int64_t n_out,
                                            mxb_stream_t stream) {
  MXB_REQUIRE(rows >= 0 && H > 0 && H % 32 == 0 && topk >= 1 && topk <= 32 && n_out >= 0,
              MXB_ERR_INVALID_ARGUMENT, "moe_permute_mxfp4: need H %% 32 == 0 and 1 <= topk <= 32");
  MXB_REQUIRE(codes_pitch >= H / 2 && scales_pitch >= H / 32, MXB_ERR_INVALID_ARGUMENT,
              "moe_permute_mxfp4: pitches must cover a row (codes H/2, scales H/32 bytes)");
  if (rows == 0 || n_out == 0) return MXB_OK;
  MXB_REQUIRE(codes && scales && dst && out_codes && out_scales, MXB_ERR_INVALID_ARGUMENT,
              "moe_permute_mxfp4: null pointer");
  return moe_permute_impl(codes, codes_pitch, scales, scales_pitch, rows, H,
                          DstMap{dst, topk, -1, topk}, out_codes, out_scales, n_out, stream);
}

extern "C" mxb_status mxb_moe_permute_mxfp4_row_id_map(const void* codes, int64_t codes_pitch,
                                                       const void* scales, int64_t scales_pitch,
                                                       int64_t T, int64_t H,
                                                       const int32_t* row_id_map, int32_t E,
                                                       void* out_codes, void* out_scales,
                                                       int64_t num_out_tokens,
                                                       mxb_stream_t stream) {
  MXB_REQUIRE(T >= 0 && H > 0 && H % 32 == 0 && E >= 1 && num_out_tokens >= 0,
              MXB_ERR_INVALID_ARGUMENT, "moe_permute_mxfp4_row_id_map: need H %% 32 == 0, E >= 1");
  MXB_REQUIRE(codes_pitch >= H / 2 && scales_pitch >= H / 32, MXB_ERR_INVALID_ARGUMENT,
              "moe_permute_mxfp4_row_id_map: pitches must cover a row");
  if (T == 0 || num_out_tokens == 0) return MXB_OK;
  MXB_REQUIRE(codes && scales && row_id_map && out_codes && out_scales, MXB_ERR_INVALID_ARGUMENT,
              "moe_permute_mxfp4_row_id_map: null pointer");
  return moe_permute_impl(codes, codes_pitch, scales, scales_pitch, T, H,
                          DstMap{row_id_map, 2LL * E + 1, 2 * E, 0}, out_codes, out_scales,
                          num_out_tokens, stream);
}

extern "C" mxb_status mxb_moe_make_row_id_map(const void* routing_map, int64_t T, int32_t E,
                                              int32_t* row_id_map, int32_t* workspace,
                                              mxb_stream_t stream) {
  MXB_REQUIRE(T >= 0 && E >= 1 && T <= INT32_MAX, MXB_ERR_INVALID_ARGUMENT,
              "moe_make_row_id_map: need 0 <= T < 2^31 and E >= 1");
  if (T == 0) return MXB_OK;
  MXB_REQUIRE(routing_map && row_id_map && workspace, MXB_ERR_INVALID_ARGUMENT,
              "moe_make_row_id_map: null pointer");
  cudaStream_t s = to_cuda(stream);
  row_id_rank_kernel<<<E, kRidThreads, 0, s>>>((const uint8_t*)routing_map, T, E, row_id_map,
                                                workspace);
  row_id_offsets_kernel<<<1, 32, 0, s>>>(workspace, E);
  const int grid = (int)min((int64_t)148 * 8, cdiv(T, 256));
  row_id_compact_kernel<<<grid, 256, 0, s>>>(row_id_map, workspace, T, E);
  return launch_status("moe_make_row_id_map");
}
