// MoE expert-parallel dispatch / combine of MXFP4 tokens over an NCCL
// communicator, as a C ABI (one process per GPU): the exchange DeepEP's
// intranode dispatch / combine performs for the reference's MXFP4 payload
// (deep_ep-1.2.1.diff:455-549, megatron-0.15.0rc7.diff:290-311), for callers
// that hold an ncclComm_t rather than peer mappings.
//
//   dispatch: device routing (mxb_ep_route), send slots grouped by destination
//   rank, the fused quantize + pack of each token once into its wire rows
//   (mxb_ep_pack) plus per-row routing metadata, a grouped send/recv of the
//   per-peer row counts, one host synchronisation to learn them (DeepEP's
//   layout step), then a grouped send/recv of the wire rows and metadata.
//   combine: a grouped send/recv of the BF16 expert rows back to their source
//   ranks, then the rank-ordered BF16 sum per token (mxb_ep_combine).
//
// NCCL is opened at run time (dlopen of libnccl.so.2, which resolves to the
// copy a process already loaded, e.g. torch's), so the library itself loads
// without NCCL; only these entry points need it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "capi_util.h"
#include "common.cuh"

namespace mxb {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) =
      nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
    api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.group_start &&
             api.group_end && api.send && api.recv && api.error_string;
  });
  return api;
}

#define MXB_NCCL(call, what)                                                              \
  do {                                                                                    \
    const ncclResult_t r_ = (call);                                                       \
    MXB_REQUIRE(r_ == ncclSuccess, MXB_ERR_CUDA, "%s: %s", what, nccl().error_string(r_)); \
  } while (0)

// Workspace layout (256-byte aligned pieces) for T tokens, hidden H, top-k,
// world G; S = T * min(G, topk) bounds the send rows.
struct NcclWs {
  int64_t within, slots, counts, wire, meta, back, total;
};

NcclWs ws_layout(int64_t T, int64_t H, int64_t topk, int64_t G) {
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  const int64_t S = T * (G < topk ? G : topk);
  const int64_t rb = H / 2 + H / 32;
  NcclWs w;
  int64_t o = 0;
  w.within = o;
  o = up(o + 4 * T * G);
  w.slots = o;
  o = up(o + 4 * T * G);
  w.counts = o;  // send [G], recv [G] (int32)
  o = up(o + 8 * G);
  w.wire = o;
  o = up(o + S * rb);
  w.meta = o;  // per send row: topk int32 local expert ids, topk float weights
  o = up(o + S * topk * 8);
  w.back = o;  // returned BF16 rows, by send slot
  o = up(o + S * H * 2);
  w.total = o;
  return w;
}

// slots[t, g] = (rows this rank sends to ranks < g) + within[t, g], or -1.
__global__ void slots_kernel(const int32_t* __restrict__ within, const int32_t* __restrict__ counts,
                             int64_t T, int G, int32_t* __restrict__ slots) {
  __shared__ int32_t off[64];
  if (threadIdx.x == 0) {
    int32_t acc = 0;
    for (int g = 0; g < G; ++g) {
      off[g] = acc;
      acc += counts[g];
    }
  }
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < T * G;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t w = within[i];
    slots[i] = w >= 0 ? off[i % G] + w : -1;
  }
}

// Routing metadata of each send row: the token's experts local to the
// destination rank (-1 elsewhere) and their weights (0 elsewhere).
__global__ void meta_kernel(const int32_t* __restrict__ slots, const int64_t* __restrict__ topk_idx,
                            const float* __restrict__ topk_w, int64_t T, int G, int topk,
                            int experts_per_rank, int32_t* __restrict__ meta) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < T * G;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t s = slots[i];
    if (s < 0) continue;
    const int64_t t = i / G;
    const int g = (int)(i - t * G);
    int32_t* ids = meta + (int64_t)s * 2 * topk;
    float* ws = reinterpret_cast<float*>(ids + topk);
    for (int j = 0; j < topk; ++j) {
      const int64_t e = topk_idx[t * topk + j];
      const bool here = e >= (int64_t)g * experts_per_rank && e < (int64_t)(g + 1) * experts_per_rank;
      ids[j] = here ? (int32_t)(e - (int64_t)g * experts_per_rank) : -1;
      ws[j] = here ? topk_w[t * topk + j] : 0.0f;
    }
  }
}

int grid_for(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (int)(b < 148 * 8 ? (b > 0 ? b : 1) : 148 * 8);
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_nccl_unique_id(void* id128) {
  MXB_REQUIRE(id128, MXB_ERR_INVALID_ARGUMENT, "nccl_unique_id: null pointer");
  MXB_REQUIRE(nccl().ok, MXB_ERR_UNSUPPORTED, "nccl_unique_id: libnccl.so.2 not found");
  ncclUniqueId id;
  MXB_NCCL(nccl().get_unique_id(&id), "ncclGetUniqueId");
  static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
  memcpy(id128, &id, sizeof(id));
  return MXB_OK;
}

extern "C" mxb_status mxb_nccl_comm_init(void** comm, int32_t world, int32_t rank,
                                         const void* id128) {
  MXB_REQUIRE(comm && id128 && world >= 1 && rank >= 0 && rank < world, MXB_ERR_INVALID_ARGUMENT,
              "nccl_comm_init: bad arguments");
  MXB_REQUIRE(nccl().ok, MXB_ERR_UNSUPPORTED, "nccl_comm_init: libnccl.so.2 not found");
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  ncclComm_t c = nullptr;
  MXB_NCCL(nccl().comm_init_rank(&c, world, id, rank), "ncclCommInitRank");
  *comm = c;
  return MXB_OK;
}

extern "C" mxb_status mxb_nccl_comm_destroy(void* comm) {
  MXB_REQUIRE(comm, MXB_ERR_INVALID_ARGUMENT, "nccl_comm_destroy: null communicator");
  MXB_REQUIRE(nccl().ok, MXB_ERR_UNSUPPORTED, "nccl_comm_destroy: libnccl.so.2 not found");
  MXB_NCCL(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
  return MXB_OK;
}

extern "C" int64_t mxb_ep_nccl_workspace_bytes(int64_t T, int32_t H, int32_t topk, int32_t world) {
  if (T < 0 || H <= 0 || topk <= 0 || world <= 0) return 0;
  return ws_layout(T, H, topk, world).total;
}

extern "C" mxb_status mxb_ep_nccl_dispatch(void* comm, int32_t world, int32_t rank, const void* x,
                                           int64_t T, int32_t H, const int64_t* topk_idx,
                                           const float* topk_w, int32_t topk,
                                           int32_t experts_per_rank, void* workspace,
                                           int64_t workspace_bytes, void* recv_wire,
                                           void* recv_meta, int64_t recv_cap,
                                           mxb_ep_handle* handle, mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_nccl_dispatch");
  MXB_REQUIRE(comm && handle && world >= 1 && world <= MXB_EP_MAX_WORLD && rank >= 0 &&
                  rank < world && T >= 0 && H > 0 && H % 128 == 0 && topk >= 1 &&
                  topk <= 32 && experts_per_rank >= 1 && recv_cap >= 0,
              MXB_ERR_INVALID_ARGUMENT, "ep_nccl_dispatch: bad arguments");
  MXB_REQUIRE(nccl().ok, MXB_ERR_UNSUPPORTED, "ep_nccl_dispatch: libnccl.so.2 not found");
  const NcclWs L = ws_layout(T, H, topk, world);
  MXB_REQUIRE(workspace && workspace_bytes >= L.total && aligned(workspace, 256),
              MXB_ERR_INVALID_ARGUMENT,
              "ep_nccl_dispatch: workspace must be 256-byte aligned and hold %lld bytes "
              "(mxb_ep_nccl_workspace_bytes)",
              (long long)L.total);
  MXB_REQUIRE(recv_cap == 0 || (recv_wire && recv_meta), MXB_ERR_INVALID_ARGUMENT,
              "ep_nccl_dispatch: null receive buffer");
  MXB_REQUIRE(T == 0 || (x && topk_idx && topk_w), MXB_ERR_INVALID_ARGUMENT,
              "ep_nccl_dispatch: null input");
  cudaStream_t s = to_cuda(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* within = reinterpret_cast<int32_t*>(ws + L.within);
  int32_t* slots = reinterpret_cast<int32_t*>(ws + L.slots);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);  // send [G], recv [G]
  uint8_t* wire = ws + L.wire;
  int32_t* meta = reinterpret_cast<int32_t*>(ws + L.meta);
  const int64_t rb = H / 2 + H / 32, mb = 8LL * topk;
  mxb_status st = mxb_ep_route(topk_idx, T, topk, experts_per_rank, world, within, counts, stream);
  if (st != MXB_OK) return st;
  if (T > 0) {
    slots_kernel<<<grid_for(T * world), 256, 0, s>>>(within, counts, T, world, slots);
    meta_kernel<<<grid_for(T * world), 256, 0, s>>>(slots, topk_idx, topk_w, T, world, topk,
                                                    experts_per_rank, meta);
    st = launch_status("ep_nccl_dispatch (slots)");
    if (st != MXB_OK) return st;
    st = mxb_ep_pack(x, T, H, slots, world, wire, 1e-10f, stream);
    if (st != MXB_OK) return st;
  }
  // per-peer row counts
  MXB_NCCL(nccl().group_start(), "ncclGroupStart");
  for (int g = 0; g < world; ++g) {
    nccl().send(counts + g, 1, ncclInt32, g, static_cast<ncclComm_t>(comm), s);
    nccl().recv(counts + world + g, 1, ncclInt32, g, static_cast<ncclComm_t>(comm), s);
  }
  MXB_NCCL(nccl().group_end(), "ncclGroupEnd (counts)");
  int32_t host[2 * MXB_EP_MAX_WORLD];
  MXB_REQUIRE(cudaMemcpyAsync(host, counts, 8 * world, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
                  cudaStreamSynchronize(s) == cudaSuccess,
              MXB_ERR_CUDA, "ep_nccl_dispatch: count read-back failed: %s",
              cudaGetErrorString(cudaGetLastError()));
  int64_t n_send = 0, n_recv = 0;
  for (int g = 0; g < world; ++g) {
    MXB_REQUIRE(host[world + g] >= 0 && host[world + g] <= (1LL << 30), MXB_ERR_INVALID_ARGUMENT,
                "ep_nccl_dispatch: impossible row count %d from rank %d", host[world + g], g);
    handle->send_counts[g] = host[g];
    handle->recv_counts[g] = host[world + g];
    n_send += host[g];
    n_recv += host[world + g];
  }
  handle->n_send = n_send;
  handle->n_recv = n_recv;
  handle->world = world;
  handle->rank = rank;
  handle->tokens = T;
  handle->hidden = H;
  handle->topk = topk;
  MXB_REQUIRE(n_recv <= recv_cap, MXB_ERR_INVALID_ARGUMENT,
              "ep_nccl_dispatch: %lld rows arrive but the receive buffers hold %lld",
              (long long)n_recv, (long long)recv_cap);
  // rows and metadata, grouped by source rank on the receive side
  MXB_NCCL(nccl().group_start(), "ncclGroupStart");
  int64_t so = 0, ro = 0;
  uint8_t* rw = static_cast<uint8_t*>(recv_wire);
  uint8_t* rm = static_cast<uint8_t*>(recv_meta);
  for (int g = 0; g < world; ++g) {
    const int64_t sc = handle->send_counts[g], rc = handle->recv_counts[g];
    if (sc > 0) {
      nccl().send(wire + so * rb, (size_t)(sc * rb), ncclUint8, g, static_cast<ncclComm_t>(comm), s);
      nccl().send(reinterpret_cast<uint8_t*>(meta) + so * mb, (size_t)(sc * mb), ncclUint8, g,
                  static_cast<ncclComm_t>(comm), s);
    }
    if (rc > 0) {
      nccl().recv(rw + ro * rb, (size_t)(rc * rb), ncclUint8, g, static_cast<ncclComm_t>(comm), s);
      nccl().recv(rm + ro * mb, (size_t)(rc * mb), ncclUint8, g, static_cast<ncclComm_t>(comm), s);
    }
    so += sc;
    ro += rc;
  }
  MXB_NCCL(nccl().group_end(), "ncclGroupEnd (rows)");
  return MXB_OK;
}

extern "C" mxb_status mxb_ep_nccl_combine(void* comm, const mxb_ep_handle* handle, const void* y,
                                          void* workspace, int64_t workspace_bytes, void* out,
                                          mxb_stream_t stream) {
  NvtxRange nvtx_range("mxb_ep_nccl_combine");
  MXB_REQUIRE(comm && handle && handle->world >= 1 && handle->world <= MXB_EP_MAX_WORLD,
              MXB_ERR_INVALID_ARGUMENT, "ep_nccl_combine: bad arguments");
  MXB_REQUIRE(nccl().ok, MXB_ERR_UNSUPPORTED, "ep_nccl_combine: libnccl.so.2 not found");
  const int G = handle->world;
  const int64_t T = handle->tokens, H = handle->hidden;
  const NcclWs L = ws_layout(T, H, handle->topk, G);
  MXB_REQUIRE(workspace && workspace_bytes >= L.total && aligned(workspace, 256),
              MXB_ERR_INVALID_ARGUMENT, "ep_nccl_combine: workspace too small or misaligned");
  MXB_REQUIRE((handle->n_recv == 0 || y) && (T == 0 || out), MXB_ERR_INVALID_ARGUMENT,
              "ep_nccl_combine: null pointer");
  cudaStream_t s = to_cuda(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* back = ws + L.back;
  const int32_t* slots = reinterpret_cast<const int32_t*>(ws + L.slots);
  const int64_t row = H * 2;
  MXB_NCCL(nccl().group_start(), "ncclGroupStart");
  int64_t so = 0, ro = 0;
  for (int g = 0; g < G; ++g) {
    const int64_t sc = handle->send_counts[g], rc = handle->recv_counts[g];
    if (rc > 0)
      nccl().send(static_cast<const uint8_t*>(y) + ro * row, (size_t)(rc * row), ncclUint8, g,
                  static_cast<ncclComm_t>(comm), s);
    if (sc > 0)
      nccl().recv(back + so * row, (size_t)(sc * row), ncclUint8, g, static_cast<ncclComm_t>(comm),
                  s);
    so += sc;
    ro += rc;
  }
  MXB_NCCL(nccl().group_end(), "ncclGroupEnd (combine)");
  if (T == 0) return MXB_OK;
  return mxb_ep_combine(back, T, H, slots, G, out, stream);
}
