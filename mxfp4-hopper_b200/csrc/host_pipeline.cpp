// Host-buffer entry point of the fused rowwise + columnwise quantize: the call a
// user with data in (pinned) host memory makes.  The work is cut into chunks of
// rows; three CUDA streams overlap chunk i's host->device copy, chunk i-1's
// quantize (mxb_quant_mxfp4_rowcol on the caller's stream) and chunk i-2's
// device->host copies, so a step costs about the larger of the two PCIe
// directions instead of their sum (the link is full duplex).  Two device
// buffers per direction alternate between chunks; the caller provides them as
// one workspace.  Column outputs are [K, chunk/2] per chunk on the device and
// land at column offset r0/2 of the host [K, M/2] matrix through pitched copies.
#include <cuda_runtime.h>

#include <mutex>

#include "capi_util.h"
#include "mxfp4_b200.h"

namespace mxb {
namespace {

constexpr int kBufs = 2;
constexpr int kMaxDevices = 64;

// Per-device copy streams and events, created on first use and kept for the
// life of the process; the mutex serialises the enqueue sequences of calls.
struct PipelineState {
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t start = nullptr, in[kBufs] = {}, out[kBufs] = {}, free_[kBufs] = {};
  bool ok = false;
};
std::mutex g_mu;
PipelineState g_state[kMaxDevices];

bool state_for(int dev, PipelineState*& st) {
  if (dev < 0 || dev >= kMaxDevices) return false;
  PipelineState& s = g_state[dev];
  if (!s.ok) {
    const unsigned fl = cudaEventDisableTiming;
    bool good = cudaStreamCreateWithFlags(&s.h2d, cudaStreamNonBlocking) == cudaSuccess &&
                cudaStreamCreateWithFlags(&s.d2h, cudaStreamNonBlocking) == cudaSuccess &&
                cudaEventCreateWithFlags(&s.start, fl) == cudaSuccess;
    for (int b = 0; good && b < kBufs; ++b)
      good = cudaEventCreateWithFlags(&s.in[b], fl) == cudaSuccess &&
             cudaEventCreateWithFlags(&s.out[b], fl) == cudaSuccess &&
             cudaEventCreateWithFlags(&s.free_[b], fl) == cudaSuccess;
    if (!good) return false;
    s.ok = true;
  }
  st = &s;
  return true;
}

// Device bytes of one chunk buffer set (input + the four outputs).
int64_t chunk_bytes(int64_t R, int64_t K) {
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  return up(R * K * 2) + up(R * K / 2) + up(R * K / 32) + up(K * R / 2) + up(K * R / 32);
}

int64_t default_chunk(int64_t M) {
  int64_t R = 1024;
  while (R > 128 && R > M) R /= 2;
  return R;
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" int64_t mxb_quant_mxfp4_rowcol_host_workspace(int64_t M, int64_t K, int64_t chunk_rows) {
  if (M <= 0 || K <= 0) return 0;
  const int64_t R = chunk_rows > 0 ? chunk_rows : default_chunk(M);
  return kBufs * chunk_bytes(R, K);
}

extern "C" mxb_status mxb_quant_mxfp4_rowcol_host(const void* x_host, int64_t M, int64_t K,
                                                  void* codes_row_host, void* scales_row_host,
                                                  void* codes_col_host, void* scales_col_host,
                                                  void* workspace, int64_t workspace_bytes,
                                                  int64_t chunk_rows, float eps, float fp4_min,
                                                  float fp4_max, mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && K >= 0 && M % 32 == 0 && K % 32 == 0, MXB_ERR_INVALID_ARGUMENT,
              "quant_rowcol_host: need M %% 32 == 0 and K %% 32 == 0 (M=%lld K=%lld)",
              (long long)M, (long long)K);
  MXB_REQUIRE(chunk_rows >= 0 && chunk_rows % 128 == 0, MXB_ERR_INVALID_ARGUMENT,
              "quant_rowcol_host: chunk_rows must be 0 (default) or a multiple of 128");
  if (M == 0 || K == 0) return MXB_OK;
  MXB_REQUIRE(x_host && codes_row_host && scales_row_host && codes_col_host && scales_col_host &&
                  workspace,
              MXB_ERR_INVALID_ARGUMENT, "quant_rowcol_host: null pointer");
  const int64_t R = chunk_rows > 0 ? chunk_rows : default_chunk(M);
  const int64_t per = chunk_bytes(R, K);
  MXB_REQUIRE(workspace_bytes >= kBufs * per, MXB_ERR_INVALID_ARGUMENT,
              "quant_rowcol_host: workspace of %lld bytes is smaller than the %lld needed "
              "(mxb_quant_mxfp4_rowcol_host_workspace)",
              (long long)workspace_bytes, (long long)(kBufs * per));
  MXB_REQUIRE(aligned(workspace, 256), MXB_ERR_MISALIGNED,
              "quant_rowcol_host: workspace must be 256-byte aligned");
  NvtxRange nvtx_call("mxb_quant_mxfp4_rowcol_host");
  int dev = 0;
  MXB_REQUIRE(cudaGetDevice(&dev) == cudaSuccess, MXB_ERR_CUDA, "quant_rowcol_host: no device");
  std::lock_guard<std::mutex> lk(g_mu);
  PipelineState* st = nullptr;
  MXB_REQUIRE(state_for(dev, st), MXB_ERR_CUDA, "quant_rowcol_host: cannot create streams/events");
  cudaStream_t cs = to_cuda(stream);
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  auto fail = [](const char* what) {
    set_error("quant_rowcol_host: %s failed: %s", what, cudaGetErrorString(cudaGetLastError()));
    return MXB_ERR_CUDA;
  };
  // work already on the caller's stream (e.g. earlier users of the workspace) first
  if (cudaEventRecord(st->start, cs) != cudaSuccess ||
      cudaStreamWaitEvent(st->h2d, st->start, 0) != cudaSuccess ||
      cudaStreamWaitEvent(st->d2h, st->start, 0) != cudaSuccess)
    return fail("stream ordering");
  const uint8_t* xh = static_cast<const uint8_t*>(x_host);
  uint8_t* crh = static_cast<uint8_t*>(codes_row_host);
  uint8_t* srh = static_cast<uint8_t*>(scales_row_host);
  uint8_t* cch = static_cast<uint8_t*>(codes_col_host);
  uint8_t* sch = static_cast<uint8_t*>(scales_col_host);
  int i = 0;
  for (int64_t r0 = 0; r0 < M; r0 += R, ++i) {
    const int64_t rows = M - r0 < R ? M - r0 : R;
    const int b = i % kBufs;
    NvtxRange nvtx_chunk("rowcol_host chunk");
    uint8_t* base = static_cast<uint8_t*>(workspace) + b * per;
    uint8_t* xd = base;
    uint8_t* crd = xd + up(R * K * 2);
    uint8_t* srd = crd + up(R * K / 2);
    uint8_t* ccd = srd + up(R * K / 32);
    uint8_t* scd = ccd + up(K * R / 2);
    // buffer b is free once chunk i - kBufs's output copies have finished
    if (cudaStreamWaitEvent(st->h2d, st->free_[b], 0) != cudaSuccess ||
        cudaMemcpyAsync(xd, xh + r0 * K * 2, rows * K * 2, cudaMemcpyHostToDevice, st->h2d) !=
            cudaSuccess ||
        cudaEventRecord(st->in[b], st->h2d) != cudaSuccess ||
        cudaStreamWaitEvent(cs, st->in[b], 0) != cudaSuccess)
      return fail("input copy");
    const mxb_status qs = mxb_quant_mxfp4_rowcol(xd, rows, K, K, crd, srd, ccd, scd, nullptr, eps,
                                                 fp4_min, fp4_max, stream);
    if (qs != MXB_OK) return qs;
    if (cudaEventRecord(st->out[b], cs) != cudaSuccess ||
        cudaStreamWaitEvent(st->d2h, st->out[b], 0) != cudaSuccess ||
        cudaMemcpyAsync(crh + r0 * K / 2, crd, rows * K / 2, cudaMemcpyDeviceToHost, st->d2h) !=
            cudaSuccess ||
        cudaMemcpyAsync(srh + r0 * K / 32, srd, rows * K / 32, cudaMemcpyDeviceToHost, st->d2h) !=
            cudaSuccess ||
        cudaMemcpy2DAsync(cch + r0 / 2, M / 2, ccd, rows / 2, rows / 2, K, cudaMemcpyDeviceToHost,
                          st->d2h) != cudaSuccess ||
        cudaMemcpy2DAsync(sch + r0 / 32, M / 32, scd, rows / 32, rows / 32, K,
                          cudaMemcpyDeviceToHost, st->d2h) != cudaSuccess ||
        cudaEventRecord(st->free_[b], st->d2h) != cudaSuccess)
      return fail("output copies");
  }
  // the caller's stream reaches its end only after the last output copy
  if (cudaEventRecord(st->start, st->d2h) != cudaSuccess ||
      cudaStreamWaitEvent(cs, st->start, 0) != cudaSuccess)
    return fail("completion ordering");
  return MXB_OK;
}
