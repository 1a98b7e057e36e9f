// TMA (cp.async.bulk.tensor) and mbarrier helpers for sm_100a, plus the
// host-side tensor-map encoder.  Loads here never use .multicast::cluster: the
// tile always comes from this GPU's own memory into this CTA's shared memory.
//
// Every wait is bounded.  A wait that runs out increments the including
// file's g_mxb_wait_timeouts counter and the kernel abandons its remaining
// work after a second bounded wait for its own copies in flight.  Each
// translation unit that includes this header has its own counter (device code
// is not relocatable); a static registrar below adds a reader for it to the
// library-wide list that mxb_wait_timeouts() sums.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "capi_util.h"

namespace mxb {

// One counter per translation unit that uses these helpers.
static __device__ unsigned int g_mxb_wait_timeouts;

// Host: reads (and with `reset`, zeroes) this translation unit's counter on
// the current device; 0xFFFFFFFF if the read fails.
static unsigned int read_tu_wait_timeouts(bool reset) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_mxb_wait_timeouts, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset) {
    const unsigned int z = 0;
    if (cudaMemcpyToSymbol(g_mxb_wait_timeouts, &z, sizeof(z)) != cudaSuccess) return 0xFFFFFFFFu;
  }
  return v;
}
namespace {
const bool g_tu_wait_reader_registered = register_wait_timeout_reader(&read_tu_wait_timeouts);
}  // namespace

constexpr uint32_t kWaitSpins = 1u << 24;  // try_wait rounds before giving up

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) accesses to shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Returns true once the phase with the given parity has completed; false
// after kWaitSpins unsuccessful rounds (the timeout is recorded).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t i = 0; i < kWaitSpins; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  atomicAdd(&g_mxb_wait_timeouts, 1u);
  return false;
}

// 2-D tiled TMA load of box {x .. x+bx, y .. y+by} into shared memory,
// completion signalled on `bar` (complete_tx).  x * element size must be a
// multiple of 16 bytes; out-of-range elements are filled with zero.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// 1-D bulk copy of `bytes` contiguous bytes global -> shared, completion
// signalled on `bar` (complete_tx).  Both addresses 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 2-D tiled TMA store of a shared-memory box to global memory (bulk group).
// Elements outside the tensor are not written.  The writing threads must have
// executed fence_proxy_async_smem() and synchronised before this is issued.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int32_t x, int32_t y,
                                             const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(smem_addr(src))
      : "memory");
}
// 1-D bulk copy of `bytes` contiguous bytes shared -> global (bulk group).
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_store_1d(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(dst)),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until at most one committed bulk store group is still reading shared memory.
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Waits until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Barrier over the first `threads` threads of the CTA (named barrier `id`).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool named_sync_or(uint32_t id, uint32_t threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n"
      " bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

}  // namespace mxb
