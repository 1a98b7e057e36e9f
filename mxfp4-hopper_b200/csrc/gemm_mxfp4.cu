// Block-scaled MXFP4 GEMM on the 5th-generation tensor cores (sm_100a): the
// consumer on the far side of the quantize path.  C[M, N] (BF16) = A[M, K] .
// B[N, K]^T where A and B are MXFP4 exactly as this library's rowwise quantize
// writes them: E2M1 codes [rows, K/2] (element 2i in the low nibble) and E8M0
// scales in the 128x4-tile swizzled layout of mxb_swizzle_scales /
// scales_row_swizzled (the tcgen05 block-scale layout: a 512-byte atom holds
// the 4 scales of 128 rows, row r at (r % 32) * 16 + (r / 32) * 4).
//
// Persistent: one CTA per SM walks the 128 x 256 tiles of C (tile =
// blockIdx.x + i * gridDim.x, N-tiles fastest), each in one f32 accumulator in
// tensor memory (128 lanes x 256 columns); K walks 256-element steps through a
// 3-stage shared-memory ring that runs on across tile boundaries:
//   * warp 0 (one thread) lands each step's A tile (128 rows x 128 bytes), B
//     tile (256 rows x 128 bytes) with TMA (128-byte swizzle) and the step's
//     scale atoms (2 for A, 4 for B, 512 bytes each) with 1-D bulk copies,
//     completing on full[s]; it streams the next tile's steps while the
//     current tile's epilogue runs;
//   * warp 1 (one thread) waits for acc_empty (the accumulator read out), copies
//     the scale atoms into the stage's own tensor memory columns with
//     tcgen05.cp (32 rows x 16 bytes replicated to the four lane quadrants: 4
//     columns per atom; B's 128-row blocks of one K-atom sit in consecutive
//     column groups), issues 4 tcgen05.mma.kind::mxf4.block_scale.block32 of
//     128 x 256 x 64 per step (the scale byte pair of a K-half is selected by
//     the top two bits of the TMEM scale addresses) and commits them to
//     empty[s], which frees the stage when they have run; after a tile's last
//     step it commits to acc_full;
//   * warps 2..5 read the accumulator with tcgen05.ld, 64 columns per load
//     (warp w owns lane quadrant w % 4 = rows 32(w%4) .. +31), arrive on
//     acc_empty, convert to BF16 into a staging area of four 128-byte swizzled
//     boxes of 128 rows x 64 columns, and the tile leaves as four TMA stores
//     that drain while the next tile's MMAs run.
// Measured against one CTA per tile with a 4-stage ring (same epilogue, bytes
// identical): 257.5 -> 229.8 us at 8192 x 8192 x 7168, 191.7 -> 140.5 us at
// 16384 x 7168 x 2048.
// Descriptor formats follow the Blackwell UMMA descriptors (CUTLASS
// cute/arch/mma_sm100_desc.hpp).  Every wait is bounded; a CTA whose wait gives
// up records it, skips its stores and still releases its tensor memory.
#include <cuda_bf16.h>

#include <algorithm>

#include "capi_util.h"
#include "common.cuh"
#include "tma.cuh"

namespace mxb {
namespace {

constexpr int kGemmThreads = 192;                         // producer, MMA, 4 epilogue warps
constexpr int kTileM = 128, kTileN = 256, kTileK = 256;   // elements
constexpr int kStages = 3;
constexpr uint32_t kABytes = 128 * 128;                   // 128 rows x 128 code bytes
constexpr uint32_t kBBytes = 256 * 128;
constexpr uint32_t kSfaBytes = 2 * 512, kSfbBytes = 4 * 512;
constexpr uint32_t kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;  // 1024-multiple
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCol = 0;                           // accumulators: columns 0..255
constexpr uint32_t kSfCol = 256;                          // per stage: 8 SFA + 16 SFB columns
constexpr uint32_t kSfColsPerStage = 24;
// Epilogue staging of the bf16 tile beside the ring: four boxes of 128 rows x
// 64 columns (128-byte rows, TMA 128-byte swizzle).
constexpr uint32_t kCBoxBytes = 128 * 128;
constexpr size_t kGemmSmem = 1024 + kStages * kStageBytes + 4 * kCBoxBytes + 256;
static_assert(kGemmSmem <= 227 * 1024, "one CTA per SM");
static_assert(kSfCol + kStages * kSfColsPerStage <= kTmemCols, "scale columns fit in TMEM");

__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
  // K-major, 128-byte swizzle: 8-row atoms of 128-byte rows, SBO = 1024 B,
  // LBO = 16 B (unused for swizzled K-major), version 1, layout type 2
  const uint64_t a = (smem_addr(p) >> 4) & 0x3FFFu;
  return a | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

__device__ __forceinline__ uint64_t smem_desc_sf(const void* p) {
  // scale atom: 32 rows of 16 bytes, no swizzle: SBO = 128 B between 8-row
  // core matrices, LBO = 512 B, version 1, layout type 0
  const uint64_t a = (smem_addr(p) >> 4) & 0x3FFFu;
  return a | (uint64_t(512 >> 4) << 16) | (uint64_t(128 >> 4) << 32) | (uint64_t(1) << 46);
}

// Instruction descriptor of kind::mxf4 block_scale: E2M1 x E2M1, E8M0 scales,
// K-major A and B, M = 128, N = 256; sf ids in bits 4-5 (B) and 29-30 (A).
__host__ __device__ constexpr uint32_t gemm_idesc(uint32_t a_sf_id, uint32_t b_sf_id) {
  return (b_sf_id << 4) | (1u << 7) | (1u << 10) | (uint32_t(kTileN >> 3) << 17) | (1u << 23) |
         (uint32_t(kTileM >> 4) << 24) | (a_sf_id << 29);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_copy_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}"
      ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}
// 64 consecutive accumulator columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63"
      "}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]),
        "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]),
        "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]),
        "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]),
        "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_mxfp4_kernel(
    const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
    const __grid_constant__ CUtensorMap tmap_c, const uint8_t* __restrict__ sfa,
    const uint8_t* __restrict__ sfb, int64_t M, int64_t N, int64_t K,
    unsigned int* __restrict__ timeouts) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* cst = smem + kStages * kStageBytes;  // C staging: 4 boxes of 128 x 64 bf16
  uint64_t* full = reinterpret_cast<uint64_t*>(cst + 4 * kCBoxBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  int* failed = reinterpret_cast<int*>(tmem_base_slot + 1);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int ksteps = (int)(K / kTileK);
  const int64_t sp4 = K / 128;  // scale atoms per 128-row block along K
  const int ntn = (int)(N / kTileN);
  const int tiles = ntn * (int)(M / kTileM);
  const int my_tiles =
      (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (t == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    fence_mbar_init();
    *failed = 0;
  }
  if (warp == 0) {
    tmem_alloc(tmem_base_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;  // global K steps over this CTA's tiles
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        const int64_t m0 = (int64_t)(tile / ntn) * kTileM, n0 = (int64_t)(tile % ntn) * kTileN;
        for (int ks = 0; ks < ksteps; ++ks) {
          const int g = issued, s = g % kStages;
          if (g >= kStages && !mbar_wait(&empty[s], (uint32_t)((g / kStages - 1) & 1))) {
            atomicExch(failed, 1);
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          const int32_t kx = ks * (kTileK / 2);
          tma_load_2d(st, &tmap_a, kx, (int32_t)m0, &full[s]);
          tma_load_2d(st + kABytes, &tmap_b, kx, (int32_t)n0, &full[s]);
          tma_load_2d(st + kABytes + kABytes, &tmap_b, kx, (int32_t)(n0 + 128), &full[s]);
          uint8_t* ssf = st + kABytes + kBBytes;
          bulk_load_1d(ssf, sfa + ((m0 / 128) * sp4 + ks * 2) * 512, kSfaBytes, &full[s]);
          bulk_load_1d(ssf + kSfaBytes, sfb + ((n0 / 128) * sp4 + ks * 2) * 512, kSfaBytes,
                       &full[s]);
          bulk_load_1d(ssf + kSfaBytes + kSfaBytes, sfb + ((n0 / 128 + 1) * sp4 + ks * 2) * 512,
                       kSfaBytes, &full[s]);
          issued = g + 1;
        }
      }
      // do not leave while copies of this CTA are still landing
      for (int g = issued > kStages ? issued - kStages : 0; g < issued; ++g)
        mbar_wait(&full[g % kStages], (uint32_t)((g / kStages) & 1));
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      int g = 0;
      for (int i = 0; ok && i < my_tiles; ++i) {
        // the epilogue has read tile i-1's accumulator out of tensor memory
        if (i > 0 && !mbar_wait(acc_empty, (uint32_t)((i - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int ks = 0; ks < ksteps; ++ks, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(&full[s], (uint32_t)((g / kStages) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + s * kStageBytes;
          const uint8_t* ssf = st + kABytes + kBBytes;
          const uint32_t sfc = tmem + kSfCol + (uint32_t)(s * kSfColsPerStage);
#pragma unroll
          for (int a = 0; a < 2; ++a) tc_copy_sf(sfc + 4 * a, smem_desc_sf(ssf + a * 512));
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int a = 0; a < 2; ++a)
              tc_copy_sf(sfc + 8 + 8 * a + 4 * h,
                         smem_desc_sf(ssf + kSfaBytes + (2 * h + a) * 512));
          const uint64_t da = smem_desc_sw128(st);
          const uint64_t db = smem_desc_sw128(st + kABytes);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t sf_id = (uint32_t)(j & 1) * 2u;
            const uint32_t tsfa = (sfc + 4 * (j >> 1)) | (sf_id << 30);
            const uint32_t tsfb = (sfc + 8 + 8 * (j >> 1)) | (sf_id << 30);
            tc_mma(tmem + kAccCol, da + (uint64_t)(2 * j), db + (uint64_t)(2 * j),
                   gemm_idesc(sf_id, sf_id), tsfa, tsfb, (ks > 0 || j > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        tc_commit(acc_full);  // tile i's MMAs have completed when this arrives
      }
      if (!ok) atomicExch(failed, 1);
    }
  } else {
    // ------------------------------------------------ epilogue warps 2..5
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    for (int i = 0; i < my_tiles; ++i) {
      const bool ok = mbar_wait(acc_full, (uint32_t)(i & 1));
      tc_fence_after();
      const bool live = ok && !*((volatile int*)failed);
      // tile i-1's stores have read the staging boxes; the four warps leave
      // together if any of them saw a wait give up
      if (warp == 2 && lane == 0) bulk_wait_read_all();
      if (named_sync_or(1, 128, !live)) {
        if (lane == 0 && quad == 0) atomicAdd(timeouts, 1u);
        break;
      }
#pragma unroll 1
      for (int b = 0; b < kTileN / 64; ++b) {
        uint32_t v[64];
        tmem_ld64(tmem + kAccCol + ((uint32_t)(quad * 32) << 16) + (uint32_t)(64 * b), v);
        tmem_ld_wait();
        uint8_t* bx = cst + b * kCBoxBytes + r * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          uint32_t o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            o[q] = cvt_bf16x2(__uint_as_float(v[8 * k + 2 * q]),
                              __uint_as_float(v[8 * k + 2 * q + 1]));
          *reinterpret_cast<uint4*>(bx + ((k ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      // the accumulator is free for tile i+1's MMAs
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      fence_proxy_async_smem();
      named_sync(1, 128);
      if (warp == 2 && lane == 0) {
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        const int64_t m0 = (int64_t)(tile / ntn) * kTileM, n0 = (int64_t)(tile % ntn) * kTileN;
#pragma unroll
        for (int b = 0; b < kTileN / 64; ++b)
          tma_store_2d(&tmap_c, (int32_t)(n0 + 64 * b), (int32_t)m0, cst + b * kCBoxBytes);
        bulk_commit();
      }
    }
    if (warp == 2 && lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

__device__ unsigned int g_gemm_timeouts;

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" mxb_status mxb_gemm_mxfp4(const void* a_codes, const void* a_scales_swizzled,
                                     const void* b_codes, const void* b_scales_swizzled,
                                     int64_t M, int64_t N, int64_t K, void* c,
                                     mxb_stream_t stream) {
  MXB_REQUIRE(M >= 0 && N >= 0 && K >= 0 && M % kTileM == 0 && N % kTileN == 0 &&
                  K % kTileK == 0,
              MXB_ERR_INVALID_ARGUMENT,
              "gemm_mxfp4: need M %% 128, N %% 256 and K %% 256 == 0 (M=%lld N=%lld K=%lld)",
              (long long)M, (long long)N, (long long)K);
  if (M == 0 || N == 0) return MXB_OK;
  MXB_REQUIRE(a_codes && a_scales_swizzled && b_codes && b_scales_swizzled && c,
              MXB_ERR_INVALID_ARGUMENT, "gemm_mxfp4: null pointer");
  MXB_REQUIRE(aligned(a_codes, 16) && aligned(b_codes, 16) && aligned(a_scales_swizzled, 16) &&
                  aligned(b_scales_swizzled, 16) && aligned(c, 16),
              MXB_ERR_MISALIGNED, "gemm_mxfp4: operands must be 16-byte aligned");
  MXB_REQUIRE(K > 0, MXB_ERR_INVALID_ARGUMENT, "gemm_mxfp4: K must be positive");
  CUtensorMap ta, tb, tc;
  if (!make_tensor_map_2d(&ta, a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K / 2, K / 2, 128,
                          128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&tb, b_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, 128,
                          128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&tc, c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, N, N, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return MXB_ERR_CUDA;
  static const bool attr_ok =
      cudaFuncSetAttribute((const void*)gemm_mxfp4_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem) == cudaSuccess;
  MXB_REQUIRE(attr_ok, MXB_ERR_CUDA, "gemm_mxfp4: cannot reserve shared memory");
  unsigned int* timeouts = nullptr;
  MXB_REQUIRE(cudaGetSymbolAddress((void**)&timeouts, g_gemm_timeouts) == cudaSuccess, MXB_ERR_CUDA,
              "gemm_mxfp4: cannot find the timeout counter");
  // persistent: one CTA per SM walks tiles blockIdx.x, + gridDim.x, ...
  const int64_t tiles = (N / kTileN) * (M / kTileM);
  MXB_REQUIRE(tiles <= INT32_MAX, MXB_ERR_INVALID_ARGUMENT, "gemm_mxfp4: too many tiles");
  const int ctas = persistent_ctas((const void*)gemm_mxfp4_kernel, kGemmThreads, kGemmSmem);
  const dim3 grid((unsigned)std::min<int64_t>(tiles, ctas));
  gemm_mxfp4_kernel<<<grid, kGemmThreads, kGemmSmem, to_cuda(stream)>>>(
      ta, tb, tc, (const uint8_t*)a_scales_swizzled, (const uint8_t*)b_scales_swizzled, M, N, K,
      timeouts);
  return launch_status("gemm_mxfp4");
}

extern "C" unsigned int mxb_gemm_wait_timeouts(void) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_timeouts, sizeof(v));
  return v;
}
