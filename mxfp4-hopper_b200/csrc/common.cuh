// Shared device helpers for the sm_100a MXFP4 / FP8 kernels.
//
// Formats (the reference's wire layout, code/kernel/per_token_quant_mxfp4.cu:256
// and per_token_Mxfp4ToBf16_dequant.cu:22-27,137-151):
//   * MXFP4 code byte: element 2i in the low nibble, 2i+1 in the high nibble;
//     a nibble is s.ee.m (E2M1).
//   * E8M0 scale byte e means 2^(e-127); the reference decodes it as the BF16
//     bit pattern e<<7, so e = 0 reads as 0.0 and e = 255 as +Inf.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace mxb {

constexpr int kSMs = 148;  // B200: 2 dies x 74 SMs

// ---------------------------------------------------------------- memory
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_stream_u8(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
// Loads of data that neighbouring tiles read again soon (a tile's few bytes
// of a longer E8M0 row): kept in L2 with the evict-last priority, so that the
// sector is still there when the tiles beside it arrive.
__device__ __forceinline__ uint64_t l2_keep_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint32_t ld_keep_u32(const void* p, uint64_t pol) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;"
               : "=r"(r)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint2 ld_keep_v2(const void* p, uint64_t pol) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p), "l"(pol));
  return r;
}
// Streaming (evict-first) stores for outputs that are not re-read.
__device__ __forceinline__ void st_stream_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_stream_v2(void* p, uint2 v) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void st_stream_u32(void* p, uint32_t v) {
  asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_stream_f32(void* p, float v) {
  asm volatile("st.global.cs.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
__device__ __forceinline__ void st_stream_u8(void* p, uint32_t v) {
  asm volatile("st.global.cs.u8 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---------------------------------------------------------------- bit ops
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// Per-16-bit-lane unsigned maximum.
__device__ __forceinline__ uint32_t vmax_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// Per-byte unsigned maximum, built on the native 16-bit-lane max (the byte
// form vmax4 is a video instruction that sm_100 emulates with a long sequence:
// replacing it took the per-row FP8 converter from 111 to 79 us).
__device__ __forceinline__ uint32_t max_u8x4(uint32_t a, uint32_t b) {
  return vmax_u16x2(a & 0x00FF00FFu, b & 0x00FF00FFu) |
         (vmax_u16x2((a >> 8) & 0x00FF00FFu, (b >> 8) & 0x00FF00FFu) << 8);
}

// Per-lane max(|a|, |b|) of two BF16 pairs; a NaN in either input yields the
// canonical NaN 0x7FFF (whose magnitude sorts above Inf), so one instruction
// both reduces magnitudes and flags non-finite inputs.  The result's sign bits
// are meaningless (xorsign): mask them off before use.
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Tree reduction of N BF16 pairs with absmax_bf16x2 (depth log2 N).
template <int N>
__device__ __forceinline__ uint32_t absmax_tree(const uint32_t* w) {
  if constexpr (N == 1) {
    return w[0];
  } else {
    return absmax_bf16x2(absmax_tree<N / 2>(w), absmax_tree<N - N / 2>(w + N / 2));
  }
}

__device__ __forceinline__ float bf16lo_to_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// ---------------------------------------------------------------- conversions
// Four float pairs -> four E2M1x2 bytes, round-to-nearest-even, saturating to
// +-6 (Blackwell cvt.rn.satfinite.e2m1x2.f32).  v[2i] lands in the low nibble.
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float v[8]) {
  uint32_t r;
  asm("{\n"
      ".reg .b8 b0, b1, b2, b3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      "mov.b32 %0, {b0, b1, b2, b3};\n"
      "}"
      : "=r"(r)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return r;
}
// Two floats -> two E4M3 bytes (lo = a, hi = b), RNE, saturating to +-448;
// this is the conversion __nv_fp8_e4m3(float) performs on sm_89 and later.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}
// Two floats -> BF16x2 (lo = a, hi = b), RNE; NaN becomes canonical 0x7FFF.
__device__ __forceinline__ uint32_t cvt_bf16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// (a, b) * s for two floats given as bit patterns, one mul.rn.f32x2.
__device__ __forceinline__ void mul2_f32(uint32_t a, uint32_t b, float s, float& ra, float& rb) {
  asm("{\n .reg .b64 x, y;\n"
      " mov.b64 x, {%2, %3};\n"
      " mov.b64 y, {%4, %4};\n"
      " mul.rn.f32x2 x, x, y;\n"
      " mov.b64 {%0, %1}, x;\n}"
      : "=f"(ra), "=f"(rb)
      : "r"(a), "r"(b), "f"(s));
}

// (a, b) * (sa, sb), one mul.rn.f32x2; free of register moves when (a, b) and
// (sa, sb) already sit in register pairs (e.g. neighbouring outputs of one
// decode8_scaled and neighbouring words of one vector load).
__device__ __forceinline__ void mul2_f32_pairs(float a, float b, float sa, float sb, float& ra,
                                               float& rb) {
  asm("{\n .reg .b64 x, y;\n"
      " mov.b64 x, {%2, %3};\n"
      " mov.b64 y, {%4, %5};\n"
      " mul.rn.f32x2 x, x, y;\n"
      " mov.b64 {%0, %1}, x;\n}"
      : "=f"(ra), "=f"(rb)
      : "f"(a), "f"(b), "f"(sa), "f"(sb));
}

// ---------------------------------------------------------------- E2M1 decode
// BF16 bit patterns of the eight E2M1 magnitudes {0,.5,1,1.5,2,3,4,6}, split
// into byte tables so that `prmt` can look up four nibbles at once.
//   low bytes : 00 00 80 C0 00 40 80 C0
//   high bytes: 00 3F 3F 3F 40 40 40 40
constexpr uint32_t kE2m1Lo0 = 0xC0800000u, kE2m1Lo1 = 0xC0804000u;
constexpr uint32_t kE2m1Hi0 = 0x3F3F3F00u, kE2m1Hi1 = 0x40404040u;

// Decode the four nibbles in the low 16 bits of `w` into two BF16x2 words
// (unscaled E2M1 values, sign included): out0 = {e0, e1}, out1 = {e2, e3}.
// Bit-identical to the reference's shift/add decode
// (per_token_Mxfp4ToBf16_dequant.cu:137-151), including -0 for code 8.
__device__ __forceinline__ void e2m1x4_to_bf16x4(uint32_t w, uint32_t& out0, uint32_t& out1) {
  const uint32_t sel = w & 0x7777u;
  const uint32_t lo = prmt(kE2m1Lo0, kE2m1Lo1, sel);
  uint32_t hi = prmt(kE2m1Hi0, kE2m1Hi1, sel);
  // sign bits (bit 3 of each nibble) -> 0x80 in the matching high byte
  const uint32_t sgn = prmt(0x00008000u, 0u, ((w >> 3) & 0x1111u));
  hi |= sgn;
  out0 = prmt(lo, hi, 0x5140u);
  out1 = prmt(lo, hi, 0x7362u);
}

// Eight E2M1 codes (one code word: value i in nibble i) times the factor sf
// -> eight floats; with sf an E8M0 power of two these are exactly the
// reference's BF16 products widened:
// Blackwell's cvt.rn.f16x2.e2m1x2 decodes a code byte, the sm_100
// mixed-precision add.rn.f32.f16 widens each half (adding -0 keeps the sign of
// zero), and mul.rn.f32x2 scales by the power of two sf (exact; sf = 0 gives
// zeros, sf = Inf gives Inf or the NaN of 0 * Inf, as the BF16 product does).
__device__ __forceinline__ void decode8_scaled(uint32_t w, float sf, float (&o)[8]) {
  asm("{\n"
      ".reg .b8 b0, b1, b2, b3;\n"
      ".reg .b32 h0, h1, h2, h3;\n"
      ".reg .b16 p0, p1, p2, p3, p4, p5, p6, p7;\n"
      ".reg .f32 f0, f1, f2, f3, f4, f5, f6, f7;\n"
      ".reg .b64 x0, x1, x2, x3, s2;\n"
      "mov.b32 {b0, b1, b2, b3}, %8;\n"
      "cvt.rn.f16x2.e2m1x2 h0, b0;\n"
      "cvt.rn.f16x2.e2m1x2 h1, b1;\n"
      "cvt.rn.f16x2.e2m1x2 h2, b2;\n"
      "cvt.rn.f16x2.e2m1x2 h3, b3;\n"
      "mov.b32 {p0, p1}, h0;\n"
      "mov.b32 {p2, p3}, h1;\n"
      "mov.b32 {p4, p5}, h2;\n"
      "mov.b32 {p6, p7}, h3;\n"
      "add.rn.f32.f16 f0, p0, 0f80000000;\n"
      "add.rn.f32.f16 f1, p1, 0f80000000;\n"
      "add.rn.f32.f16 f2, p2, 0f80000000;\n"
      "add.rn.f32.f16 f3, p3, 0f80000000;\n"
      "add.rn.f32.f16 f4, p4, 0f80000000;\n"
      "add.rn.f32.f16 f5, p5, 0f80000000;\n"
      "add.rn.f32.f16 f6, p6, 0f80000000;\n"
      "add.rn.f32.f16 f7, p7, 0f80000000;\n"
      "mov.b64 s2, {%9, %9};\n"
      "mov.b64 x0, {f0, f1};\n"
      "mov.b64 x1, {f2, f3};\n"
      "mov.b64 x2, {f4, f5};\n"
      "mov.b64 x3, {f6, f7};\n"
      "mul.rn.f32x2 x0, x0, s2;\n"
      "mul.rn.f32x2 x1, x1, s2;\n"
      "mul.rn.f32x2 x2, x2, s2;\n"
      "mul.rn.f32x2 x3, x3, s2;\n"
      "mov.b64 {%0, %1}, x0;\n"
      "mov.b64 {%2, %3}, x1;\n"
      "mov.b64 {%4, %5}, x2;\n"
      "mov.b64 {%6, %7}, x3;\n"
      "}"
      : "=f"(o[0]), "=f"(o[1]), "=f"(o[2]), "=f"(o[3]), "=f"(o[4]), "=f"(o[5]), "=f"(o[6]),
        "=f"(o[7])
      : "r"(w), "f"(sf));
}

// Two floats per cvt: four E4M3 bytes of (a0, a1, b0, b1), RNE, saturating.
__device__ __forceinline__ uint32_t cvt_e4m3x4(float a0, float a1, float b0, float b1) {
  uint32_t r;
  asm("{\n .reg .b16 lo, hi;\n"
      " cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n"
      " cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n"
      " mov.b32 %0, {lo, hi};\n}"
      : "=r"(r)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
  return r;
}

// E8M0 byte -> float via the reference's BF16 reinterpretation.
__device__ __forceinline__ float e8m0_to_f(uint32_t e) { return __uint_as_float(e << 23); }

// Four code bytes (eight E2M1 codes) times the E8M0 factor of their block ->
// eight BF16 values (two per word, element 2i in the low half), exactly the
// reference's dequantize (per_token_Mxfp4ToBf16_dequant.cu:129-156): one exact
// BF16 multiply by 2^(e-127) for e in [2, 254], the float product rounded to
// BF16 for e in {0, 1, 255} (zero, the smallest binade, Inf / NaN).
__device__ __forceinline__ uint4 dq_bf16_chunk(uint32_t w, uint32_t e) {
  uint32_t o[4];
  e2m1x4_to_bf16x4(w, o[0], o[1]);
  e2m1x4_to_bf16x4(w >> 16, o[2], o[3]);
  if (e - 2u <= 252u) {  // e in [2, 254]: exact BF16 product
    const uint32_t s2 = (e << 7) | (e << 23);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = mul_bf16x2(o[i], s2);
  } else {
    const float s = e8m0_to_f(e);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = cvt_bf16x2(bf16lo_to_f(o[i]) * s, bf16hi_to_f(o[i]) * s);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__host__ __device__ __forceinline__ int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace mxb
