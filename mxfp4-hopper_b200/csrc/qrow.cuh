// Q-row arithmetic shared by every kernel that quantizes BF16 to MXFP4 (the
// quantizers, the SwiGLU quantize and the EP dispatch kernels), so that one
// statement of the reference's scale rule and E2M1 rounding serves them all.
//
// Bit-exact contract (reference: code/kernel/per_token_quant_mxfp4.cu:121-266):
//   amax  = max(eps, max |x|) over a 1x32 block (32x1 for columnwise)
//   y_s   = exp2f(ceilf(log2f(max(amax / fp4_max, 1e-10))))
//   scale = (uint8)((int)log2f(y_s) + 127)
//   code  = E2M1_RNE(clamp(x * (1 / y_s), fp4_min, fp4_max)), sign kept on zero
// The fast path (scale_fast, encode8_*) is exact for fp4_max = 6,
// fp4_min = -6, 0 <= eps <= 6e-10 and finite blocks; the generic path
// evaluates the formula literally.  Why the fast path is exact is stated in
// quantize.cu's header.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace mxb {

struct QuantParams {
  float eps, fp4_min, fp4_max;
};

// ------------------------------------------------------------ generic path
// Reference E2M1 rounding of an already clamped float
// (per_token_quant_mxfp4.cu:213-256): re-bias the exponent from 127 to 1,
// denormalise values below 1.0 by a right shift, round to nearest even on the
// two retained bits, saturate at code 7, keep the sign in bit 3.
__device__ __forceinline__ uint32_t e2m1_encode_generic(float q) {
  const uint32_t b = __float_as_uint(q);
  const uint32_t sign = b >> 28 & 0x8u;
  uint32_t ex = (b >> 23) & 0xFFu;
  uint32_t man = b & 0x7FFFFFu;
  if (ex < 127u) {
    const uint32_t sh = 126u - ex;
    man = sh >= 32u ? 0u : ((0x400000u | (man >> 1)) >> sh);
  }
  ex = (ex > 126u ? ex : 126u) - 126u;
  const uint32_t m2 = man >> 21;
  const uint32_t inc = (m2 & 1u) & (((man & 0x1FFFFFu) != 0u) | ((m2 >> 1) & 1u));
  uint32_t r = (((ex << 2) | m2) + inc) >> 1;
  r = r > 7u ? 7u : r;
  return sign | r;
}

// The reference scale rule, evaluated literally.
__device__ __forceinline__ void scale_generic(float amax, const QuantParams& p, float& inv,
                                              uint32_t& byte) {
  float y = amax / p.fp4_max;
  y = exp2f(ceilf(log2f(fmaxf(y, 1e-10f))));
  const int t = (int)log2f(y);  // +Inf saturates to INT_MAX, as on the reference path
  byte = ((uint32_t)t + 127u) & 0xFFu;
  inv = 1.0f / y;
}

// 8 values given as float bit patterns -> one word of 8 E2M1 codes (element
// 2i in the low nibble of byte i), generic rounding.
__device__ __forceinline__ uint32_t encode8_generic(const uint32_t (&f)[8], float inv,
                                                    const QuantParams& p) {
  uint32_t r = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float q = fminf(fmaxf(__uint_as_float(f[j]) * inv, p.fp4_min), p.fp4_max);
    r |= e2m1_encode_generic(q) << (4 * j);
  }
  return r;
}

template <int N>
__device__ __forceinline__ float amax_generic(const uint32_t (&f)[N], float init) {
  float a = init;
#pragma unroll
  for (int i = 0; i < N; ++i) a = fmaxf(a, fabsf(__uint_as_float(f[i])));
  return a;
}

// ------------------------------------------------------------ fast path
// Exact scale exponent from the largest finite |x| pattern (see file header);
// inv = 2^-k as a BF16 bit pattern (127 - k lies in [2, 160]: always normal).
__device__ __forceinline__ void scale_fast(uint32_t mb, uint32_t& byte, uint32_t& inv) {
  int k = (int)(mb >> 7) - 129 + ((mb & 0x7Fu) > 0x40u ? 1 : 0);
  k = k < -33 ? -33 : k;
  byte = (uint32_t)(k + 127);
  inv = (uint32_t)(127 - k) << 7;
}

// ---- OCP scale rule (MX specification v1.0: shared exponent
// floor(log2(amax)) - emax(E2M1) with emax = 2), selectable instead of the
// reference rule.  amax = max(1e-10, max |x|) as on the reference path, so an
// all-zero block has exponent floor(log2(1e-10)) - 2 = -36 (byte 91).
// Fast path: a finite BF16 amax pattern mb = 1.m * 2^(E - 127) gives
// k = E - 129, and the 1e-10 floor is the clamp k >= -36.
__device__ __forceinline__ void scale_fast_ocp(uint32_t mb, uint32_t& byte, uint32_t& inv) {
  int k = (int)(mb >> 7) - 129;
  k = k < -36 ? -36 : k;
  byte = (uint32_t)(k + 127);
  inv = (uint32_t)(127 - k) << 7;
}
// Generic path of the OCP rule (amax already floored at eps and NaN-free, as
// fmaxf leaves it).  An infinite amax gives the E8M0 NaN byte 0xFF and inv = 0,
// so finite elements encode as signed zeros and infinite ones saturate.
__device__ __forceinline__ void scale_generic_ocp(float amax, float& inv, uint32_t& byte) {
  const uint32_t e = (__float_as_uint(amax) >> 23) & 0xFFu;
  if (e == 0xFFu) {
    byte = 0xFFu;
    inv = 0.0f;
    return;
  }
  const int k = (int)e - 129;
  byte = (uint32_t)(k + 127);
  inv = __uint_as_float((uint32_t)(127 - k) << 23);
}
// The rule chosen at compile time: kOcp selects the OCP rule.
template <bool kOcp>
__device__ __forceinline__ void scale_fast_rule(uint32_t mb, uint32_t& byte, uint32_t& inv) {
  if constexpr (kOcp) scale_fast_ocp(mb, byte, inv); else scale_fast(mb, byte, inv);
}
template <bool kOcp>
__device__ __forceinline__ void scale_generic_rule(float amax, const QuantParams& p, float& inv,
                                                   uint32_t& byte) {
  if constexpr (kOcp) scale_generic_ocp(amax, inv, byte); else scale_generic(amax, p, inv, byte);
}

// Eight BF16 values times the BF16 power of two `inv` -> one word of eight
// E2M1 codes (value i in nibble i).  Each product is formed by the sm_100
// mixed-precision fma.rn.f32.bf16 (a * b + -0 in f32), which widens and scales
// in one full-rate FMA-pipe instruction; the product of a BF16 value and a
// power of two is exact in f32 (or rounds once below its subnormal range,
// exactly like the reference's float multiply), and adding -0 keeps the sign
// of zero.  kLo / kHi pick which 16-bit half of each word holds the values:
//   encode8_pairs: words w[0..3], element order lo0, hi0, lo1, hi1, ...
//   encode8_half<kHi>: words w[0..7], value i = half kHi of w[i].
__device__ __forceinline__ uint32_t encode8_pairs(const uint32_t* w, uint32_t inv) {
  uint32_t r;
  asm("{\n"
      ".reg .b16 l0, h0, l1, h1, l2, h2, l3, h3, s, sx;\n"
      ".reg .f32 a0, b0, a1, b1, a2, b2, a3, b3;\n"
      ".reg .b8 c0, c1, c2, c3;\n"
      "mov.b32 {l0, h0}, %1;\n"
      "mov.b32 {l1, h1}, %2;\n"
      "mov.b32 {l2, h2}, %3;\n"
      "mov.b32 {l3, h3}, %4;\n"
      "mov.b32 {s, sx}, %5;\n"
      "fma.rn.f32.bf16 a0, l0, s, 0f80000000;\n"
      "fma.rn.f32.bf16 b0, h0, s, 0f80000000;\n"
      "fma.rn.f32.bf16 a1, l1, s, 0f80000000;\n"
      "fma.rn.f32.bf16 b1, h1, s, 0f80000000;\n"
      "fma.rn.f32.bf16 a2, l2, s, 0f80000000;\n"
      "fma.rn.f32.bf16 b2, h2, s, 0f80000000;\n"
      "fma.rn.f32.bf16 a3, l3, s, 0f80000000;\n"
      "fma.rn.f32.bf16 b3, h3, s, 0f80000000;\n"
      "cvt.rn.satfinite.e2m1x2.f32 c0, b0, a0;\n"
      "cvt.rn.satfinite.e2m1x2.f32 c1, b1, a1;\n"
      "cvt.rn.satfinite.e2m1x2.f32 c2, b2, a2;\n"
      "cvt.rn.satfinite.e2m1x2.f32 c3, b3, a3;\n"
      "mov.b32 %0, {c0, c1, c2, c3};\n"
      "}"
      : "=r"(r)
      : "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(inv));
  return r;
}

#define MXB_ENCODE8_HALF_BODY(MOVS)                                                      \
  asm("{\n"                                                                              \
      ".reg .b16 p0, x0, p1, x1, p2, x2, p3, x3, p4, x4, p5, x5, p6, x6, p7, x7, s, sx;\n" \
      ".reg .f32 v0, v1, v2, v3, v4, v5, v6, v7;\n"                                      \
      ".reg .b8 c0, c1, c2, c3;\n" MOVS                                                  \
      "mov.b32 {s, sx}, %9;\n"                                                           \
      "fma.rn.f32.bf16 v0, p0, s, 0f80000000;\n"                                         \
      "fma.rn.f32.bf16 v1, p1, s, 0f80000000;\n"                                         \
      "fma.rn.f32.bf16 v2, p2, s, 0f80000000;\n"                                         \
      "fma.rn.f32.bf16 v3, p3, s, 0f80000000;\n"                                         \
      "fma.rn.f32.bf16 v4, p4, s, 0f80000000;\n"                                         \
      "fma.rn.f32.bf16 v5, p5, s, 0f80000000;\n"                                         \
      "fma.rn.f32.bf16 v6, p6, s, 0f80000000;\n"                                         \
      "fma.rn.f32.bf16 v7, p7, s, 0f80000000;\n"                                         \
      "cvt.rn.satfinite.e2m1x2.f32 c0, v1, v0;\n"                                        \
      "cvt.rn.satfinite.e2m1x2.f32 c1, v3, v2;\n"                                        \
      "cvt.rn.satfinite.e2m1x2.f32 c2, v5, v4;\n"                                        \
      "cvt.rn.satfinite.e2m1x2.f32 c3, v7, v6;\n"                                        \
      "mov.b32 %0, {c0, c1, c2, c3};\n"                                                  \
      "}"                                                                                \
      : "=r"(r)                                                                          \
      : "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]),     \
        "r"(w[7]), "r"(inv))

template <bool kHi>
__device__ __forceinline__ uint32_t encode8_half(const uint32_t* w, uint32_t inv) {
  uint32_t r;
  if constexpr (kHi) {
    MXB_ENCODE8_HALF_BODY("mov.b32 {x0, p0}, %1;\n mov.b32 {x1, p1}, %2;\n mov.b32 {x2, p2}, %3;\n"
                          "mov.b32 {x3, p3}, %4;\n mov.b32 {x4, p4}, %5;\n mov.b32 {x5, p5}, %6;\n"
                          "mov.b32 {x6, p6}, %7;\n mov.b32 {x7, p7}, %8;\n");
  } else {
    MXB_ENCODE8_HALF_BODY("mov.b32 {p0, x0}, %1;\n mov.b32 {p1, x1}, %2;\n mov.b32 {p2, x2}, %3;\n"
                          "mov.b32 {p3, x3}, %4;\n mov.b32 {p4, x4}, %5;\n mov.b32 {p5, x5}, %6;\n"
                          "mov.b32 {p6, x6}, %7;\n mov.b32 {p7, x7}, %8;\n");
  }
  return r;
}
#undef MXB_ENCODE8_HALF_BODY

// Largest |x| BF16 pattern of the BF16 pairs in w; >= 0x7F80 when an Inf or
// NaN is present (NaN reduces to 0x7FFF).
template <int N>
__device__ __forceinline__ uint32_t max_abs_pairs(const uint32_t (&w)[N]) {
  const uint32_t m = absmax_tree<N>(w) & 0x7FFF7FFFu;
  return max(m & 0xFFFFu, m >> 16);
}

// Four BF16 pairs (8 consecutive elements) -> their float bit patterns.
__device__ __forceinline__ void unpack8(const uint32_t* w, uint32_t (&f)[8]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = w[j] << 16;
    f[2 * j + 1] = w[j] & 0xFFFF0000u;
  }
}

// Quantizes one 32-element block held as 16 BF16 pairs in element order.
template <bool kFast, bool kOcp = false>
__device__ __forceinline__ void quant_block32(const uint32_t (&w)[16], const QuantParams& p,
                                              uint32_t (&out)[4], uint32_t& byte) {
  const uint32_t mb = max_abs_pairs(w);
  if (kFast && mb < 0x7F80u) {
    uint32_t inv;
    scale_fast_rule<kOcp>(mb, byte, inv);
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = encode8_pairs(&w[4 * i], inv);
  } else {
    uint32_t fa[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t f[8];
      unpack8(&w[4 * i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) fa[8 * i + j] = f[j];
    }
    float inv;
    scale_generic_rule<kOcp>(amax_generic(fa, p.eps), p, inv, byte);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t f[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = fa[8 * i + j];
      out[i] = encode8_generic(f, inv, p);
    }
  }
}


}  // namespace mxb
