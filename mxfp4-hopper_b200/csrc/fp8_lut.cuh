// Compile-time lookup tables for the MXFP4 -> FP8 E4M3 converters.
//
// Both reference converters re-base each 32-element block onto a group
// exponent with 16-bit integer arithmetic on the BF16 pattern of the E2M1
// value, clamp to +-448 and round to E4M3:
//   row (per_token_Mxfp4ToFp8.cu:165-229):
//     adj = (uint16)(max_e - 6 - e);  a = (uint16)(bf16(code) - (adj << 7))
//     q = fmaxf(-448, fminf(448, a))            (NaN -> +448)
//   col (per_token_Mxfp4ToFp8_col.cu:195,218,241-290):
//     adj = (uint8)(max_e - 6 - e);   a = (uint16)(bf16(code) - (adj << 7)) & 0x7FFF
//     q = fminf(fmaxf(a, -448), 448)            (NaN -> -448)
// The result depends only on the nibble and on d = max_e - e (0..255), so
// each converter's arithmetic collapses into a 256 x 16 table of E4M3 bytes,
// generated here at compile time from those rules.  A row of the table (16
// bytes, one block's worth) then serves four nibbles per pair of `prmt`.
#pragma once
#include <cstdint>

namespace mxb {

struct Fp8Lut {
  uint8_t v[256][16];
};

// BF16 pattern of E2M1 nibble n, as the reference decodes it
// (per_token_Mxfp4ToBf16_dequant.cu:137-151).
constexpr uint32_t lut_e2m1_bf16(uint32_t n) {
  const uint32_t em = n & 7u;
  uint32_t x = (em << 6) | ((n & 8u) << 12);
  if (em & 6u) x += 126u << 7;
  if (em == 1u) x = 16128u | (x & 0x8000u);
  return x & 0xFFFFu;
}

// E4M3 (RNE, saturating) of a finite BF16 pattern whose magnitude is <= 448.
constexpr uint8_t lut_bf16_to_e4m3(uint32_t b) {
  const uint32_t sign = (b >> 8) & 0x80u;
  const int ex = (int)((b >> 7) & 0xFFu);
  const uint32_t man = b & 0x7Fu;
  if (ex == 0) return (uint8_t)sign;  // BF16 subnormals are far below 2^-10
  const int E = ex - 127;
  uint32_t code = 0;
  if (E >= -6) {
    uint32_t m3 = man >> 4, rem = man & 0xFu;
    int e8 = E + 7;
    if (rem > 8u || (rem == 8u && (m3 & 1u))) ++m3;
    if (m3 == 8u) { m3 = 0; ++e8; }
    code = ((uint32_t)e8 << 3) | m3;
    if (code > 0x7Eu) code = 0x7Eu;
  } else {
    // multiples of 2^-9: (128 + man) * 2^(E + 2), rounded to nearest even
    const int s = -(E + 2);  // >= 5
    if (s > 9) return (uint8_t)sign;
    const uint32_t v = 128u + man;
    uint32_t q = v >> s;
    const uint32_t rem = v & ((1u << s) - 1u), half = 1u << (s - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    code = q;
  }
  return (uint8_t)(sign | code);
}

// Clamp of a BF16 pattern to +-448 with the given NaN result; returns the
// BF16 pattern of the clamped value.
constexpr uint32_t lut_clamp448(uint32_t a, uint32_t nan_result) {
  const uint32_t mag = a & 0x7FFFu;
  if (mag > 0x7F80u) return nan_result;           // NaN
  if (mag > 0x43E0u) return (a & 0x8000u) | 0x43E0u;  // |a| > 448 (incl. Inf) -> +-448
  return a;
}

constexpr Fp8Lut make_fp8_lut(bool col) {
  Fp8Lut t{};
  for (uint32_t d = 0; d < 256; ++d) {
    for (uint32_t n = 0; n < 16; ++n) {
      const uint32_t x = lut_e2m1_bf16(n);
      uint32_t a = 0;
      if (!col) {
        const uint32_t adj = (d - 6u) & 0xFFFFu;
        a = (x - ((adj << 7) & 0xFFFFu)) & 0xFFFFu;
        a = lut_clamp448(a, 0x43E0u);  // fminf(448, NaN) = 448
      } else {
        const uint32_t adj = (d - 6u) & 0xFFu;
        a = ((x - (adj << 7)) & 0xFFFFu) & 0x7FFFu;
        a = lut_clamp448(a, 0xC3E0u);  // fmaxf(NaN, -448) = -448
      }
      t.v[d][n] = lut_bf16_to_e4m3(a);
    }
  }
  return t;
}

// The strict rowwise table: the true value e2m1(n) * 2^(6 - d) of a nibble
// re-based onto the group scale 2^(max_e - 6 - 127), rounded to E4M3 (RNE,
// values below half the smallest subnormal become a signed zero), instead of
// the reference's 16-bit re-basing, whose wrap turns zero codes (and tiny
// codes far below the group maximum) into +-448.  No reference counterpart.
constexpr Fp8Lut make_fp8_lut_strict() {
  Fp8Lut t{};
  for (uint32_t d = 0; d < 256; ++d) {
    for (uint32_t n = 0; n < 16; ++n) {
      const uint32_t em = n & 7u, sign = (n & 8u) << 4;
      if (em == 0u) {
        t.v[d][n] = (uint8_t)sign;
        continue;
      }
      // e2m1 magnitude = (1 + f/2) * 2^E0: em 1 -> 0.5, 2 -> 1, 3 -> 1.5, 4 -> 2,
      // 5 -> 3, 6 -> 4, 7 -> 6
      const int E0 = em == 1u ? -1 : (int)(em >> 1) - 1;
      const uint32_t half = (em >= 2u && (em & 1u)) ? 0x40u : 0u;
      const int E = E0 + 6 - (int)d;
      if (E + 127 < 1) {
        t.v[d][n] = (uint8_t)sign;
        continue;
      }
      const uint32_t bf = (sign << 8) | ((uint32_t)(E + 127) << 7) | half;
      t.v[d][n] = lut_bf16_to_e4m3(bf);
    }
  }
  return t;
}

// The col table ignores the nibble's sign bit (the reference masks bit 15 after
// the subtraction), so entries n and n | 8 coincide and 8 entries suffice.
constexpr bool col_lut_sign_free(const Fp8Lut& t) {
  for (int d = 0; d < 256; ++d)
    for (int n = 0; n < 8; ++n)
      if (t.v[d][n] != t.v[d][n | 8]) return false;
  return true;
}
static_assert(col_lut_sign_free(make_fp8_lut(true)), "col table must not depend on the sign bit");

// Four sign-free nibbles (low 16 bits of x) -> four E4M3 bytes from table
// entries 0-7 held in t0, t1.
__device__ __forceinline__ uint32_t lut_lookup4_nosign(uint32_t x, uint32_t t0, uint32_t t1) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(t0), "r"(t1), "r"(x & 0x7777u));
  return r;
}

// Four nibbles (low 16 bits of x) -> four E4M3 bytes through a 16-byte table
// row held in t0..t3 (entries 0-3, 4-7, 8-11, 12-15).
__device__ __forceinline__ uint32_t lut_lookup4(uint32_t x, uint32_t t0, uint32_t t1, uint32_t t2,
                                                uint32_t t3) {
  uint32_t lo, hi, m, r;
  const uint32_t sel = x & 0x7777u;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(lo) : "r"(t0), "r"(t1), "r"(sel));
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(t2), "r"(t3), "r"(sel));
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(m) : "r"(0x0000FF00u), "r"(0u), "r"((x >> 3) & 0x1111u));
  asm("lop3.b32 %0, %1, %2, %3, 0xD8;" : "=r"(r) : "r"(lo), "r"(hi), "r"(m));  // m ? hi : lo
  return r;
}

}  // namespace mxb
