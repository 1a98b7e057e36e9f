/*
 * mxfp4_oracle.c -- TEST INFRASTRUCTURE ONLY (the parity checker, never the product).
 *
 * A plain-C, single-source restatement of the reference's MXFP4 quantize /
 * dequantize / convert kernels (anonymous-git-2026/MXFP4-Hopper, code/kernel/).
 * Every function follows the integer and IEEE-float arithmetic of the
 * reference kernel it names, quirks included, so that its outputs are the
 * bit-exact expectation for the CUDA kernels of this repository.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.
 *
 * Parity pin: the restatement is checked against the reference kernels
 * themselves, compiled unmodified from the reference sources
 * (oracle/build_ref.py) and run on a B200, through golden fixtures committed
 * under tests/golden/ (generator: tests/golden/make_golden.py).  The per-token
 * FP8 functions have no reference kernel; they follow the reference's only FP8
 * convention (per_token_Mxfp4RowToBf16ToFp8Col.cu:142,161,173-177) and are
 * "parity unpinned".
 *
 * Build: see oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).  No
 * fast-math: every float operation must round exactly as the GPU's IEEE path.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ helpers */

static inline float f_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_from_f(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf16_to_f(uint16_t h) { return f_from_bits((uint32_t)h << 16); }

/* float -> bf16, round to nearest even; every NaN becomes the canonical 0x7FFF
 * (the result of the GPU's cvt.rn.bf16x2.f32 used by __floats2bfloat162_rn). */
uint16_t orc_f32_to_bf16(float f) {
  uint32_t u = bits_from_f(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFF;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* float -> FP8 E4M3 (OCP "fn" variant: no infinities, S.1111.111 is NaN),
 * round to nearest even, saturating to +-448 like cvt.rn.satfinite.e4m3x2.f32
 * (what __nv_fp8_e4m3(float) lowers to on sm_89 and later). */
uint8_t orc_f32_to_e4m3(float f) {
  uint32_t u = bits_from_f(f);
  uint8_t s = (uint8_t)((u >> 24) & 0x80u);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint8_t)(s | 0x7F);
  double v = fabs((double)f);
  if (v >= 448.0) return (uint8_t)(s | 0x7E);
  if (v < 0.015625) { /* below the smallest normal 2^-6: multiples of 2^-9 */
    double q = nearbyint(v * 512.0);
    return (uint8_t)(s | (uint8_t)q);
  }
  int e2;
  (void)frexp(v, &e2);
  int ex = e2 - 1; /* v = 1.f * 2^ex, ex in [-6, 8] */
  double q = nearbyint(ldexp(v, 3 - ex)); /* in [8, 16] */
  if (q >= 16.0) { q = 8.0; ex += 1; }
  unsigned code = (unsigned)(((ex + 7) << 3) | ((int)q - 8));
  if (code > 0x7E) code = 0x7E;
  return (uint8_t)(s | code);
}

float orc_e4m3_to_f32(uint8_t c) {
  int s = c >> 7, e = (c >> 3) & 0xF, m = c & 7;
  float v;
  if (e == 0xF && m == 7) return f_from_bits(0x7FC00000u | ((uint32_t)s << 31));
  if (e == 0) v = ldexpf((float)m, -9);
  else v = ldexpf((float)(8 + m), e - 10);
  return s ? -v : v;
}

/* E2M1 nibble -> BF16 bit pattern, as the reference decodes it
 * (per_token_Mxfp4ToBf16_dequant.cu:137-151): exponent/mantissa shifted into
 * place, bias 126 added for normal codes, code 1 (0.5) special-cased. */
static inline uint16_t e2m1_to_bf16_bits(unsigned nib) {
  unsigned em = nib & 7u;
  uint16_t x = (uint16_t)((em << 6) | ((nib & 8u) << 12));
  if (em & 6u) x = (uint16_t)(x + (126u << 7));
  if (em == 1u) x = (uint16_t)(16128u | (x & 0x8000u));
  return x;
}

/* E8M0 byte -> float through the reference's BF16 reinterpretation
 * (per_token_Mxfp4ToBf16_dequant.cu:22-27): 0 -> 0.0, 255 -> +Inf. */
static inline float e8m0_to_f(uint8_t e) { return f_from_bits((uint32_t)e << 23); }

/* Reference E2M1 encode of an already clamped float q
 * (per_token_quant_mxfp4.cu:213-256): sign bit moved to bit 3, exponent
 * re-biased from 127 to 1 with values below 1.0 denormalised by a right
 * shift, then round-to-nearest-even on the two retained bits. */
static inline uint8_t e2m1_encode_ref(float q) {
  uint32_t b = bits_from_f(q);
  uint32_t sign = b & 0x80000000u;
  uint32_t ex = (b >> 23) & 0xFFu;
  uint32_t man = b & 0x7FFFFFu;
  if (ex < 127u) { /* shift uses unsigned wrap exactly as the reference */
    uint32_t sh = 127u - (ex + 1u);
    man = (sh >= 32u) ? 0u : ((0x400000u | (man >> 1)) >> sh);
  }
  ex = (ex > 126u ? ex : 126u) - 126u;
  uint32_t m2 = man >> 21;
  uint32_t lsb = (m2 >> 1) & 1u, guard = m2 & 1u, sticky = (man & 0x1FFFFFu) != 0u;
  uint32_t r = (((ex << 2) | m2) + (guard & (sticky | lsb))) >> 1;
  if (r > 7u) r = 7u;
  return (uint8_t)((sign >> 28) | r);
}

/* The reference's shared-scale rule (per_token_quant_mxfp4.cu:185-196):
 * y_s = exp2f(ceilf(log2f(max(amax / fp4_max, 1e-10)))), stored as
 * (uint8)((int)log2f(y_s) + 127).  Restated with exact exponent arithmetic
 * (ceil(log2 y) from y's bits); an infinite y_s stores byte 126, the value the
 * GPU's saturating float->int conversion produces for log2f(+Inf). */
static inline void scale_rule_ref(float amax, float fp4_max, float* y_s, uint8_t* byte) {
  float y = amax / fp4_max;
  y = fmaxf(y, 1e-10f);
  int k;
  if (isinf(y)) {
    *y_s = INFINITY; *byte = 126; return;
  }
  {
    uint32_t b = bits_from_f(y);
    int ex = (int)((b >> 23) & 0xFFu);
    uint32_t man = b & 0x7FFFFFu;
    k = ex - 127 + (man != 0u); /* y >= 1e-10 is always normal */
  }
  if (k >= 128) { *y_s = INFINITY; *byte = 126; return; }
  *y_s = ldexpf(1.0f, k);
  *byte = (uint8_t)(k + 127);
}

/* The OCP MX shared-exponent rule, a selectable alternative to the reference
 * rule (no reference counterpart; OCP Microscaling Formats spec v1.0, section
 * 6.3): X = 2^(floor(log2(amax)) - emax) with emax = 2 for E2M1, amax floored
 * at eps = 1e-10 as on the reference path.  An infinite amax gives the E8M0
 * NaN byte 0xFF and a zero multiplier.  Returns the multiplier 1/X. */
static inline float scale_rule_ocp(float amax, uint8_t* byte) {
  uint32_t e = (bits_from_f(amax) >> 23) & 0xFFu;
  if (e == 0xFFu) { *byte = 0xFF; return 0.0f; }
  int k = (int)e - 127 - 2; /* amax >= 1e-10 is normal */
  *byte = (uint8_t)(k + 127);
  return ldexpf(1.0f, -k);
}

/* One 1x32 block (values v[0..31]) under the reference rule (ocp = 0) or the
 * OCP rule (ocp = 1, with the reference API's eps and clamp). */
static inline void quant_block(const float* v, float eps, float fp4_min, float fp4_max, int ocp,
                               uint8_t* cb, uint8_t* sb) {
  float amax = eps;
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  float inv;
  if (ocp) {
    inv = scale_rule_ocp(amax, sb);
  } else {
    float y_s;
    scale_rule_ref(amax, fp4_max, &y_s, sb);
    inv = 1.0f / y_s;
  }
  for (int i = 0; i < 16; ++i) {
    float q0 = fminf(fmaxf(v[2 * i] * inv, fp4_min), fp4_max);
    float q1 = fminf(fmaxf(v[2 * i + 1] * inv, fp4_min), fp4_max);
    cb[i] = (uint8_t)((e2m1_encode_ref(q0) & 0x0F) | ((e2m1_encode_ref(q1) & 0x0F) << 4));
  }
}

/* ----------------------------------------------------------- Q-row (C1) */
/* Rowwise BF16 -> MXFP4 quantize, 1x32 blocks (per_token_quant_mxfp4.cu:121-266:
 * amax :151,171-178, scale :183-196, clamp and encode :200-256).
 * x: [M, K] bf16 bits, row stride ldx elements; codes: [M, K/2]; scales: [M, K/32]. */
static void quant_rows(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, float eps,
                       float fp4_min, float fp4_max, int ocp, uint8_t* codes, uint8_t* scales) {
  const int64_t G = K / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < G; ++g) {
      float v[32];
      for (int i = 0; i < 32; ++i) v[i] = bf16_to_f(x[r * ldx + g * 32 + i]);
      quant_block(v, eps, fp4_min, fp4_max, ocp, codes + r * (K / 2) + g * 16, scales + r * G + g);
    }
  }
}

/* Columnwise quantize: the reference applies Q-row to tensor.T.contiguous()
 * (transformer_engine-2.8.diff:1465-1466), so a block is 32 consecutive rows
 * of one column.  codes_t: [K, M/2]; scales_t: [K, M/32]. */
static void quant_cols(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, float eps,
                       float fp4_min, float fp4_max, int ocp, uint8_t* codes_t, uint8_t* scales_t) {
  const int64_t G = M / 32;
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < K; ++c) {
    for (int64_t g = 0; g < G; ++g) {
      float v[32];
      for (int i = 0; i < 32; ++i) v[i] = bf16_to_f(x[(g * 32 + i) * ldx + c]);
      quant_block(v, eps, fp4_min, fp4_max, ocp, codes_t + c * (M / 2) + g * 16,
                  scales_t + c * G + g);
    }
  }
}

void orc_quant_mxfp4_rows(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, float eps,
                          float fp4_min, float fp4_max, uint8_t* codes, uint8_t* scales) {
  quant_rows(x, M, K, ldx, eps, fp4_min, fp4_max, 0, codes, scales);
}
void orc_quant_mxfp4_cols(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, float eps,
                          float fp4_min, float fp4_max, uint8_t* codes_t, uint8_t* scales_t) {
  quant_cols(x, M, K, ldx, eps, fp4_min, fp4_max, 0, codes_t, scales_t);
}
/* The same two under the OCP scale rule (eps 1e-10, clamp +-6). */
void orc_quant_mxfp4_rows_ocp(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                              uint8_t* codes, uint8_t* scales) {
  quant_rows(x, M, K, ldx, 1e-10f, -6.0f, 6.0f, 1, codes, scales);
}
void orc_quant_mxfp4_cols_ocp(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                              uint8_t* codes_t, uint8_t* scales_t) {
  quant_cols(x, M, K, ldx, 1e-10f, -6.0f, 6.0f, 1, codes_t, scales_t);
}

/* Swizzled scale layout used by tcgen05 block-scaled MMA and cuBLAS
 * (128x4 tiles, transformer_engine-2.8.diff:752-786): scale (r, c) of an
 * [M, S] row-major scale matrix lands at byte
 *   ((r/128) * ceil(S/4) + c/4) * 512 + (r%32)*16 + ((r%128)/32)*4 + c%4
 * of an [round_up(M,128), round_up(S,4)] buffer; padding bytes are zero. */
void orc_swizzle_scales(const uint8_t* s, int64_t M, int64_t S, uint8_t* out) {
  const int64_t Mp = (M + 127) / 128 * 128, Sp = (S + 3) / 4 * 4;
  memset(out, 0, (size_t)(Mp * Sp));
  for (int64_t r = 0; r < M; ++r)
    for (int64_t c = 0; c < S; ++c) {
      int64_t off = ((r / 128) * (Sp / 4) + c / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + c % 4;
      out[off] = s[r * S + c];
    }
}

/* ---------------------------------------------------------- DQ-bf16 (C2) */
/* MXFP4 -> BF16 (per_token_Mxfp4ToBf16_dequant.cu:129-156): decoded code times
 * the E8M0 scale as float, rounded to BF16.  codes: [M, Kb] bytes (2*Kb
 * elements per row), scales: [M, 2*Kb/32]; out: [M, 2*Kb] bf16 bits. */
void orc_dequant_bf16(const uint8_t* codes, const uint8_t* scales, int64_t M, int64_t Kb,
                      uint16_t* out) {
  const int64_t S = 2 * Kb / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t b = 0; b < Kb; ++b) {
      uint8_t v = codes[r * Kb + b];
      float sc = e8m0_to_f(scales[r * S + (2 * b) / 32]);
      float lo = bf16_to_f(e2m1_to_bf16_bits(v & 0xFu)) * sc;
      float hi = bf16_to_f(e2m1_to_bf16_bits(v >> 4)) * sc;
      out[r * 2 * Kb + 2 * b] = orc_f32_to_bf16(lo);
      out[r * 2 * Kb + 2 * b + 1] = orc_f32_to_bf16(hi);
    }
  }
}

/* Element value of the reference's MXFP4 -> FP8 exponent re-basing
 * (per_token_Mxfp4ToFp8.cu:191-229): BF16 bits of the code minus
 * (adj << 7) in 16-bit arithmetic, then clamped to +-448 (min first) and
 * converted to E4M3. */
static inline uint8_t fp8_from_rebased_row(unsigned nib, uint16_t adj) {
  uint16_t x = e2m1_to_bf16_bits(nib);
  uint16_t off = (uint16_t)(adj << 7);
  uint16_t a = (uint16_t)(x - off);
  float q = bf16_to_f(a);
  q = fmaxf(-448.0f, fminf(448.0f, q));
  return orc_f32_to_e4m3(q);
}

/* ------------------------------------------------------- DQ-fp8-row (C3) */
/* MXFP4 -> FP8 E4M3 with 1x128 groups (per_token_Mxfp4ToFp8.cu:157-233).
 * Group exponent g = (uint16)(max of the 4 E8M0 bytes - 6); group scale
 * float bits ((uint8)g) << 23 written to scales_out[(group col) * M + row].
 * codes: [M, Kb] with Kb % 64 == 0; scales: [M, Kb/16]; out: [M, 2*Kb];
 * scales_out: [Kb/64, M] float. */
void orc_mxfp4_to_fp8_rows(const uint8_t* codes, const uint8_t* scales, int64_t M, int64_t Kb,
                           uint8_t* out, float* scales_out) {
  const int64_t S = Kb / 16, NG = Kb / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < NG; ++g) {
      const uint8_t* sp = scales + r * S + g * 4;
      uint8_t mx = sp[0];
      for (int j = 1; j < 4; ++j) mx = sp[j] > mx ? sp[j] : mx;
      uint16_t ge = (uint16_t)((int)mx - 6);
      scales_out[g * M + r] = f_from_bits((uint32_t)(uint8_t)ge << 23);
      for (int j = 0; j < 4; ++j) {
        uint16_t adj = (uint16_t)((int)ge - (int)sp[j]);
        const uint8_t* cb = codes + r * Kb + g * 64 + j * 16;
        uint8_t* ob = out + r * 2 * Kb + g * 128 + j * 32;
        for (int b = 0; b < 16; ++b) {
          ob[2 * b] = fp8_from_rebased_row(cb[b] & 0xFu, adj);
          ob[2 * b + 1] = fp8_from_rebased_row(cb[b] >> 4, adj);
        }
      }
    }
  }
}

/* The rowwise convert without the re-basing wrap (no reference counterpart):
 * the same group scale, each element its true value e2m1 * 2^(e - g - 127)
 * with g = max e - 6, rounded to E4M3 (RNE, saturating; underflow gives a
 * signed zero). */
void orc_mxfp4_to_fp8_rows_strict(const uint8_t* codes, const uint8_t* scales, int64_t M,
                                  int64_t Kb, uint8_t* out, float* scales_out) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const int64_t S = Kb / 16, NG = Kb / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < NG; ++g) {
      const uint8_t* sp = scales + r * S + g * 4;
      int mx = sp[0];
      for (int j = 1; j < 4; ++j) mx = sp[j] > mx ? sp[j] : mx;
      scales_out[g * M + r] = f_from_bits((uint32_t)(uint8_t)(mx - 6) << 23);
      for (int j = 0; j < 4; ++j) {
        const int shift = 6 - (mx - (int)sp[j]); /* <= 6 */
        const uint8_t* cb = codes + r * Kb + g * 64 + j * 16;
        uint8_t* ob = out + r * 2 * Kb + g * 128 + j * 32;
        for (int b = 0; b < 32; ++b) {
          unsigned nib = (b & 1) ? (cb[b / 2] >> 4) : (cb[b / 2] & 0xFu);
          float v = ldexpf(mag[nib & 7u], shift);
          ob[b] = orc_f32_to_e4m3((nib & 8u) ? -v : v);
        }
      }
    }
  }
}

/* ------------------------------------------------------- DQ-fp8-col (C4) */
/* MXFP4 -> transposed FP8 E4M3 (per_token_Mxfp4ToFp8_col.cu:160-290).  For
 * each 128-row block and 32-column scale block: wa = (uint8)(max E8M0 - 6);
 * per element adj = (uint8)(wa - e); value bits = (code bits - (adj << 7))
 * & 0x7FFF (the sign is dropped), clamped to +-448 (max first), E4M3.
 * codes: [M, Kb] with M % 128 == 0 and Kb % 128 == 0; out: [2*Kb, M];
 * scales_out: [M/128, 2*Kb] float, each scale repeated over its 32 columns. */
void orc_mxfp4_to_fp8_cols(const uint8_t* codes, const uint8_t* scales, int64_t M, int64_t Kb,
                           uint8_t* out, float* scales_out) {
  const int64_t S = Kb / 16, N = 2 * Kb;
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < S; ++c) {
    for (int64_t rb = 0; rb < M / 128; ++rb) {
      uint8_t mx = 0;
      for (int i = 0; i < 128; ++i) {
        uint8_t e = scales[(rb * 128 + i) * S + c];
        mx = e > mx ? e : mx;
      }
      uint8_t wa = (uint8_t)(mx - 6);
      float ys = f_from_bits((uint32_t)wa << 23);
      for (int j = 0; j < 32; ++j) scales_out[rb * N + c * 32 + j] = ys;
      for (int i = 0; i < 128; ++i) {
        int64_t r = rb * 128 + i;
        uint8_t adj = (uint8_t)(wa - scales[r * S + c]);
        for (int b = 0; b < 16; ++b) {
          uint8_t v = codes[r * Kb + c * 16 + b];
          for (int h = 0; h < 2; ++h) {
            uint16_t x = e2m1_to_bf16_bits(h ? (v >> 4) : (v & 0xFu));
            uint16_t a = (uint16_t)((uint16_t)(x - (uint16_t)((uint16_t)adj << 7)) & 0x7FFFu);
            float q = fminf(fmaxf(bf16_to_f(a), -448.0f), 448.0f);
            out[(c * 32 + 2 * b + h) * M + r] = orc_f32_to_e4m3(q);
          }
        }
      }
    }
  }
}

/* Decoded element value (code times E8M0 scale, float) as C5/C6 compute it
 * (per_token_Mxfp4RowToBf16ToFp8Col.cu:108-126). */
static inline float dq_val(const uint8_t* codes, const uint8_t* scales, int64_t N, int64_t r,
                           int64_t n) {
  uint8_t v = codes[r * (N / 2) + n / 2];
  unsigned nib = (n & 1) ? (v >> 4) : (v & 0xFu);
  return bf16_to_f(e2m1_to_bf16_bits(nib)) * e8m0_to_f(scales[r * (N / 32) + n / 32]);
}

/* ------------------------------------------------------ DQ-fp8-colT (C5) */
/* MXFP4 -> transposed FP8 with a true-amax scale per (128-row block, column)
 * (per_token_Mxfp4RowToBf16ToFp8Col.cu:76-195, race-free semantics):
 * amax = max(eps, max |v|); scale_out = amax / 448; q = E4M3(clamp(v * (448 /
 * amax), +-448)), or v * 0 when amax <= 1e-9.  codes: [M, N/2]; out: [N, M];
 * scales_out: [ceil(M/128), N]. */
void orc_mxfp4_to_fp8_colT(const uint8_t* codes, const uint8_t* scales, int64_t M, int64_t N,
                           float eps, uint8_t* out, float* scales_out) {
  const int64_t RB = (M + 127) / 128;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t rb = 0; rb < RB; ++rb) {
      int64_t r0 = rb * 128, r1 = r0 + 128 < M ? r0 + 128 : M;
      float amax = eps;
      for (int64_t r = r0; r < r1; ++r) amax = fmaxf(amax, fabsf(dq_val(codes, scales, N, r, n)));
      scales_out[rb * N + n] = amax / 448.0f;
      float qs = (amax > 1e-9f) ? (448.0f / amax) : 0.0f;
      for (int64_t r = r0; r < r1; ++r) {
        float q = dq_val(codes, scales, N, r, n) * qs;
        q = fminf(fmaxf(q, -448.0f), 448.0f);
        out[n * M + r] = orc_f32_to_e4m3(q);
      }
    }
  }
}

/* TE-style power-of-two scale (per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu:23-43). */
static inline float te_pow2_scale(float amax, float eps) {
  if (amax <= eps) return 1.0f;
  float raw = amax / 448.0f;
  uint32_t b = bits_from_f(raw);
  uint32_t ex = (b >> 23) & 0xFFu;
  if (b & 0x7FFFFFu) ex += 1u;
  float div = f_from_bits(ex << 23);
  return (float)(1.0 / (double)div);
}

/* ------------------------------------------------ DQ-fp8-colT-split (C6) */
/* As orc_mxfp4_to_fp8_colT per split i of m_splits (rows split_offsets[i] ..
 * + m_splits[i]), amax initialised to 0, power-of-two scale, 1/scale stored
 * at row scale_offsets[i] + block of scales_out [*, N]; the split's output is
 * the contiguous [N, m_i] block at split_offsets[i] * N
 * (per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu:96-222). */
void orc_mxfp4_to_fp8_colT_split(const uint8_t* codes, const uint8_t* scales, int64_t N,
                                 const int32_t* m_splits, const int32_t* split_offsets,
                                 const int32_t* scale_offsets, int64_t num_splits, float eps,
                                 uint8_t* out, float* scales_out) {
  for (int64_t i = 0; i < num_splits; ++i) {
    const int64_t mi = m_splits[i], o = split_offsets[i], so = scale_offsets[i];
    const int64_t RB = (mi + 127) / 128;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      for (int64_t b = 0; b < RB; ++b) {
        int64_t r0 = b * 128, r1 = r0 + 128 < mi ? r0 + 128 : mi;
        float amax = 0.0f;
        for (int64_t r = r0; r < r1; ++r)
          amax = fmaxf(amax, fabsf(dq_val(codes, scales, N, o + r, n)));
        float sc = te_pow2_scale(amax, eps);
        scales_out[(so + b) * N + n] = 1.0f / sc;
        for (int64_t r = r0; r < r1; ++r) {
          float q = dq_val(codes, scales, N, o + r, n) * sc;
          q = fminf(fmaxf(q, -448.0f), 448.0f);
          out[o * N + n * mi + r] = orc_f32_to_e4m3(q);
        }
      }
    }
  }
}

/* ------------------------------------------------------------ FP8-tok */
/* Per-token FP8 quantize (no reference kernel: parity unpinned).  Follows the
 * reference's FP8 convention (per_token_Mxfp4RowToBf16ToFp8Col.cu:142,161,
 * 173-177): amax = max(eps, max |x|) over the row, scale = amax / 448,
 * q = E4M3(clamp(x * (448 / amax), +-448)). */
void orc_fp8_quant_rows(const uint16_t* x, int64_t M, int64_t K, float eps, uint8_t* q,
                        float* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; ++r) {
    const uint16_t* xr = x + r * K;
    float amax = eps;
    for (int64_t k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(bf16_to_f(xr[k])));
    scale[r] = amax / 448.0f;
    float qs = 448.0f / amax;
    for (int64_t k = 0; k < K; ++k) {
      float v = fminf(fmaxf(bf16_to_f(xr[k]) * qs, -448.0f), 448.0f);
      q[r * K + k] = orc_f32_to_e4m3(v);
    }
  }
}

/* Per-token FP8 dequantize: bf16(float(q) * scale[row]). */
void orc_fp8_dequant_rows(const uint8_t* q, const float* scale, int64_t M, int64_t K,
                          uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; ++r)
    for (int64_t k = 0; k < K; ++k)
      out[r * K + k] = orc_f32_to_bf16(orc_e4m3_to_f32(q[r * K + k]) * scale[r]);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
