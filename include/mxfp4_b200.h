/*
 * mxfp4_b200.h -- C ABI of the B200 (sm_100a) MXFP4 quantize / dequantize /
 * convert library (libmxfp4_b200.so).
 *
 * Every entry point takes raw device pointers, sizes in elements (or bytes
 * where named `_bytes`), and a CUDA stream (`mxb_stream_t` is ABI-identical to
 * `cudaStream_t`; pass 0 for the legacy default stream).  Calls are
 * asynchronous on that stream, allocate nothing, keep no state between calls
 * and are safe to issue from several host threads.  The caller allocates every
 * output, as the reference's Python wrappers do (code/kernel/api/mxfp4.py:110,
 * code/kernel/api/mxfp4_dequant.py:61).  A non-zero status means nothing was
 * launched; `mxb_last_error()` returns a message for the calling thread.
 *
 * Layouts (identical to the reference's, so its Megatron / Transformer Engine
 * / DeepEP consumers read our outputs unchanged):
 *   MXFP4 codes   uint8 [rows, cols/2]; element 2i in the low nibble
 *                 (code/kernel/per_token_quant_mxfp4.cu:256).
 *   E8M0 scales   uint8 [rows, cols/32], row-major, unpadded
 *                 (code/kernel/api/mxfp4.py:135,155-161); byte e = 2^(e-127).
 *   BF16 / FP8    bf16 / float8_e4m3fn bit patterns, row-major.
 *
 * Each declaration names the reference entry point it replaces (file:line in
 * anonymous-git-2026/MXFP4-Hopper).
 */
#ifndef MXFP4_B200_H_
#define MXFP4_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mxb_stream_t;

typedef enum {
  MXB_OK = 0,
  MXB_ERR_INVALID_ARGUMENT = 1, /* shape, stride or parameter out of contract */
  MXB_ERR_MISALIGNED = 2,       /* a pointer or row pitch breaks the vector alignment */
  MXB_ERR_CUDA = 3,             /* the launch itself failed */
  MXB_ERR_UNSUPPORTED = 4       /* a mode the reference rejects too */
} mxb_status;

/* Message of the last non-OK status returned on this host thread. */
const char* mxb_last_error(void);
/* Library version string. */
const char* mxb_version(void);
/* Number of bounded pipeline waits that gave up on the current device since
 * the library was loaded (or last reset), summed over every kernel of the
 * library that waits on an mbarrier: the quantizers, the column / split FP8
 * converters and the GEMM (0 in correct operation; a non-zero value means a
 * kernel abandoned its work and its outputs are invalid).  Synchronises.
 * 0xFFFFFFFF if the counters cannot be read. */
unsigned int mxb_wait_timeouts(void);
/* Returns mxb_wait_timeouts() and zeroes the counters on the current device. */
unsigned int mxb_reset_wait_timeouts(void);

/* ------------------------------------------------------------ quantize */

/* Rowwise BF16 -> MXFP4, 1x32 blocks, E8M0 shared scale, E2M1 codes RNE.
 * Replaces omo_per_token_group_quant_fp4 (code/kernel/ops.cu:28,
 * code/kernel/per_token_quant_mxfp4.cu:387-487; kernel :121-266).
 * input bf16 [M, K] with row pitch ldx elements (ldx % 8 == 0, 16-byte
 * aligned base), K % 32 == 0; output_q uint8 [M, K/2]; output_s uint8
 * [M, K/32].  group_size must be 32 and scale_ue8m0 0 (the reference's only
 * live configuration: api/mxfp4.py:167-172).  eps is the initial block amax,
 * fp4_min/fp4_max the clamp (reference defaults 1e-10, -6, 6). */
mxb_status mxb_per_token_group_quant_fp4(const void* input, int64_t M, int64_t K, int64_t ldx,
                                         void* output_q, void* output_s, int group_size,
                                         float eps, float fp4_min, float fp4_max,
                                         int scale_ue8m0, mxb_stream_t stream);

/* Q-row and the rowwise FP8 convert of its result in one pass: output_q /
 * output_s exactly as mxb_per_token_group_quant_fp4, output_fp8 [M, K] E4M3 and
 * output_fp8_s float [K/128, M] exactly as mxb_per_token_Mxfp4ToFp8 applied to
 * them, without re-reading the codes.  K % 128 == 0.  Replaces
 * omo_per_token_group_quant_fp4_fused_ToFp8 (code/kernel/ops.cu:34-35, whose
 * source the reference does not ship; this is its two shipped halves fused). */
mxb_status mxb_per_token_group_quant_fp4_fused_ToFp8(const void* input, int64_t M, int64_t K,
                                                     int64_t ldx, void* output_q, void* output_s,
                                                     void* output_fp8, void* output_fp8_s,
                                                     int group_size, float eps, float fp4_min,
                                                     float fp4_max, int scale_ue8m0,
                                                     mxb_stream_t stream);

/* Megatron's SwiGLU with fp4_input_store in one pass (megatron-0.15.0rc7.diff:
 * 164-193, next row 4 of the path): input bf16 [M, 2H] -> output bf16 [M, H] =
 * silu(x[:, :H]) * x[:, H:] (f32, one rounding to BF16), and the rowwise MXFP4
 * of the input itself, codes [M, H] (= 2H/2) and E8M0 scales [M, H/16] (=
 * 2H/32), bit-identical to mxb_per_token_group_quant_fp4 on the input.  H % 32
 * == 0.  No reference counterpart as one kernel (the reference runs the
 * quantizer and the activation separately). */
mxb_status mxb_swiglu_quant_mxfp4(const void* input, int64_t M, int64_t H, void* output,
                                  void* codes, void* scales, float eps, float fp4_min,
                                  float fp4_max, mxb_stream_t stream);

/* Rowwise AND columnwise BF16 -> MXFP4 in one pass over the input.
 * Replaces the Transformer Engine quantize of the reference
 * (code/transformer_engine-2.8.diff:1464-1466): rowwise = Q-row of input,
 * columnwise = Q-row of input.T.contiguous(), without materialising the
 * transpose.  input bf16 [M, K], M % 32 == 0, K % 32 == 0;
 * codes_row [M, K/2], scales_row [M, K/32] (both may be NULL for a
 * columnwise-only call); codes_col [K, M/2], scales_col [K, M/32];
 * scales_row_swizzled (nullable) receives the row scales again in the
 * 128x4-tile layout of tcgen05 block-scaled MMA, padded to
 * [round_up(M,128), round_up(K/32,4)] with zero padding
 * (code/transformer_engine-2.8.diff:752-786). */
mxb_status mxb_quant_mxfp4_rowcol(const void* input, int64_t M, int64_t K, int64_t ldx,
                                  void* codes_row, void* scales_row, void* codes_col,
                                  void* scales_col, void* scales_row_swizzled, float eps,
                                  float fp4_min, float fp4_max, mxb_stream_t stream);

/* Shared-scale rule of a quantize call. */
typedef enum {
  /* The reference's rule: y_s = 2^ceil(log2(max(amax / 6, 1e-10)))
   * (code/kernel/per_token_quant_mxfp4.cu:183-192). */
  MXB_SCALE_REFERENCE = 0,
  /* The OCP MX rule: 2^(floor(log2(max(amax, 1e-10))) - 2), the E2M1 emax
   * being 2; a block whose amax is infinite gets the E8M0 NaN byte 0xFF.
   * Differs from the reference rule on ~29% of N(0,1) blocks (by +1 in the
   * reference's favour); no reference counterpart. */
  MXB_SCALE_OCP = 1
} mxb_scale_rule;

/* One entry for the rowwise and/or columnwise quantize with a selectable
 * scale rule (mxb_scale_rule; eps 1e-10 and clamp +-6, the reference API's
 * configuration).  With codes_col and scales_col NULL it is the rowwise
 * quantize of mxb_per_token_group_quant_fp4 (M any, ldx % 8 == 0), the
 * swizzled copy of the row scales written if scales_row_swizzled is given;
 * otherwise it is mxb_quant_mxfp4_rowcol (M % 32 == 0).  With
 * MXB_SCALE_REFERENCE the bytes equal those entry points'. */
mxb_status mxb_quantize_mxfp4(const void* input, int64_t M, int64_t K, int64_t ldx,
                              void* codes_row, void* scales_row, void* codes_col,
                              void* scales_col, void* scales_row_swizzled, int scale_rule,
                              mxb_stream_t stream);

/* mxb_quant_mxfp4_rowcol on HOST buffers (the end-to-end call for data in host
 * memory; pinned memory for full speed): x_host bf16 [M, K] -> codes_row_host
 * [M, K/2], scales_row_host [M, K/32], codes_col_host [K, M/2], scales_col_host
 * [K, M/32], the same bytes as the device call.  Row chunks of chunk_rows
 * (a multiple of 128; 0 picks 1024) are pipelined: chunk i's host->device copy,
 * chunk i-1's quantize on `stream` and chunk i-2's device->host copies overlap,
 * on two internal copy streams per device.  workspace: DEVICE memory, 256-byte
 * aligned, of mxb_quant_mxfp4_rowcol_host_workspace(M, K, chunk_rows) bytes,
 * for two chunks in flight; nothing is allocated.  Asynchronous: the outputs are
 * complete when `stream` reaches the point after this call.  No reference
 * counterpart (the reference works on device tensors only). */
mxb_status mxb_quant_mxfp4_rowcol_host(const void* x_host, int64_t M, int64_t K,
                                       void* codes_row_host, void* scales_row_host,
                                       void* codes_col_host, void* scales_col_host,
                                       void* workspace, int64_t workspace_bytes,
                                       int64_t chunk_rows, float eps, float fp4_min,
                                       float fp4_max, mxb_stream_t stream);
int64_t mxb_quant_mxfp4_rowcol_host_workspace(int64_t M, int64_t K, int64_t chunk_rows);

/* Rewrites row-major E8M0 scales [M, S] into the 128x4-tile swizzled layout
 * [round_up(M,128), round_up(S,4)] (zero padding).  Shape rule from
 * MXFP4Quantizer.get_scale_shape (code/transformer_engine-2.8.diff:752-786). */
mxb_status mxb_swizzle_scales(const void* scales, int64_t M, int64_t S, void* out,
                              mxb_stream_t stream);

/* ------------------------------------------------------------ dequantize */

/* MXFP4 -> BF16.  Replaces omo_per_token_Mxfp4ToBf16_dequant
 * (code/kernel/ops.cu:30, per_token_Mxfp4ToBf16_dequant.cu:164-240; kernel
 * :70-160).  input uint8 [M, Kb] (Kb % 16 == 0), input_s uint8 [M, Kb/16],
 * output bf16 [M, 2*Kb].  The reference's output_s is never written
 * (per_token_Mxfp4ToBf16_dequant.cu:122) and is not taken here. */
mxb_status mxb_per_token_Mxfp4ToBf16_dequant(const void* input, const void* input_s, int64_t M,
                                             int64_t Kb, void* output, mxb_stream_t stream);

/* MXFP4 -> FP8 E4M3 rowwise, 1x128 groups with power-of-two FP32 scales
 * derived from the group's largest E8M0 exponent.  Replaces
 * omo_per_token_Mxfp4ToFp8 (code/kernel/api/mxfp4_dequant.py:1,167;
 * per_token_Mxfp4ToFp8.cu:239-310; kernel :92-235).  input uint8 [M, Kb]
 * (Kb % 64 == 0), input_s uint8 [M, Kb/16], output_q fp8 [M, 2*Kb],
 * output_s float [Kb/64, M] (M-contiguous, Transformer Engine GEMM_READY). */
mxb_status mxb_per_token_Mxfp4ToFp8(const void* input, const void* input_s, int64_t M, int64_t Kb,
                                    void* output_q, void* output_s, mxb_stream_t stream);

/* mxb_per_token_Mxfp4ToFp8 without the reference's 16-bit re-basing wrap:
 * every element is its true value e2m1 * 2^(e - 127) divided by the group
 * scale 2^(max e - 6 - 127), rounded to E4M3 (RNE, saturating), so zero codes
 * stay zero where the reference writes +-448 and far-below-maximum blocks
 * underflow to zero.  Same shapes and group scales.  No reference
 * counterpart (an option of the rowwise converter, off by default). */
mxb_status mxb_per_token_Mxfp4ToFp8_strict(const void* input, const void* input_s, int64_t M,
                                           int64_t Kb, void* output_q, void* output_s,
                                           mxb_stream_t stream);

/* MXFP4 -> FP8 E4M3 with ONE FP32 scale per row: each row is dequantized as
 * mxb_per_token_Mxfp4ToBf16_dequant does, then quantized per token as
 * mxb_per_token_quant_fp8 does (amax = max(eps, max |x|), scale = amax/448,
 * q = E4M3(clamp(x * 448/amax, +-448))), in one pass.  input uint8 [M, Kb]
 * (Kb % 16 == 0), input_s uint8 [M, Kb/16], output_q fp8 [M, 2*Kb],
 * output_s float [M].  No reference kernel: the per-row variant of the
 * rowwise converter (the reference's groups are 1x128). */
mxb_status mxb_per_token_Mxfp4ToFp8_rowscale(const void* input, const void* input_s, int64_t M,
                                             int64_t Kb, void* output_q, void* output_s, float eps,
                                             mxb_stream_t stream);

/* Same operation under the name the reference binds at code/kernel/ops.cu:32
 * (omo_per_token_Mxfp4ToBf16ToFp8, whose source the reference does not ship). */
mxb_status mxb_per_token_Mxfp4ToBf16ToFp8(const void* input, const void* input_s, int64_t M,
                                          int64_t Kb, void* output_q, void* output_s,
                                          mxb_stream_t stream);

/* MXFP4 -> transposed FP8 E4M3 with a scale per (128-row block, 32-column
 * block) from the largest E8M0 exponent.  Replaces omo_per_token_Mxfp4ToFp8_col
 * (code/kernel/ops.cu:40, per_token_Mxfp4ToFp8_col.cu:305-384; kernel
 * :110-301), quirks included (the outputs carry no sign).  input uint8
 * [M, Kb], M % 128 == 0, Kb % 128 == 0; output_q fp8 [2*Kb, M]; output_s
 * float [M/128, 2*Kb]. */
mxb_status mxb_per_token_Mxfp4ToFp8_col(const void* input, const void* input_s, int64_t M,
                                        int64_t Kb, void* output_q, void* output_s,
                                        mxb_stream_t stream);

/* MXFP4 (rowwise) -> FP8 E4M3 columnwise with a true-amax scale per
 * (128-row block, column): the wgrad operand.  Replaces
 * omo_per_token_Mxfp4RowToBf16ToFp8Col (code/kernel/ops.cu:36,
 * per_token_Mxfp4RowToBf16ToFp8Col.cu:204-247; kernel :42-197), with the
 * kernel's missing barrier restored.  input uint8 [M, N/2], N % 32 == 0;
 * input_s uint8 [M, N/32]; output_q fp8 [N, M]; output_s float
 * [ceil(M/128), N] holding amax/448. */
mxb_status mxb_per_token_Mxfp4RowToBf16ToFp8Col(const void* input, const void* input_s,
                                                int64_t M, int64_t N, void* output_q,
                                                void* output_s, float eps, mxb_stream_t stream);

/* As above for a grouped GEMM: rows split into num_splits segments of
 * m_splits[i] rows, each quantized with power-of-two scales into its own
 * contiguous [N, m_i] block at split_offsets[i] * N of output_q; scales
 * (1/scale) at rows scale_offsets[i] + b of output_s [sum ceil(m_i/128), N].
 * m_splits / split_offsets / scale_offsets are int32 DEVICE arrays; max_split_len
 * bounds m_splits.  Replaces omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit
 * (code/kernel/ops.cu:38, per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu:232-282;
 * kernel :51-224). */
mxb_status mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit(
    const void* input, const void* input_s, int64_t total_M, int64_t N, void* output_q,
    void* output_s, const int32_t* m_splits, const int32_t* split_offsets,
    const int32_t* scale_offsets, int64_t num_splits, int64_t max_split_len, float eps,
    mxb_stream_t stream);

/* No reference counterpart.  The same conversion with only m_splits (int32
 * DEVICE [num_splits], e.g. straight from a router) and no caller-allocated
 * offsets: split_offsets and scale_offsets are computed on the device, by a
 * one-block exclusive scan on `stream`, into a file-scope device array of
 * 2 x MXB_MSPLIT_MAX_SEGMENTS int32 (32 KiB per device); the call allocates
 * nothing.  num_splits above MXB_MSPLIT_MAX_SEGMENTS is rejected with
 * MXB_ERR_INVALID_ARGUMENT.  max_split_len must be at least every m_splits[i]
 * (total_M always is); segments must sum to total_M.  Nothing in the array has
 * to start at zero: the scan writes every word the conversion reads.  Calls
 * that overlap on the GPU (on other streams, or from other host threads
 * without ordering) share that array and race; order them, e.g. on one
 * stream. */
#define MXB_MSPLIT_MAX_SEGMENTS 4096
mxb_status mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit_noalloc(
    const void* input, const void* input_s, int64_t total_M, int64_t N, void* output_q,
    void* output_s, const int32_t* m_splits, int64_t num_splits, int64_t max_split_len, float eps,
    mxb_stream_t stream);

/* ------------------------------------------------------------ MXFP4 GEMM */

/* No reference counterpart (the consumer of the quantized operands: next row 3
 * of the path).  C bf16 [M, N] = A . B^T on the tcgen05 tensor cores
 * (kind::mxf4 block_scale, f32 accumulation): A codes [M, K/2] and B codes
 * [N, K/2] as mxb_per_token_group_quant_fp4 writes them, their E8M0 scales in
 * the 128x4-tile swizzled layout of mxb_swizzle_scales ([M, K/32] -> [M, K/32]
 * for M % 128 == 0 and K % 128 == 0).  M % 128, N % 128, K % 256 == 0. */
mxb_status mxb_gemm_mxfp4(const void* a_codes, const void* a_scales_swizzled, const void* b_codes,
                          const void* b_scales_swizzled, int64_t M, int64_t N, int64_t K, void* c,
                          mxb_stream_t stream);
unsigned int mxb_gemm_wait_timeouts(void);

/* ------------------------------------------------------------ per-token FP8 */

/* BF16 -> FP8 E4M3 with one FP32 scale per row: amax = max(eps, max|x|),
 * scale = amax/448, q = E4M3(clamp(x * 448/amax, +-448)).  The reference ships
 * no kernel for this (code/kernel/setup.py:62 names per_token_quant_fp8.cu in
 * a comment only); the arithmetic follows its FP8 convention
 * (per_token_Mxfp4RowToBf16ToFp8Col.cu:142,161,173-177).  input bf16 [M, K],
 * K % 8 == 0; output_q fp8 [M, K]; output_s float [M]. */
mxb_status mxb_per_token_quant_fp8(const void* input, int64_t M, int64_t K, void* output_q,
                                   void* output_s, float eps, mxb_stream_t stream);

/* FP8 E4M3 with per-row FP32 scale -> BF16: out = bf16(float(q) * scale[row]). */
mxb_status mxb_per_token_dequant_fp8(const void* input_q, const void* input_s, int64_t M,
                                     int64_t K, void* output, mxb_stream_t stream);

/* ------------------------------------------------------------ MoE expert parallel */

/* Dispatch pack: quantizes each token row of x (bf16 [T, H], H % 128 == 0) to
 * MXFP4 once (bit-exact Q-row, eps <= 6e-10) and writes its wire row
 * codes[H/2] || scales[H/32] (megatron-0.15.0rc7.diff:32-63, the packing
 * `fp4_quantize` hands to DeepEP at :290-297) to wire + slots[t*G + g] * (17H/32)
 * for every g with slots[t*G + g] >= 0.  slots: int32 DEVICE array [T, G]. */
mxb_status mxb_ep_pack(const void* x, int64_t T, int64_t H, const int32_t* slots, int G, void* wire,
                       float eps, mxb_stream_t stream);

/* Receive side: wire rows [R, 17H/32] -> bf16 [R, H], bit-exact with
 * `get_fp4_tensor(recv_x).dequantize()` (megatron-0.15.0rc7.diff:101-124,303-309).
 * If weight (float DEVICE [R]) is given, each row is multiplied by weight[row]
 * after the dequantize and rounded to bf16 again. */
mxb_status mxb_ep_unpack(const void* wire, int64_t R, int64_t H, const float* weight, void* out,
                         mxb_stream_t stream);

/* Combine: out[t] = bf16(sum over g = 0..G-1 with slots[t*G + g] >= 0 of
 * float(recv[slots[t*G + g]])), summed in rank order; recv bf16 [S, H],
 * out bf16 [T, H].  The BF16 combine of DeepEP (deep_ep-1.2.1.diff:132-139). */
mxb_status mxb_ep_combine(const void* recv, int64_t T, int64_t H, const int32_t* slots, int G,
                          void* out, mxb_stream_t stream);

/* MoE permute of MXFP4 rows (the MXFP4 branch of Transformer Engine's moe_permute,
 * transformer_engine-2.8.diff:253-261,338-356), fused with the EP receive split:
 * source row i (codes at codes + i*codes_pitch, H/2 bytes; E8M0 scales at
 * scales + i*scales_pitch, H/32 bytes; wire rows: scales = codes + H/2 and both
 * pitches 17H/32) is copied to output rows dst[i*topk + k] of out_codes
 * [n_out, H/2] and out_scales [n_out, H/32] for k < topk; destinations outside
 * [0, n_out) (e.g. -1) are skipped.  dst: int32 DEVICE [rows, topk], topk <= 32.
 * The caller derives dst from its routing map (TE's row_id_map, DeepEP's
 * handle); each row is read once whatever topk is. */
mxb_status mxb_moe_permute_mxfp4(const void* codes, int64_t codes_pitch, const void* scales,
                                 int64_t scales_pitch, int64_t rows, int64_t H, const int32_t* dst,
                                 int topk, void* out_codes, void* out_scales, int64_t n_out,
                                 mxb_stream_t stream);

/* Transformer Engine's row_id_map for moe_permute with a mask routing map
 * (the MXFP4 branch calls it at transformer_engine-2.8.diff:253-261,338-356;
 * the map itself is upstream TE code the reference does not ship, restated
 * here): routing_map bool (one byte) DEVICE [T, E]; the permuted output holds
 * expert 0's tokens in token order, then expert 1's, ...; row_id_map int32
 * DEVICE [T, 2E + 1]: per token its n destination rows (ascending expert
 * order) in columns 0..n-1, those experts in columns E..E+n-1, n in column
 * 2E, -1 elsewhere.  workspace: int32 DEVICE [E] (per-expert offsets). */
mxb_status mxb_moe_make_row_id_map(const void* routing_map, int64_t T, int32_t E,
                                   int32_t* row_id_map, int32_t* workspace, mxb_stream_t stream);

/* mxb_moe_permute_mxfp4 driven by that row_id_map: token row t (codes and E8M0
 * scales, any pitches as there) goes to rows row_id_map[t, 0..n-1] of
 * out_codes [num_out_tokens, H/2] and out_scales [num_out_tokens, H/32]. */
mxb_status mxb_moe_permute_mxfp4_row_id_map(const void* codes, int64_t codes_pitch,
                                            const void* scales, int64_t scales_pitch, int64_t T,
                                            int64_t H, const int32_t* row_id_map, int32_t E,
                                            void* out_codes, void* out_scales,
                                            int64_t num_out_tokens, mxb_stream_t stream);

/* ---- dispatch / combine over an NCCL communicator ----
 * The DeepEP-style exchange of the reference's MXFP4 payload
 * (deep_ep-1.2.1.diff:455-549, megatron-0.15.0rc7.diff:290-311) for a caller
 * holding an ncclComm_t (one process per GPU).  NCCL is opened at run time
 * (libnccl.so.2); these entry points return MXB_ERR_UNSUPPORTED without it.
 * comm is an ncclComm_t passed as void*. */
#define MXB_EP_MAX_WORLD 64
/* Host record a dispatch fills and its combine reads. */
typedef struct {
  int64_t send_counts[MXB_EP_MAX_WORLD]; /* rows this rank sent to each rank */
  int64_t recv_counts[MXB_EP_MAX_WORLD]; /* rows it received from each rank */
  int64_t n_send, n_recv, tokens;
  int32_t world, rank, hidden, topk;
} mxb_ep_handle;
/* A fresh 128-byte NCCL unique id (rank 0 makes it and shares it). */
mxb_status mxb_nccl_unique_id(void* id128);
/* ncclCommInitRank: *comm receives the communicator. */
mxb_status mxb_nccl_comm_init(void** comm, int32_t world, int32_t rank, const void* id128);
mxb_status mxb_nccl_comm_destroy(void* comm);
/* DEVICE workspace bytes a dispatch / combine pair needs (256-byte aligned; it
 * carries the send slots from the dispatch to its combine). */
int64_t mxb_ep_nccl_workspace_bytes(int64_t T, int32_t H, int32_t topk, int32_t world);
/* Tokens x bf16 [T, H] (H % 128 == 0) routed by topk_idx int64 / topk_w float
 * [T, topk] (global expert ids, experts_per_rank consecutive experts per rank):
 * each token is quantized once to its wire row codes[H/2] || E8M0[H/32] and
 * sent once to every rank hosting one of its experts.  On return the receive
 * buffers hold handle->n_recv rows grouped by source rank (token order within):
 * recv_wire uint8 [recv_cap, 17H/32], recv_meta [recv_cap] records of topk
 * int32 expert ids local to this rank (-1 for experts elsewhere) followed by
 * topk float routing weights (0 elsewhere).  The call synchronises `stream`
 * once, after the per-peer counts arrive (MXB_ERR_INVALID_ARGUMENT if more rows
 * arrive than recv_cap); the row exchange itself is asynchronous. */
mxb_status mxb_ep_nccl_dispatch(void* comm, int32_t world, int32_t rank, const void* x, int64_t T,
                                int32_t H, const int64_t* topk_idx, const float* topk_w,
                                int32_t topk, int32_t experts_per_rank, void* workspace,
                                int64_t workspace_bytes, void* recv_wire, void* recv_meta,
                                int64_t recv_cap, mxb_ep_handle* handle, mxb_stream_t stream);
/* y bf16 [handle->n_recv, H]: the expert output of each received row, in
 * receive order.  Sends each row back to its source rank and writes
 * out[t] = bf16(sum over ranks, in rank order, of the rows returned for token t)
 * (DeepEP's BF16 combine, deep_ep-1.2.1.diff:132-139); out bf16 [T, H].
 * Asynchronous on `stream`; `workspace` is the dispatch's. */
mxb_status mxb_ep_nccl_combine(void* comm, const mxb_ep_handle* handle, const void* y,
                               void* workspace, int64_t workspace_bytes, void* out,
                               mxb_stream_t stream);

/* ---- fused dispatch / combine over NVLink peer memory ----
 * One buffer per rank with the layout below, mapped into every peer with CUDA
 * IPC (mxb_ipc_export / mxb_ipc_import); `bases` is a DEVICE array of the world
 * base addresses (this rank's own buffer at index rank).  A step is
 *   mxb_ep_p2p_counts(epoch e+1)  -> every rank learns every send count
 *   mxb_ep_p2p_dispatch            -> tokens quantized once and stored into the
 *                                     destinations' receive rows over NVLink
 *   mxb_ep_p2p_barrier(e+2)
 *   mxb_ep_p2p_return              -> expert rows stored back into the sources
 *   mxb_ep_p2p_barrier(e+3)
 *   mxb_ep_combine on this rank's back rows.
 * The same semantics as DeepEP's intranode dispatch/combine with the MXFP4
 * payload of the reference (deep_ep-1.2.1.diff:455-549, megatron-0.15.0rc7.diff:
 * 290-311), without host synchronisation.  Parity alternates per step.  All
 * cross-GPU waits are bounded; mxb_ep_wait_timeouts() counts waits that gave up.
 * Layout limits: world <= 32, topk <= 32, world * topk <= 256, hidden a multiple
 * of 512 and at most 65536. */
typedef struct {
  int64_t sig_off, cnt_off, wire_off, meta_off, back_off; /* byte offsets in the buffer */
  int64_t tcap;                                           /* max tokens per rank */
  int32_t world, rank, topk, hidden, experts_per_rank;
} mxb_ep_layout;

mxb_status mxb_ep_layout_init(int32_t world, int32_t rank, int64_t tcap, int32_t hidden,
                              int32_t topk, int32_t experts_per_rank, mxb_ep_layout* layout,
                              int64_t* total_bytes);
/* CUDA IPC of a device allocation: 64-byte handle + offset of ptr in it. */
mxb_status mxb_ipc_export(const void* ptr, void* handle64, int64_t* offset);
mxb_status mxb_ipc_import(const void* handle64, int64_t offset, void** ptr);
mxb_status mxb_ipc_close(void* ptr, int64_t offset);
/* send_counts: int32 DEVICE [world]. */
mxb_status mxb_ep_p2p_counts(const uint64_t* bases, const mxb_ep_layout* layout,
                             const int32_t* send_counts, int parity, uint32_t epoch,
                             mxb_stream_t stream);
/* x bf16 [T, hidden]; within int32 DEVICE [T, world]: index of token t among the
 * tokens this rank sends to rank g, or -1; topk_idx int64 / topk_w float DEVICE
 * [T, topk] global expert ids and routing weights. */
mxb_status mxb_ep_p2p_dispatch(const void* x, int64_t T, const int32_t* within,
                               const int64_t* topk_idx, const float* topk_w,
                               const uint64_t* bases, const mxb_ep_layout* layout, int parity,
                               mxb_stream_t stream);
mxb_status mxb_ep_p2p_barrier(const uint64_t* bases, const mxb_ep_layout* layout, uint32_t epoch,
                              mxb_stream_t stream);
/* y: bf16 DEVICE [world*tcap, hidden] expert outputs per received row, or NULL
 * for the routing-weighted identity expert fused with the dequantize. */
mxb_status mxb_ep_p2p_return(const void* y, const uint64_t* bases, const mxb_ep_layout* layout,
                             int parity, mxb_stream_t stream);
/* Routing on the device: within[t*world + g] = index of token t among the
 * tokens routed to rank g (experts contiguous per rank, topk_idx int64
 * [T, topk] global ids), -1 if none; send_counts[g] = number of such tokens. */
mxb_status mxb_ep_route(const int64_t* topk_idx, int64_t T, int32_t topk, int32_t experts_per_rank,
                        int32_t world, int32_t* within, int32_t* send_counts, mxb_stream_t stream);
/* Local combine of the returned rows: out[t] = bf16(sum over g of
 * float(back[sum_{g'<g} send_counts[g'] + within[t, g]])). */
mxb_status mxb_ep_p2p_combine(const void* back, int64_t T, int64_t H, const int32_t* within,
                              const int32_t* send_counts, int32_t world, void* out,
                              mxb_stream_t stream);
/* Cross-GPU waits (barriers, count exchange) that gave up on the current
 * device since load or the last reset; a non-zero value means the step's
 * outputs are invalid and a peer is late or gone.  Synchronises. */
unsigned int mxb_ep_wait_timeouts(void);
/* Returns mxb_ep_wait_timeouts() and zeroes the counter on the current device. */
unsigned int mxb_ep_reset_wait_timeouts(void);
/* Polls (each ~64 ns of sleep plus one system-scope load) a cross-GPU wait
 * makes on the current device before it gives up; 0 restores the default
 * 2^22 (~0.3 s).  Synchronous; set it between steps, not while a step runs. */
mxb_status mxb_ep_set_wait_polls(uint32_t polls);

#ifdef __cplusplus
}
#endif
#endif /* MXFP4_B200_H_ */
