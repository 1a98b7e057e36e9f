// `omo` torch extension for the B200 library: the reference's operator names,
// argument names and checks (code/kernel/ops.cu:27-43), implemented as thin
// C++ host code over the C ABI of libmxfp4_b200.so (include/mxfp4_b200.h).
//
// Every op runs asynchronously on torch's current CUDA stream and writes into
// caller-allocated outputs, as the reference's ops do.  Argument errors raise
// RuntimeError (TORCH_CHECK), like the reference's CHECK_INPUT / CHECK_EQ.
// There is no CPU path: a CPU tensor is an error.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <nvtx3/nvToolsExt.h>
#include <torch/extension.h>

#include "mxfp4_b200.h"

namespace {

// NVTX range over one operator call (visible in Nsight Systems timelines next
// to the kernels it launches; costs nothing when no tool is attached).
struct OmoRange {
  explicit OmoRange(const char* name) { nvtxRangePushA(name); }
  ~OmoRange() { nvtxRangePop(); }
};

#define OMO_CHECK_INPUT(x)                                               \
  TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor");               \
  TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")

mxb_stream_t cur_stream() {
  return reinterpret_cast<mxb_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

void check_status(mxb_status s, const char* op) {
  TORCH_CHECK(s == MXB_OK, op, ": ", mxb_last_error());
}

void check_dtype(const at::Tensor& t, at::ScalarType st, const char* name) {
  TORCH_CHECK(t.scalar_type() == st, name, " must have dtype ", c10::toString(st), ", got ",
              c10::toString(t.scalar_type()));
}

// ---- per_token_quant_mxfp4.cu:387-487
void omo_per_token_group_quant_fp4(at::Tensor input, at::Tensor output_q, at::Tensor output_s,
                                   int64_t group_size, double eps, double fp4_min, double fp4_max,
                                   bool scale_ue8m0) {
  OmoRange nvtx_range("omo_per_token_group_quant_fp4");
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  TORCH_CHECK(input.numel() % group_size == 0, "CHECK_EQ(input.numel() % group_size, 0) failed");
  TORCH_CHECK(output_s.dim() == 2, "CHECK_EQ(output_s.dim(), 2) failed");
  check_dtype(input, at::kBFloat16, "input");
  check_dtype(output_q, at::kByte, "output_q");
  check_dtype(output_s, at::kByte, "output_s");
  TORCH_CHECK(output_s.is_contiguous() && output_s.is_cuda(),
              "output_s must be a contiguous CUDA tensor (row-major scales)");
  if (input.numel() == 0) return;
  const int64_t K = input.size(-1), M = input.numel() / K;
  TORCH_CHECK(output_q.numel() == M * K / 2, "output_q must hold numel/2 bytes");
  // The reference writes group g's scale at output_s.data_ptr() + g whatever the
  // tensor's shape (per_token_quant_mxfp4.cu:161), and its fp4 wrapper sizes
  // output_s from the code shape, [M, K/2] (api/mxfp4.py:106-111): any
  // contiguous buffer of at least numel/32 bytes is accepted and the scales
  // fill its first numel/32 bytes.
  TORCH_CHECK(output_s.numel() >= M * K / 32, "output_s must hold numel/32 scales");
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_group_quant_fp4(input.data_ptr(), M, K, K, output_q.data_ptr(),
                                             output_s.data_ptr(), (int)group_size, (float)eps,
                                             (float)fp4_min, (float)fp4_max, scale_ue8m0 ? 1 : 0,
                                             cur_stream()),
               "omo_per_token_group_quant_fp4");
}

// ---- per_token_Mxfp4ToBf16_dequant.cu:164-240.  The reference indexes codes
// and scales as flat arrays (element i uses scale i/32), so the op is launched
// over the flattened tensors.  output_s is accepted and left untouched, as on
// the reference (per_token_Mxfp4ToBf16_dequant.cu:122).
void omo_per_token_Mxfp4ToBf16_dequant(at::Tensor input, at::Tensor input_s, at::Tensor output_q,
                                       at::Tensor output_s, int64_t group_size, double eps,
                                       double fp4_min, double fp4_max, bool scale_ue8m0) {
  OmoRange nvtx_range("omo_per_token_Mxfp4ToBf16_dequant");
  (void)group_size; (void)eps; (void)fp4_min; (void)fp4_max;
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  TORCH_CHECK(input.numel() % 128 == 0, "CHECK_EQ(input.numel() % group_size, 0) failed (group_size is 128)");
  TORCH_CHECK(output_s.dim() == 2, "CHECK_EQ(output_s.dim(), 2) failed");
  TORCH_CHECK(!scale_ue8m0, "scale_ue8m0=True is not supported (reference host assert)");
  check_dtype(input, at::kByte, "input");
  check_dtype(input_s, at::kByte, "input_s");
  check_dtype(output_q, at::kBFloat16, "output_q");
  OMO_CHECK_INPUT(input_s);
  const int64_t n = input.numel();
  if (n == 0) return;
  TORCH_CHECK(input_s.numel() >= n / 16, "input_s must hold one scale per 16 code bytes");
  TORCH_CHECK(output_q.numel() >= 2 * n, "output_q must hold 2 elements per code byte");
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_Mxfp4ToBf16_dequant(input.data_ptr(), input_s.data_ptr(), 1, n,
                                                 output_q.data_ptr(), cur_stream()),
               "omo_per_token_Mxfp4ToBf16_dequant");
}

void mxfp4_to_fp8_row_common(at::Tensor& input, at::Tensor& input_s, at::Tensor& output_q,
                             at::Tensor& output_s, bool scale_ue8m0, const char* op) {
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  OMO_CHECK_INPUT(input_s);
  TORCH_CHECK(input.numel() % 128 == 0, "CHECK_EQ(input.numel() % group_size, 0) failed (group_size is 128)");
  TORCH_CHECK(output_s.dim() == 2, "CHECK_EQ(output_s.dim(), 2) failed");
  TORCH_CHECK(!scale_ue8m0, "scale_ue8m0=True is not supported (reference host assert)");
  TORCH_CHECK(input.dim() == 2, op, ": input must be 2-D [M, K/2]");
  check_dtype(input, at::kByte, "input");
  check_dtype(input_s, at::kByte, "input_s");
  check_dtype(output_q, at::kFloat8_e4m3fn, "output_q");
  check_dtype(output_s, at::kFloat, "output_s");
  TORCH_CHECK(output_s.is_contiguous() && output_s.is_cuda(), "output_s must be a contiguous CUDA tensor");
  const int64_t M = input.size(0), Kb = input.size(1);
  if (M == 0 || Kb == 0) return;
  TORCH_CHECK(Kb % 64 == 0, op, ": the code row must be a multiple of 64 bytes (1x128 groups); "
              "the Python wrapper pads it");
  TORCH_CHECK(input_s.numel() >= M * Kb / 16, op, ": input_s too small");
  TORCH_CHECK(output_q.numel() == 2 * M * Kb, op, ": output_q must be [M, 2*K]");
  TORCH_CHECK(output_s.numel() == M * Kb / 64, op, ": output_s must be [K/64, M]");
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_Mxfp4ToFp8(input.data_ptr(), input_s.data_ptr(), M, Kb,
                                        output_q.data_ptr(), output_s.data_ptr(), cur_stream()),
               op);
}

// ---- per_token_Mxfp4ToFp8.cu:239-310
void omo_per_token_Mxfp4ToFp8(at::Tensor input, at::Tensor input_s, at::Tensor output_q,
                              at::Tensor output_s, int64_t group_size, double eps, double fp4_min,
                              double fp4_max, bool scale_ue8m0) {
  OmoRange nvtx_range("omo_per_token_Mxfp4ToFp8");
  (void)group_size; (void)eps; (void)fp4_min; (void)fp4_max;
  mxfp4_to_fp8_row_common(input, input_s, output_q, output_s, scale_ue8m0,
                          "omo_per_token_Mxfp4ToFp8");
}

// ---- ops.cu:32 binds this name; its source is not in the reference.  Same
// operation as omo_per_token_Mxfp4ToFp8.
void omo_per_token_Mxfp4ToBf16ToFp8(at::Tensor input, at::Tensor input_s, at::Tensor output_q,
                                    at::Tensor output_s, int64_t group_size, double eps,
                                    double fp4_min, double fp4_max, bool scale_ue8m0) {
  OmoRange nvtx_range("omo_per_token_Mxfp4ToBf16ToFp8");
  (void)group_size; (void)eps; (void)fp4_min; (void)fp4_max;
  mxfp4_to_fp8_row_common(input, input_s, output_q, output_s, scale_ue8m0,
                          "omo_per_token_Mxfp4ToBf16ToFp8");
}

// ---- ops.cu:34 binds this name; its source is not in the reference.  Q-row
// into (output_q, output_s), then the rowwise FP8 convert of that result into
// (output_bf16_q [M, K] fp8, output_bf16_s [K/128, M] float).
void omo_per_token_group_quant_fp4_fused_ToFp8(at::Tensor input, at::Tensor output_q,
                                               at::Tensor output_s, at::Tensor output_bf16_q,
                                               at::Tensor output_bf16_s, int64_t group_size,
                                               double eps, double fp4_min, double fp4_max,
                                               bool scale_ue8m0) {
  OmoRange nvtx_range("omo_per_token_group_quant_fp4_fused_ToFp8");
  // the checks of both halves (omo_per_token_group_quant_fp4 and omo_per_token_Mxfp4ToFp8)
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  OMO_CHECK_INPUT(output_bf16_q);
  TORCH_CHECK(input.numel() % group_size == 0, "CHECK_EQ(input.numel() % group_size, 0) failed");
  TORCH_CHECK(output_s.dim() == 2 && output_bf16_s.dim() == 2, "CHECK_EQ(output_s.dim(), 2) failed");
  check_dtype(input, at::kBFloat16, "input");
  check_dtype(output_q, at::kByte, "output_q");
  check_dtype(output_s, at::kByte, "output_s");
  check_dtype(output_bf16_q, at::kFloat8_e4m3fn, "output_bf16_q");
  check_dtype(output_bf16_s, at::kFloat, "output_bf16_s");
  TORCH_CHECK(output_s.is_contiguous() && output_s.is_cuda() && output_bf16_s.is_contiguous() &&
                  output_bf16_s.is_cuda(),
              "scale outputs must be contiguous CUDA tensors");
  if (input.numel() == 0) return;
  const int64_t K = input.size(-1), M = input.numel() / K;
  TORCH_CHECK(K % 128 == 0, "omo_per_token_group_quant_fp4_fused_ToFp8: K must be a multiple of "
              "128 (1x128 FP8 groups)");
  TORCH_CHECK(output_q.numel() == M * K / 2, "output_q must hold numel/2 bytes");
  TORCH_CHECK(output_s.numel() >= M * K / 32, "output_s must hold numel/32 scales");
  TORCH_CHECK(output_bf16_q.numel() == M * K, "output_bf16_q must be [M, K]");
  TORCH_CHECK(output_bf16_s.numel() == M * K / 128, "output_bf16_s must be [K/128, M]");
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_group_quant_fp4_fused_ToFp8(
                   input.data_ptr(), M, K, K, output_q.data_ptr(), output_s.data_ptr(),
                   output_bf16_q.data_ptr(), output_bf16_s.data_ptr(), (int)group_size, (float)eps,
                   (float)fp4_min, (float)fp4_max, scale_ue8m0 ? 1 : 0, cur_stream()),
               "omo_per_token_group_quant_fp4_fused_ToFp8");
}

// ---- per_token_Mxfp4ToFp8_col.cu:305-384
void omo_per_token_Mxfp4ToFp8_col(at::Tensor input, at::Tensor input_s, at::Tensor output_q,
                                  at::Tensor output_s, int64_t group_size, double eps,
                                  double fp4_min, double fp4_max, bool scale_ue8m0) {
  OmoRange nvtx_range("omo_per_token_Mxfp4ToFp8_col");
  (void)group_size; (void)eps; (void)fp4_min; (void)fp4_max;
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  OMO_CHECK_INPUT(input_s);
  TORCH_CHECK(input.numel() % 128 == 0, "CHECK_EQ(input.numel() % group_size, 0) failed (group_size is 128)");
  TORCH_CHECK(output_s.dim() == 2, "CHECK_EQ(output_s.dim(), 2) failed");
  TORCH_CHECK(!scale_ue8m0, "scale_ue8m0=True is not supported (reference host assert)");
  TORCH_CHECK(input.dim() == 2, "input must be 2-D [M, K/2]");
  check_dtype(input, at::kByte, "input");
  check_dtype(input_s, at::kByte, "input_s");
  check_dtype(output_q, at::kFloat8_e4m3fn, "output_q");
  check_dtype(output_s, at::kFloat, "output_s");
  const int64_t M = input.size(0), Kb = input.size(1);
  if (M == 0 || Kb == 0) return;
  TORCH_CHECK(M % 128 == 0 && Kb % 128 == 0,
              "omo_per_token_Mxfp4ToFp8_col: M and the code row length must be multiples of 128 "
              "(the reference kernel tiles 128x128 bytes without bounds checks)");
  TORCH_CHECK(input_s.numel() == M * Kb / 16, "input_s must be [M, K/16]");
  TORCH_CHECK(output_q.numel() == 2 * M * Kb, "output_q must be [2*K, M]");
  TORCH_CHECK(output_s.numel() == (M / 128) * 2 * Kb, "output_s must be [M/128, 2*K]");
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_Mxfp4ToFp8_col(input.data_ptr(), input_s.data_ptr(), M, Kb,
                                            output_q.data_ptr(), output_s.data_ptr(), cur_stream()),
               "omo_per_token_Mxfp4ToFp8_col");
}

// ---- per_token_Mxfp4RowToBf16ToFp8Col.cu:204-247 (same shape checks)
void omo_per_token_Mxfp4RowToBf16ToFp8Col(at::Tensor input, at::Tensor input_s,
                                          at::Tensor output_q, at::Tensor output_s, double eps) {
  OmoRange nvtx_range("omo_per_token_Mxfp4RowToBf16ToFp8Col");
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  TORCH_CHECK(input.dim() == 2, "CHECK_EQ(input.dim(), 2) failed");
  TORCH_CHECK(output_q.dim() == 2, "CHECK_EQ(output_q.dim(), 2) failed");
  const int64_t M = input.size(0), N = input.size(1) * 2;
  TORCH_CHECK(input_s.size(0) == M, "CHECK_EQ(input_s.size(0), M) failed");
  TORCH_CHECK(input_s.size(1) == (N + 31) / 32, "CHECK_EQ(input_s.size(1), (N + 31) / 32) failed");
  TORCH_CHECK(output_q.size(0) == N, "CHECK_EQ(output_q.size(0), N) failed");
  TORCH_CHECK(output_q.size(1) == M, "CHECK_EQ(output_q.size(1), M) failed");
  TORCH_CHECK(output_s.size(0) == (M + 127) / 128, "CHECK_EQ(output_s.size(0), (M + 127) / 128) failed");
  TORCH_CHECK(output_s.size(1) == N, "CHECK_EQ(output_s.size(1), N) failed");
  check_dtype(input, at::kByte, "input");
  check_dtype(input_s, at::kByte, "input_s");
  check_dtype(output_q, at::kFloat8_e4m3fn, "output_q");
  check_dtype(output_s, at::kFloat, "output_s");
  OMO_CHECK_INPUT(input_s);
  OMO_CHECK_INPUT(output_s);
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_Mxfp4RowToBf16ToFp8Col(input.data_ptr(), input_s.data_ptr(), M, N,
                                                    output_q.data_ptr(), output_s.data_ptr(),
                                                    (float)eps, cur_stream()),
               "omo_per_token_Mxfp4RowToBf16ToFp8Col");
}

// ---- per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu:232-282
void omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit(at::Tensor input, at::Tensor input_s,
                                                 at::Tensor output_q, at::Tensor output_s,
                                                 at::Tensor m_splits, at::Tensor split_offsets,
                                                 at::Tensor scale_offsets, int64_t max_split_len,
                                                 double eps) {
  OmoRange nvtx_range("omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit");
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  OMO_CHECK_INPUT(m_splits);
  OMO_CHECK_INPUT(split_offsets);
  OMO_CHECK_INPUT(scale_offsets);
  OMO_CHECK_INPUT(input_s);
  OMO_CHECK_INPUT(output_s);
  check_dtype(input, at::kByte, "input");
  check_dtype(input_s, at::kByte, "input_s");
  check_dtype(output_q, at::kFloat8_e4m3fn, "output_q");
  check_dtype(output_s, at::kFloat, "output_s");
  check_dtype(m_splits, at::kInt, "m_splits");
  check_dtype(split_offsets, at::kInt, "split_offsets");
  check_dtype(scale_offsets, at::kInt, "scale_offsets");
  const int64_t total_M = input.size(0), N = input.size(1) * 2;
  const int64_t ns = m_splits.size(0);
  TORCH_CHECK(split_offsets.numel() >= ns && scale_offsets.numel() >= ns,
              "split_offsets / scale_offsets must have one entry per split");
  if (total_M == 0 || N == 0 || ns == 0) return;
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit(
                   input.data_ptr(), input_s.data_ptr(), total_M, N, output_q.data_ptr(),
                   output_s.data_ptr(), m_splits.data_ptr<int32_t>(),
                   split_offsets.data_ptr<int32_t>(), scale_offsets.data_ptr<int32_t>(), ns,
                   max_split_len, (float)eps, cur_stream()),
               "omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit");
}

// ---- additions with no reference op of their own -------------------------
// One-pass rowwise + columnwise quantize (the reference runs Q-row on x and on
// x.T.contiguous(): transformer_engine-2.8.diff:1464-1466).  Pass empty
// tensors for the row outputs to quantize columnwise only.
void omo_quant_mxfp4_rowcol(at::Tensor input, at::Tensor codes_row, at::Tensor scales_row,
                            at::Tensor codes_col, at::Tensor scales_col,
                            c10::optional<at::Tensor> scales_row_swizzled, double eps,
                            double fp4_min, double fp4_max) {
  OmoRange nvtx_range("omo_quant_mxfp4_rowcol");
  OMO_CHECK_INPUT(input);
  check_dtype(input, at::kBFloat16, "input");
  TORCH_CHECK(input.dim() == 2, "input must be 2-D");
  const int64_t M = input.size(0), K = input.size(1);
  const bool rows = codes_row.numel() > 0;
  if (rows) {
    OMO_CHECK_INPUT(codes_row);
    OMO_CHECK_INPUT(scales_row);
    TORCH_CHECK(codes_row.numel() == M * K / 2 && scales_row.numel() == M * K / 32,
                "row outputs must be [M, K/2] and [M, K/32]");
  }
  OMO_CHECK_INPUT(codes_col);
  OMO_CHECK_INPUT(scales_col);
  TORCH_CHECK(codes_col.numel() == M * K / 2 && scales_col.numel() == M * K / 32,
              "column outputs must be [K, M/2] and [K, M/32]");
  void* swz = nullptr;
  if (scales_row_swizzled.has_value() && scales_row_swizzled->numel() > 0) {
    OMO_CHECK_INPUT((*scales_row_swizzled));
    TORCH_CHECK(scales_row_swizzled->numel() == (M + 127) / 128 * 128 * ((K / 32 + 3) / 4 * 4),
                "swizzled scales must be [round_up(M,128), round_up(K/32,4)]");
    swz = scales_row_swizzled->data_ptr();
  }
  if (M == 0 || K == 0) return;
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_quant_mxfp4_rowcol(input.data_ptr(), M, K, K,
                                      rows ? codes_row.data_ptr() : nullptr,
                                      rows ? scales_row.data_ptr() : nullptr, codes_col.data_ptr(),
                                      scales_col.data_ptr(), swz, (float)eps, (float)fp4_min,
                                      (float)fp4_max, cur_stream()),
               "omo_quant_mxfp4_rowcol");
}

void omo_swizzle_scales(at::Tensor scales, at::Tensor out) {
  OmoRange nvtx_range("omo_swizzle_scales");
  OMO_CHECK_INPUT(scales);
  OMO_CHECK_INPUT(out);
  TORCH_CHECK(scales.dim() == 2, "scales must be 2-D");
  const int64_t M = scales.size(0), S = scales.size(1);
  TORCH_CHECK(out.numel() == (M + 127) / 128 * 128 * ((S + 3) / 4 * 4),
              "out must be [round_up(M,128), round_up(S,4)]");
  c10::cuda::CUDAGuard g(scales.device());
  check_status(mxb_swizzle_scales(scales.data_ptr(), M, S, out.data_ptr(), cur_stream()),
               "omo_swizzle_scales");
}

void omo_per_token_quant_fp8(at::Tensor input, at::Tensor output_q, at::Tensor output_s,
                             double eps) {
  OmoRange nvtx_range("omo_per_token_quant_fp8");
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output_q);
  OMO_CHECK_INPUT(output_s);
  check_dtype(input, at::kBFloat16, "input");
  check_dtype(output_q, at::kFloat8_e4m3fn, "output_q");
  check_dtype(output_s, at::kFloat, "output_s");
  if (input.numel() == 0) return;
  const int64_t K = input.size(-1), M = input.numel() / K;
  TORCH_CHECK(output_q.numel() == M * K && output_s.numel() == M, "bad output sizes");
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_per_token_quant_fp8(input.data_ptr(), M, K, output_q.data_ptr(),
                                       output_s.data_ptr(), (float)eps, cur_stream()),
               "omo_per_token_quant_fp8");
}

void omo_per_token_dequant_fp8(at::Tensor input_q, at::Tensor input_s, at::Tensor output) {
  OmoRange nvtx_range("omo_per_token_dequant_fp8");
  OMO_CHECK_INPUT(input_q);
  OMO_CHECK_INPUT(input_s);
  OMO_CHECK_INPUT(output);
  check_dtype(input_q, at::kFloat8_e4m3fn, "input_q");
  check_dtype(input_s, at::kFloat, "input_s");
  check_dtype(output, at::kBFloat16, "output");
  if (input_q.numel() == 0) return;
  const int64_t K = input_q.size(-1), M = input_q.numel() / K;
  TORCH_CHECK(output.numel() == M * K && input_s.numel() == M, "bad sizes");
  c10::cuda::CUDAGuard g(input_q.device());
  check_status(mxb_per_token_dequant_fp8(input_q.data_ptr(), input_s.data_ptr(), M, K,
                                         output.data_ptr(), cur_stream()),
               "omo_per_token_dequant_fp8");
}

// ---- operators with no reference binding: the next rows of the path
void omo_swiglu_quant_mxfp4(at::Tensor input, at::Tensor output, at::Tensor codes,
                            at::Tensor scales, double eps, double fp4_min, double fp4_max) {
  OmoRange nvtx_range("omo_swiglu_quant_mxfp4");
  OMO_CHECK_INPUT(input);
  OMO_CHECK_INPUT(output);
  OMO_CHECK_INPUT(codes);
  OMO_CHECK_INPUT(scales);
  check_dtype(input, at::kBFloat16, "input");
  check_dtype(output, at::kBFloat16, "output");
  check_dtype(codes, at::kByte, "codes");
  check_dtype(scales, at::kByte, "scales");
  if (input.numel() == 0) return;
  const int64_t K = input.size(-1), M = input.numel() / K;
  TORCH_CHECK(K % 64 == 0, "omo_swiglu_quant_mxfp4: the last dimension (2H) must be a multiple of 64");
  TORCH_CHECK(output.numel() == M * K / 2 && codes.numel() == M * K / 2 &&
                  scales.numel() == M * K / 32,
              "omo_swiglu_quant_mxfp4: output [.., H], codes [.., H], scales [rows, 2H/32]");
  c10::cuda::CUDAGuard g(input.device());
  check_status(mxb_swiglu_quant_mxfp4(input.data_ptr(), M, K / 2, output.data_ptr(),
                                      codes.data_ptr(), scales.data_ptr(), (float)eps,
                                      (float)fp4_min, (float)fp4_max, cur_stream()),
               "omo_swiglu_quant_mxfp4");
}

void omo_moe_permute_mxfp4(at::Tensor codes, at::Tensor scales, at::Tensor dst,
                           at::Tensor out_codes, at::Tensor out_scales) {
  OmoRange nvtx_range("omo_moe_permute_mxfp4");
  OMO_CHECK_INPUT(codes);
  OMO_CHECK_INPUT(scales);
  OMO_CHECK_INPUT(dst);
  OMO_CHECK_INPUT(out_codes);
  OMO_CHECK_INPUT(out_scales);
  check_dtype(codes, at::kByte, "codes");
  check_dtype(scales, at::kByte, "scales");
  check_dtype(dst, at::kInt, "dst");
  TORCH_CHECK(codes.dim() == 2 && scales.dim() == 2 && dst.dim() == 2 &&
                  codes.size(0) == scales.size(0) && dst.size(0) == codes.size(0),
              "omo_moe_permute_mxfp4: codes [rows, H/2], scales [rows, H/32], dst [rows, topk]");
  const int64_t rows = codes.size(0), H = codes.size(1) * 2;
  TORCH_CHECK(scales.size(1) * 32 == H, "omo_moe_permute_mxfp4: scales must be [rows, H/32]");
  TORCH_CHECK(out_codes.dim() == 2 && out_codes.size(1) == H / 2 && out_scales.dim() == 2 &&
                  out_scales.size(1) == H / 32 && out_scales.size(0) == out_codes.size(0),
              "omo_moe_permute_mxfp4: out_codes [n_out, H/2], out_scales [n_out, H/32]");
  if (rows == 0) return;
  c10::cuda::CUDAGuard g(codes.device());
  check_status(mxb_moe_permute_mxfp4(codes.data_ptr(), H / 2, scales.data_ptr(), H / 32, rows, H,
                                     (const int32_t*)dst.data_ptr(), (int)dst.size(1),
                                     out_codes.data_ptr(), out_scales.data_ptr(),
                                     out_codes.size(0), cur_stream()),
               "omo_moe_permute_mxfp4");
}

void omo_gemm_mxfp4(at::Tensor a_codes, at::Tensor a_scales_swizzled, at::Tensor b_codes,
                    at::Tensor b_scales_swizzled, at::Tensor c) {
  OmoRange nvtx_range("omo_gemm_mxfp4");
  OMO_CHECK_INPUT(a_codes);
  OMO_CHECK_INPUT(a_scales_swizzled);
  OMO_CHECK_INPUT(b_codes);
  OMO_CHECK_INPUT(b_scales_swizzled);
  OMO_CHECK_INPUT(c);
  check_dtype(a_codes, at::kByte, "a_codes");
  check_dtype(b_codes, at::kByte, "b_codes");
  check_dtype(c, at::kBFloat16, "c");
  TORCH_CHECK(a_codes.dim() == 2 && b_codes.dim() == 2 && a_codes.size(1) == b_codes.size(1),
              "omo_gemm_mxfp4: a_codes [M, K/2] and b_codes [N, K/2]");
  const int64_t M = a_codes.size(0), N = b_codes.size(0), K = a_codes.size(1) * 2;
  TORCH_CHECK(c.numel() == M * N, "omo_gemm_mxfp4: c must be [M, N]");
  TORCH_CHECK(a_scales_swizzled.numel() == M * K / 32 && b_scales_swizzled.numel() == N * K / 32,
              "omo_gemm_mxfp4: swizzled scales must hold rows * K/32 bytes");
  c10::cuda::CUDAGuard g(a_codes.device());
  check_status(mxb_gemm_mxfp4(a_codes.data_ptr(), a_scales_swizzled.data_ptr(), b_codes.data_ptr(),
                              b_scales_swizzled.data_ptr(), M, N, K, c.data_ptr(), cur_stream()),
               "omo_gemm_mxfp4");
}

}  // namespace

PYBIND11_MODULE(omo, m) {
  m.doc() = "B200 (sm_100a) MXFP4 operators with the reference `omo` interface";
  m.def("omo_per_token_group_quant_fp4", &omo_per_token_group_quant_fp4,
        "Per-token-group FP4 quantization", py::arg("input"), py::arg("output_q"),
        py::arg("output_s"), py::arg("group_size"), py::arg("eps"), py::arg("fp4_min"),
        py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4ToBf16_dequant", &omo_per_token_Mxfp4ToBf16_dequant,
        "Per-token-group FP4 dequantization BF16", py::arg("input"), py::arg("input_s"),
        py::arg("output_q"), py::arg("output_s"), py::arg("group_size"), py::arg("eps"),
        py::arg("fp4_min"), py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4ToBf16ToFp8", &omo_per_token_Mxfp4ToBf16ToFp8,
        "Per-token-group FP4 dequantization BF16->FP8", py::arg("input"), py::arg("input_s"),
        py::arg("output_q"), py::arg("output_s"), py::arg("group_size"), py::arg("eps"),
        py::arg("fp4_min"), py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4ToFp8", &omo_per_token_Mxfp4ToFp8,
        "Per-token-group FP4 -> FP8 (1x128 groups)", py::arg("input"), py::arg("input_s"),
        py::arg("output_q"), py::arg("output_s"), py::arg("group_size"), py::arg("eps"),
        py::arg("fp4_min"), py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_per_token_group_quant_fp4_fused_ToFp8", &omo_per_token_group_quant_fp4_fused_ToFp8,
        "Per-token-group FP4 quantization fused ToFp8", py::arg("input"), py::arg("output_q"),
        py::arg("output_s"), py::arg("output_bf16_q"), py::arg("output_bf16_s"),
        py::arg("group_size"), py::arg("eps"), py::arg("fp4_min"), py::arg("fp4_max"),
        py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4RowToBf16ToFp8Col", &omo_per_token_Mxfp4RowToBf16ToFp8Col,
        "Per-token-group FP4(row) dequantization BF16->FP8(col)", py::arg("input"),
        py::arg("input_s"), py::arg("output_q"), py::arg("output_s"), py::arg("eps"));
  m.def("omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit", &omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit,
        "Per-token-group FP4 dequantization col FP8 for group linear(m_split)", py::arg("input"),
        py::arg("input_s"), py::arg("output_q"), py::arg("output_s"), py::arg("m_splits"),
        py::arg("split_offsets"), py::arg("scale_offsets"), py::arg("max_split_len"),
        py::arg("eps"));
  m.def("omo_per_token_Mxfp4ToFp8_col", &omo_per_token_Mxfp4ToFp8_col,
        "Per-token-group FP4 dequantization col FP8", py::arg("input"), py::arg("input_s"),
        py::arg("output_q"), py::arg("output_s"), py::arg("group_size"), py::arg("eps"),
        py::arg("fp4_min"), py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_quant_mxfp4_rowcol", &omo_quant_mxfp4_rowcol,
        "One-pass rowwise + columnwise MXFP4 quantization", py::arg("input"),
        py::arg("codes_row"), py::arg("scales_row"), py::arg("codes_col"), py::arg("scales_col"),
        py::arg("scales_row_swizzled") = py::none(), py::arg("eps") = 1e-10,
        py::arg("fp4_min") = -6.0, py::arg("fp4_max") = 6.0);
  m.def("omo_swizzle_scales", &omo_swizzle_scales, "E8M0 scales -> 128x4 swizzled layout",
        py::arg("scales"), py::arg("out"));
  m.def("omo_per_token_quant_fp8", &omo_per_token_quant_fp8, "Per-token FP8 quantization",
        py::arg("input"), py::arg("output_q"), py::arg("output_s"), py::arg("eps") = 1e-10);
  m.def("omo_per_token_dequant_fp8", &omo_per_token_dequant_fp8, "Per-token FP8 dequantization",
        py::arg("input_q"), py::arg("input_s"), py::arg("output"));
  m.def("omo_swiglu_quant_mxfp4", &omo_swiglu_quant_mxfp4,
        "SwiGLU of [.., 2H] and the rowwise MXFP4 of its input, one pass", py::arg("input"),
        py::arg("output"), py::arg("codes"), py::arg("scales"), py::arg("eps") = 1e-10,
        py::arg("fp4_min") = -6.0, py::arg("fp4_max") = 6.0);
  m.def("omo_moe_permute_mxfp4", &omo_moe_permute_mxfp4,
        "MoE permute of MXFP4 rows (codes and scales) to expert slots", py::arg("codes"),
        py::arg("scales"), py::arg("dst"), py::arg("out_codes"), py::arg("out_scales"));
  m.def("omo_gemm_mxfp4", &omo_gemm_mxfp4, "Block-scaled MXFP4 GEMM C = A . B^T (tcgen05)",
        py::arg("a_codes"), py::arg("a_scales_swizzled"), py::arg("b_codes"),
        py::arg("b_scales_swizzled"), py::arg("c"));
}
