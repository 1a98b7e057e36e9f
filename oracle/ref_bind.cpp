// Test infrastructure only. Python binding `omo_ref` for the reference's own
// CUDA launchers, compiled unmodified from the reference sources by
// oracle/build_ref.py. It stands in for code/kernel/ops.cu:27-43, which cannot
// be compiled because it includes two headers the reference does not ship
// (ops.cu:4-5). Argument names follow ops.cu.
#include <torch/extension.h>

#include "per_token_Mxfp4RowToBf16ToFp8Col.h"
#include "per_token_Mxfp4RowToBf16ToFp8Col_msplit.h"
#include "per_token_Mxfp4ToBf16_dequant.h"
#include "per_token_Mxfp4ToFp8.h"
#include "per_token_Mxfp4ToFp8_col.h"
#include "per_token_quant_mxfp4.h"

PYBIND11_MODULE(omo_ref, m) {
  m.def("omo_per_token_group_quant_fp4", &omo::omo_per_token_group_quant_fp4, py::arg("input"),
        py::arg("output_q"), py::arg("output_s"), py::arg("group_size"), py::arg("eps"),
        py::arg("fp4_min"), py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4ToBf16_dequant", &omo::omo_per_token_Mxfp4ToBf16_dequant,
        py::arg("input"), py::arg("input_s"), py::arg("output_q"), py::arg("output_s"),
        py::arg("group_size"), py::arg("eps"), py::arg("fp4_min"), py::arg("fp4_max"),
        py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4ToFp8", &omo::omo_per_token_Mxfp4ToFp8, py::arg("input"),
        py::arg("input_s"), py::arg("output_q"), py::arg("output_s"), py::arg("group_size"),
        py::arg("eps"), py::arg("fp4_min"), py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4ToFp8_col", &omo::omo_per_token_Mxfp4ToFp8_col, py::arg("input"),
        py::arg("input_s"), py::arg("output_q"), py::arg("output_s"), py::arg("group_size"),
        py::arg("eps"), py::arg("fp4_min"), py::arg("fp4_max"), py::arg("scale_ue8m0"));
  m.def("omo_per_token_Mxfp4RowToBf16ToFp8Col", &omo::omo_per_token_Mxfp4RowToBf16ToFp8Col,
        py::arg("input"), py::arg("input_s"), py::arg("output_q"), py::arg("output_s"),
        py::arg("eps"));
  m.def("omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit",
        &omo::omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit, py::arg("input"), py::arg("input_s"),
        py::arg("output_q"), py::arg("output_s"), py::arg("m_splits"), py::arg("split_offsets"),
        py::arg("scale_offsets"), py::arg("max_split_len"), py::arg("eps"));
}
