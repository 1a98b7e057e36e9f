"""CPU-only checks of the C ABI: the library loads, exports every entry point
include/*.h declares, and rejects out-of-contract arguments with a status and
a message before touching the GPU."""
import re
from pathlib import Path

import pytest

from mxfp4_b200 import capi

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        txt = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:mxb_status|const char\s*\*|unsigned int)\s*(mxb_\w+)\s*\(", txt, flags=re.M)
    return names


def test_library_loads_and_reports_version():
    assert "sm_100a" in capi.version()


def test_every_declared_symbol_is_exported():
    L = capi.load()
    names = declared_symbols()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/ but not exported"
    for n in capi.SIGNATURES:
        assert n in names, f"{n} bound in capi.py but not declared in include/"


@pytest.mark.parametrize("name,args,status", [
    ("mxb_per_token_group_quant_fp4", (1, 4, 40, 40, 1, 1, 32, 1e-10, -6.0, 6.0, 0, None), 1),
    ("mxb_per_token_group_quant_fp4", (1, 4, 64, 64, 1, 1, 16, 1e-10, -6.0, 6.0, 0, None), 4),
    ("mxb_per_token_group_quant_fp4", (1, 4, 64, 64, 1, 1, 32, 1e-10, -6.0, 6.0, 1, None), 4),
    ("mxb_per_token_group_quant_fp4", (1, 4, 64, 60, 1, 1, 32, 1e-10, -6.0, 6.0, 0, None), 2),
    ("mxb_quant_mxfp4_rowcol", (1, 48, 64, 64, 1, 1, 1, 1, None, 1e-10, -6.0, 6.0, None), 1),
    ("mxb_quant_mxfp4_rowcol", (1, 64, 64, 64, 1, None, 1, 1, None, 1e-10, -6.0, 6.0, None), 1),
    ("mxb_per_token_Mxfp4ToBf16_dequant", (1, 1, 4, 24, 1, None), 1),
    ("mxb_per_token_Mxfp4ToFp8", (1, 1, 4, 96, 1, 1, None), 1),
    ("mxb_per_token_Mxfp4ToFp8_col", (1, 1, 64, 128, 1, 1, None), 1),
    ("mxb_per_token_Mxfp4RowToBf16ToFp8Col", (1, 1, 4, 48, 1, 1, 1e-10, None), 1),
    ("mxb_per_token_quant_fp8", (1, 4, 12, 1, 1, 1e-10, None), 1),
    ("mxb_per_token_dequant_fp8", (1, 1, 4, 20, 1, None), 1),
])
def test_out_of_contract_arguments_are_rejected(name, args, status):
    assert capi.status_of(name, *args) == status
    assert capi.last_error()


def test_empty_inputs_are_a_no_op():
    assert capi.status_of("mxb_per_token_group_quant_fp4", None, 0, 64, 64, None, None, 32, 1e-10,
                          -6.0, 6.0, 0, None) == 0
    assert capi.status_of("mxb_per_token_Mxfp4ToBf16_dequant", None, None, 0, 16, None, None) == 0


@pytest.mark.parametrize("args", [
    # N not a multiple of 32
    (1, 1, 256, 40, 1, 1, 1, 2, 256, 1e-10, None),
    # null input
    (None, 1, 256, 64, 1, 1, 1, 2, 256, 1e-10, None),
    # misaligned input
    (17, 1, 256, 64, 1, 1, 1, 2, 256, 1e-10, None),
    # too many rows per split for the grid
    (1, 1, 256, 64, 1, 1, 1, 2, 128 * 65536, 1e-10, None),
])
def test_noalloc_split_rejects_before_touching_scratch(args):
    """The no-alloc split converter validates every argument before it launches
    the offset scan into its shared device array: these calls return an error
    without any CUDA call (this container has no GPU, so a CUDA call would
    report MXB_ERR_CUDA instead)."""
    st = capi.status_of("mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit_noalloc", *args)
    assert st in (1, 2), (st, capi.last_error())
    assert "CUDA" not in capi.last_error()


def test_nccl_unique_id_and_dispatch_argument_checks():
    """The NCCL entry points open libnccl at run time: a unique id needs no GPU;
    a dispatch with an impossible world size is rejected before any NCCL or CUDA
    call."""
    import ctypes
    from mxfp4_b200.ep import NcclCDispatcher
    a, b = NcclCDispatcher.unique_id(), NcclCDispatcher.unique_id()
    assert len(a) == 128 and a != b
    h = capi.EpHandle()
    st = capi.status_of("mxb_ep_nccl_dispatch", 1, 0, 0, 1, 4, 7168, 1, 1, 8, 32, 1, 1 << 20, 1, 1,
                        16, ctypes.byref(h), None)
    assert st == 1 and "bad arguments" in capi.last_error()
    assert capi.load().mxb_ep_nccl_workspace_bytes(4096, 7168, 8, 8) > 4096 * 8 * 3808


@pytest.mark.parametrize("name,args,status,needle", [
    # GEMM tiles: M % 128, N % 256, K % 256; 16-byte aligned operands
    ("mxb_gemm_mxfp4", (1, 1, 1, 1, 100, 256, 256, 1, None), 1, "M % 128"),
    ("mxb_gemm_mxfp4", (1, 1, 1, 1, 128, 128, 256, 1, None), 1, "N % 256"),
    ("mxb_gemm_mxfp4", (1, 1, 1, 1, 128, 256, 128, 1, None), 1, "K % 256"),
    ("mxb_gemm_mxfp4", (17, 1, 1, 1, 128, 256, 256, 1, None), 2, "aligned"),
    ("mxb_gemm_mxfp4", (None, 1, 1, 1, 128, 256, 256, 1, None), 1, "null"),
    # split converter with caller-supplied offsets
    ("mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit",
     (1, 1, 256, 40, 1, 1, 1, 1, 1, 2, 256, 1e-10, None), 1, "N % 32"),
    ("mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit",
     (None, 1, 256, 64, 1, 1, 1, 1, 1, 2, 256, 1e-10, None), 1, "null"),
    # SwiGLU + quantize: H % 32
    ("mxb_swiglu_quant_mxfp4", (1, 4, 40, 1, 1, 1, 1e-10, -6.0, 6.0, None), 1, "H % 32"),
    ("mxb_swiglu_quant_mxfp4", (None, 4, 64, 1, 1, 1, 1e-10, -6.0, 6.0, None), 1, "null"),
    # fused Q-row + rowwise FP8: group size 32 only (as the reference), K % 128
    ("mxb_per_token_group_quant_fp4_fused_ToFp8",
     (1, 4, 64, 64, 1, 1, 1, 1, 16, 1e-10, -6.0, 6.0, 0, None), 4, "group_size"),
    ("mxb_per_token_group_quant_fp4_fused_ToFp8",
     (1, 4, 40, 40, 1, 1, 1, 1, 32, 1e-10, -6.0, 6.0, 0, None), 1, "K % 128"),
    # scale rule must be 0 (reference) or 1 (OCP)
    ("mxb_quantize_mxfp4", (1, 64, 64, 64, 1, 1, 1, 1, None, 7, None), 1, "scale rule"),
    ("mxb_quantize_mxfp4", (1, 48, 64, 64, 1, 1, 1, 1, None, 0, None), 1, "M % 32"),
    # the strict and aliased rowwise FP8 converters keep the 1x128 group rule
    ("mxb_per_token_Mxfp4ToFp8_strict", (1, 1, 4, 96, 1, 1, None), 1, "Kb % 64"),
    ("mxb_per_token_Mxfp4ToBf16ToFp8", (1, 1, 4, 96, 1, 1, None), 1, "Kb % 64"),
    ("mxb_per_token_Mxfp4ToFp8_rowscale", (1, 1, 4, 24, 1, 1, 1e-10, None), 1, "Kb % 16"),
    ("mxb_per_token_Mxfp4ToFp8_rowscale", (None, 1, 4, 64, 1, 1, 1e-10, None), 1, "null"),
    ("mxb_swizzle_scales", (None, 4, 4, 1, None), 1, "null"),
    # EP wire rows: H % 128, 1 <= G <= 64
    ("mxb_ep_pack", (1, 4, 40, 1, 0, 1, 1e-10, None), 1, "H % 128"),
    ("mxb_ep_unpack", (1, 4, 40, 1, 1, None), 1, "H % 128"),
])
def test_entry_point_contracts(name, args, status, needle):
    """Every remaining entry point with a shape or pointer rule rejects an
    out-of-contract call with its status and a message naming the rule, before
    any CUDA call (this container has no GPU: a CUDA call would report
    MXB_ERR_CUDA)."""
    assert capi.status_of(name, *args) == status
    msg = capi.last_error()
    assert needle in msg, msg
    assert "CUDA" not in msg
