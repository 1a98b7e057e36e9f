"""ctypes binding of the C ABI (include/mxfp4_b200.h) of libmxfp4_b200.so.

This is how Python code outside torch (tests, the benchmark's end-to-end leg,
an FFI user) reaches the CUDA kernels: raw device pointers, sizes and a stream
handle, no torch types.  Loading fails loudly when the library has not been
built; there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
LIB_PATH = PKG / "lib" / "libmxfp4_b200.so"

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

# name -> argument types (all return mxb_status as int)
SIGNATURES = {
    "mxb_per_token_group_quant_fp4": [_P, _I64, _I64, _I64, _P, _P, _I, _F, _F, _F, _I, _P],
    "mxb_quant_mxfp4_rowcol": [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _F, _F, _F, _P],
    "mxb_per_token_group_quant_fp4_fused_ToFp8": [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I, _F,
                                                  _F, _F, _I, _P],
    "mxb_quant_mxfp4_rowcol_host": [_P, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _F, _F, _F,
                                    _P],
    "mxb_swiglu_quant_mxfp4": [_P, _I64, _I64, _P, _P, _P, _F, _F, _F, _P],
    "mxb_gemm_mxfp4": [_P, _P, _P, _P, _I64, _I64, _I64, _P, _P],
    "mxb_swizzle_scales": [_P, _I64, _I64, _P, _P],
    "mxb_per_token_Mxfp4ToBf16_dequant": [_P, _P, _I64, _I64, _P, _P],
    "mxb_per_token_Mxfp4ToFp8": [_P, _P, _I64, _I64, _P, _P, _P],
    "mxb_per_token_Mxfp4ToBf16ToFp8": [_P, _P, _I64, _I64, _P, _P, _P],
    "mxb_per_token_Mxfp4ToFp8_strict": [_P, _P, _I64, _I64, _P, _P, _P],
    "mxb_per_token_Mxfp4ToFp8_rowscale": [_P, _P, _I64, _I64, _P, _P, _F, _P],
    "mxb_quantize_mxfp4": [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I, _P],
    "mxb_per_token_Mxfp4ToFp8_col": [_P, _P, _I64, _I64, _P, _P, _P],
    "mxb_per_token_Mxfp4RowToBf16ToFp8Col": [_P, _P, _I64, _I64, _P, _P, _F, _P],
    "mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit": [_P, _P, _I64, _I64, _P, _P, _P, _P, _P,
                                                    _I64, _I64, _F, _P],
    "mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit_noalloc": [_P, _P, _I64, _I64, _P, _P, _P, _I64,
                                                            _I64, _F, _P],
    "mxb_per_token_quant_fp8": [_P, _I64, _I64, _P, _P, _F, _P],
    "mxb_per_token_dequant_fp8": [_P, _P, _I64, _I64, _P, _P],
    "mxb_ep_pack": [_P, _I64, _I64, _P, _I, _P, _F, _P],
    "mxb_ep_unpack": [_P, _I64, _I64, _P, _P, _P],
    "mxb_ep_combine": [_P, _I64, _I64, _P, _I, _P, _P],
    "mxb_moe_permute_mxfp4": [_P, _I64, _P, _I64, _I64, _I64, _P, _I, _P, _P, _I64, _P],
    "mxb_moe_make_row_id_map": [_P, _I64, _I, _P, _P, _P],
    "mxb_moe_permute_mxfp4_row_id_map": [_P, _I64, _P, _I64, _I64, _I64, _P, _I, _P, _P, _I64,
                                         _P],
}

class EpLayout(ctypes.Structure):
    """mxb_ep_layout of include/mxfp4_b200.h."""
    _fields_ = [("sig_off", ctypes.c_int64), ("cnt_off", ctypes.c_int64),
                ("wire_off", ctypes.c_int64), ("meta_off", ctypes.c_int64),
                ("back_off", ctypes.c_int64), ("tcap", ctypes.c_int64),
                ("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("topk", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("experts_per_rank", ctypes.c_int32)]


_LP = ctypes.POINTER(EpLayout)
_U32 = ctypes.c_uint32

SIGNATURES.update({
    "mxb_ep_layout_init": [ctypes.c_int32, ctypes.c_int32, _I64, ctypes.c_int32, ctypes.c_int32,
                           ctypes.c_int32, _LP, ctypes.POINTER(ctypes.c_int64)],
    "mxb_ipc_export": [_P, _P, ctypes.POINTER(ctypes.c_int64)],
    "mxb_ipc_import": [_P, _I64, ctypes.POINTER(ctypes.c_void_p)],
    "mxb_ipc_close": [_P, _I64],
    "mxb_ep_p2p_counts": [_P, _LP, _P, _I, _U32, _P],
    "mxb_ep_p2p_dispatch": [_P, _I64, _P, _P, _P, _P, _LP, _I, _P],
    "mxb_ep_p2p_barrier": [_P, _LP, _U32, _P],
    "mxb_ep_p2p_return": [_P, _P, _LP, _I, _P],
    "mxb_ep_route": [_P, _I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P, _P, _P],
    "mxb_ep_p2p_combine": [_P, _I64, _I64, _P, _P, ctypes.c_int32, _P, _P],
    "mxb_ep_set_wait_polls": [_U32],
})

class EpHandle(ctypes.Structure):
    """mxb_ep_handle of include/mxfp4_b200.h."""
    _fields_ = [("send_counts", ctypes.c_int64 * 64), ("recv_counts", ctypes.c_int64 * 64),
                ("n_send", ctypes.c_int64), ("n_recv", ctypes.c_int64), ("tokens", ctypes.c_int64),
                ("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("hidden", ctypes.c_int32),
                ("topk", ctypes.c_int32)]


_HP = ctypes.POINTER(EpHandle)
_I32 = ctypes.c_int32
SIGNATURES.update({
    "mxb_nccl_unique_id": [_P],
    "mxb_nccl_comm_init": [ctypes.POINTER(ctypes.c_void_p), _I32, _I32, _P],
    "mxb_nccl_comm_destroy": [_P],
    "mxb_ep_nccl_dispatch": [_P, _I32, _I32, _P, _I64, _I32, _P, _P, _I32, _I32, _P, _I64, _P, _P,
                             _I64, _HP, _P],
    "mxb_ep_nccl_combine": [_P, _HP, _P, _P, _I64, _P, _P],
})

STATUS = {0: "MXB_OK", 1: "MXB_ERR_INVALID_ARGUMENT", 2: "MXB_ERR_MISALIGNED", 3: "MXB_ERR_CUDA",
          4: "MXB_ERR_UNSUPPORTED"}


class MxbError(RuntimeError):
    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} -> {STATUS.get(status, status)}: {msg}")
        self.status = status


_lib = None


def load() -> ctypes.CDLL:
    """Load libmxfp4_b200.so and declare every exported entry point."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with "
                              "`python mxfp4-hopper_b200/build.py` (no CPU fallback exists)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        L.mxb_last_error.restype = ctypes.c_char_p
        L.mxb_version.restype = ctypes.c_char_p
        L.mxb_wait_timeouts.restype = ctypes.c_uint
        L.mxb_reset_wait_timeouts.restype = ctypes.c_uint
        L.mxb_ep_wait_timeouts.restype = ctypes.c_uint
        L.mxb_ep_reset_wait_timeouts.restype = ctypes.c_uint
        L.mxb_gemm_wait_timeouts.restype = ctypes.c_uint
        L.mxb_ep_nccl_workspace_bytes.argtypes = [_I64, _I32, _I32, _I32]
        L.mxb_ep_nccl_workspace_bytes.restype = ctypes.c_int64
        L.mxb_quant_mxfp4_rowcol_host_workspace.argtypes = [_I64, _I64, _I64]
        L.mxb_quant_mxfp4_rowcol_host_workspace.restype = ctypes.c_int64
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point and raise MxbError on a non-OK status."""
    L = load()
    st = getattr(L, name)(*args)
    if st != 0:
        raise MxbError(name, st, L.mxb_last_error().decode())


def status_of(name: str, *args) -> int:
    """Call an entry point and return its raw status (for error-path tests)."""
    return int(getattr(load(), name)(*args))


def last_error() -> str:
    return load().mxb_last_error().decode()


def wait_timeouts() -> int:
    """Bounded waits that gave up on the current device, over every kernel
    that waits on an mbarrier (quantizers, column converters, GEMM)."""
    return int(load().mxb_wait_timeouts())


def reset_wait_timeouts() -> int:
    return int(load().mxb_reset_wait_timeouts())


def version() -> str:
    return load().mxb_version().decode()
