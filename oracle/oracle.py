"""TEST INFRASTRUCTURE ONLY: numpy front end of the CPU oracle (liborc.so).

The oracle is the bit-exact restatement of the reference kernels in
`oracle/mxfp4_oracle.c`; each function below names the reference kernel it
follows.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg may import this module; the product never does.

Arrays: BF16 tensors are passed as uint16 bit patterns, FP8 E4M3 as uint8,
MXFP4 codes and E8M0 scales as uint8, all C-contiguous.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liborc.so"

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_lib = None


def build(force: bool = False) -> Path:
    src = HERE / "mxfp4_oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        env = dict(os.environ)
        env.pop("CC", None)
        subprocess.run(["make", "-C", str(HERE), "-B", "liborc.so", "CC=gcc"], check=True,
                       capture_output=True, env=env)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB))
        sig = {
            "orc_quant_mxfp4_rows": [_P, _I64, _I64, _I64, _F, _F, _F, _P, _P],
            "orc_quant_mxfp4_cols": [_P, _I64, _I64, _I64, _F, _F, _F, _P, _P],
            "orc_quant_mxfp4_rows_ocp": [_P, _I64, _I64, _I64, _P, _P],
            "orc_quant_mxfp4_cols_ocp": [_P, _I64, _I64, _I64, _P, _P],
            "orc_mxfp4_to_fp8_rows_strict": [_P, _P, _I64, _I64, _P, _P],
            "orc_swizzle_scales": [_P, _I64, _I64, _P],
            "orc_dequant_bf16": [_P, _P, _I64, _I64, _P],
            "orc_mxfp4_to_fp8_rows": [_P, _P, _I64, _I64, _P, _P],
            "orc_mxfp4_to_fp8_cols": [_P, _P, _I64, _I64, _P, _P],
            "orc_mxfp4_to_fp8_colT": [_P, _P, _I64, _I64, _F, _P, _P],
            "orc_mxfp4_to_fp8_colT_split": [_P, _P, _I64, _P, _P, _P, _I64, _F, _P, _P],
            "orc_fp8_quant_rows": [_P, _I64, _I64, _F, _P, _P],
            "orc_fp8_dequant_rows": [_P, _P, _I64, _I64, _P],
            "orc_set_num_threads": [ctypes.c_int],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None
        L.orc_f32_to_e4m3.argtypes = [_F]
        L.orc_f32_to_e4m3.restype = ctypes.c_uint8
        L.orc_f32_to_bf16.argtypes = [_F]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ---------------------------------------------------------------- quantize
def quant_rows(x_bf16: np.ndarray, eps=1e-10, fp4_min=-6.0, fp4_max=6.0, rule="reference"):
    """Q-row, per_token_quant_mxfp4.cu:121-266 -> (codes [M,K/2], scales [M,K/32]).
    rule="ocp": the OCP MX scale rule instead (default eps and clamp only)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    codes = np.empty((M, K // 2), np.uint8)
    scales = np.empty((M, K // 32), np.uint8)
    if rule == "ocp":
        lib().orc_quant_mxfp4_rows_ocp(_p(x), M, K, K, _p(codes), _p(scales))
    else:
        lib().orc_quant_mxfp4_rows(_p(x), M, K, K, eps, fp4_min, fp4_max, _p(codes), _p(scales))
    return codes, scales


def quant_cols(x_bf16: np.ndarray, eps=1e-10, fp4_min=-6.0, fp4_max=6.0, rule="reference"):
    """Q-col: Q-row of x.T (transformer_engine-2.8.diff:1465-1466) -> ([K,M/2], [K,M/32])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    codes = np.empty((K, M // 2), np.uint8)
    scales = np.empty((K, M // 32), np.uint8)
    if rule == "ocp":
        lib().orc_quant_mxfp4_cols_ocp(_p(x), M, K, K, _p(codes), _p(scales))
    else:
        lib().orc_quant_mxfp4_cols(_p(x), M, K, K, eps, fp4_min, fp4_max, _p(codes), _p(scales))
    return codes, scales


def swizzle_scales(s: np.ndarray) -> np.ndarray:
    """128x4-tile swizzled E8M0 layout (transformer_engine-2.8.diff:752-786)."""
    s = np.ascontiguousarray(s, dtype=np.uint8)
    M, S = s.shape
    out = np.empty(((M + 127) // 128 * 128, (S + 3) // 4 * 4), np.uint8)
    lib().orc_swizzle_scales(_p(s), M, S, _p(out))
    return out


# ---------------------------------------------------------------- dequantize
def dequant_bf16(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """DQ-bf16, per_token_Mxfp4ToBf16_dequant.cu:70-160 -> bf16 bits [M, 2*Kb]."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint8)
    M, Kb = c.shape
    out = np.empty((M, 2 * Kb), np.uint16)
    lib().orc_dequant_bf16(_p(c), _p(s), M, Kb, _p(out))
    return out


def mxfp4_to_fp8_rows(codes: np.ndarray, scales: np.ndarray):
    """DQ-fp8-row, per_token_Mxfp4ToFp8.cu:92-235 -> (fp8 [M,2Kb], f32 scales [Kb/64, M])."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint8)
    M, Kb = c.shape
    out = np.empty((M, 2 * Kb), np.uint8)
    so = np.empty((Kb // 64, M), np.float32)
    lib().orc_mxfp4_to_fp8_rows(_p(c), _p(s), M, Kb, _p(out), _p(so))
    return out, so


def mxfp4_to_fp8_rows_strict(codes: np.ndarray, scales: np.ndarray):
    """Rowwise FP8 convert without the re-basing wrap (true values; no reference
    counterpart) -> (fp8 [M,2Kb], f32 scales [Kb/64, M])."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint8)
    M, Kb = c.shape
    out = np.empty((M, 2 * Kb), np.uint8)
    so = np.empty((Kb // 64, M), np.float32)
    lib().orc_mxfp4_to_fp8_rows_strict(_p(c), _p(s), M, Kb, _p(out), _p(so))
    return out, so


def mxfp4_to_fp8_rowscale(codes: np.ndarray, scales: np.ndarray, eps=1e-10):
    """MXFP4 -> FP8 with one FP32 scale per row: DQ-bf16 then the per-token FP8
    quantize (parity unpinned: no reference kernel) -> (fp8 [M,2Kb], f32 [M])."""
    return fp8_quant_rows(dequant_bf16(codes, scales), eps)


def mxfp4_to_fp8_cols(codes: np.ndarray, scales: np.ndarray):
    """DQ-fp8-col, per_token_Mxfp4ToFp8_col.cu:110-301 -> (fp8 [2Kb, M], f32 [M/128, 2Kb])."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint8)
    M, Kb = c.shape
    out = np.empty((2 * Kb, M), np.uint8)
    so = np.empty((M // 128, 2 * Kb), np.float32)
    lib().orc_mxfp4_to_fp8_cols(_p(c), _p(s), M, Kb, _p(out), _p(so))
    return out, so


def mxfp4_to_fp8_colT(codes: np.ndarray, scales: np.ndarray, eps=1e-10):
    """DQ-fp8-colT, per_token_Mxfp4RowToBf16ToFp8Col.cu:42-197 -> (fp8 [N,M], f32 [ceil(M/128), N])."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint8)
    M, Kb = c.shape
    N = 2 * Kb
    out = np.empty((N, M), np.uint8)
    so = np.empty(((M + 127) // 128, N), np.float32)
    lib().orc_mxfp4_to_fp8_colT(_p(c), _p(s), M, N, eps, _p(out), _p(so))
    return out, so


def split_offsets(m_splits):
    """Prefix sums the msplit kernel takes: (split_offsets, scale_offsets, max_split_len)."""
    m = np.asarray(m_splits, dtype=np.int64)
    so = np.concatenate([[0], np.cumsum(m)[:-1]]).astype(np.int32)
    blocks = (m + 127) // 128
    sco = np.concatenate([[0], np.cumsum(blocks)[:-1]]).astype(np.int32)
    return so, sco, int(m.max()) if len(m) else 0


def mxfp4_to_fp8_colT_split(codes: np.ndarray, scales: np.ndarray, m_splits, eps=1e-10):
    """DQ-fp8-colT-split, per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu:51-224.

    Returns (fp8 flat [N * Total_M] holding per-split [N, m_i] blocks,
    f32 scales [sum ceil(m_i/128), N])."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint8)
    M, Kb = c.shape
    N = 2 * Kb
    ms = np.asarray(m_splits, dtype=np.int32)
    assert int(ms.sum()) == M
    so, sco, _ = split_offsets(ms)
    nblk = int(((ms.astype(np.int64) + 127) // 128).sum())
    out = np.empty((N * M,), np.uint8)
    sc = np.empty((nblk, N), np.float32)
    lib().orc_mxfp4_to_fp8_colT_split(_p(c), _p(s), N, _p(ms), _p(so), _p(sco), len(ms), eps,
                                       _p(out), _p(sc))
    return out, sc


# ---------------------------------------------------------------- per-token FP8
def fp8_quant_rows(x_bf16: np.ndarray, eps=1e-10):
    """Per-token FP8 quantize (parity unpinned) -> (fp8 [M,K], f32 [M])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    q = np.empty((M, K), np.uint8)
    s = np.empty((M,), np.float32)
    lib().orc_fp8_quant_rows(_p(x), M, K, eps, _p(q), _p(s))
    return q, s


def fp8_dequant_rows(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """Per-token FP8 dequantize -> bf16 bits [M, K]."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.float32)
    M, K = q.shape
    out = np.empty((M, K), np.uint16)
    lib().orc_fp8_dequant_rows(_p(q), _p(s), M, K, _p(out))
    return out


def f32_to_e4m3(v: float) -> int:
    return int(lib().orc_f32_to_e4m3(float(v)))


def f32_to_bf16(v: float) -> int:
    return int(lib().orc_f32_to_bf16(float(v)))
