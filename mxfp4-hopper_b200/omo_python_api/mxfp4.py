"""MXFP4 quantize wrappers (reference: code/kernel/api/mxfp4.py).

Outputs are allocated here and filled by the sm_100a kernels through `omo`.
"""
from __future__ import annotations

from typing import Optional

import torch

import mxfp4_b200  # noqa: F401
from omo import (omo_per_token_group_quant_fp4, omo_per_token_group_quant_fp4_fused_ToFp8,
                 omo_quant_mxfp4_rowcol, omo_swizzle_scales)
from omo import omo_gemm_mxfp4 as _gemm_op
from omo import omo_moe_permute_mxfp4 as _permute_op
from omo import omo_swiglu_quant_mxfp4 as _swiglu_op

fp8_type_ = torch.float8_e4m3fn
uint8_type = torch.uint8
fp8_max = torch.finfo(fp8_type_).max
fp8_min = -fp8_max
mxfp4_max = 6.0
mxfp4_min = -mxfp4_max
FLOAT4_E2M1_MAX = 6.0
FLOAT8_E4M3_MAX = torch.finfo(torch.float8_e4m3fn).max


def align(x: int, y: int) -> int:
    return (x + y - 1) // y * y


def create_per_token_group_quant_fp8_output_scale(x_shape, device, group_size,
                                                  column_major_scales: bool,
                                                  scale_tma_aligned: bool, scale_ue8m0: bool):
    """Scale tensor for a quantize call (api/mxfp4.py:133-161).

    With scale_ue8m0 the reference builds a column-major packed int32 layout that
    its kernel path asserts against; the row-major uint8 [rows, cols] layout is
    the one every caller uses."""
    if scale_ue8m0:
        assert column_major_scales and scale_tma_aligned
        *x_batch, x_q_mn, x_q_k = x_shape
        x_s_mn, x_s_k = x_q_mn, x_q_k // 128
        aligned_mn = align(x_s_mn, 4)
        aligned_k = align(x_s_k, 4)
        return torch.empty((*x_batch, aligned_k // 4, aligned_mn), device=device,
                           dtype=torch.int).transpose(-1, -2)[..., :x_s_mn, :]
    return torch.empty((x_shape[0], x_shape[1]), device=device, dtype=torch.uint8)


def omo_per_token_group_quant_fp4_warpper(x: torch.Tensor, group_size: int, eps: float = 1e-10,
                                          column_major_scales: bool = False,
                                          scale_tma_aligned: bool = False,
                                          scale_ue8m0: bool = False,
                                          fuse_silu_and_mul: bool = False,
                                          masked_m: Optional[torch.Tensor] = None,
                                          enable_v2: Optional[bool] = None):
    """api/mxfp4.py:91-127 (the scale tensor is sized from the code shape, as there)."""
    assert x.shape[-1] % group_size == 0, \
        "the last dimension of `x` cannot be divisible by `group_size`"
    assert x.is_contiguous(), "`x` is not contiguous"
    out_shape = (*x.shape[:-1], x.shape[-1] // 2)
    x_q = torch.empty(out_shape, device=x.device, dtype=uint8_type)
    x_s = create_per_token_group_quant_fp8_output_scale(
        x_shape=out_shape, device=x.device, group_size=group_size,
        column_major_scales=column_major_scales, scale_tma_aligned=scale_tma_aligned,
        scale_ue8m0=scale_ue8m0)
    if x.shape[0] > 0:
        omo_per_token_group_quant_fp4(x, x_q, x_s, group_size, eps, mxfp4_min, mxfp4_max,
                                      scale_ue8m0)
    return x_q, x_s


def omo_per_token_group_quant_4bit_warpper(x: torch.Tensor, group_size: int,
                                           dst_dtype: torch.dtype, eps: float = 1e-10,
                                           column_major_scales: bool = False,
                                           scale_tma_aligned: bool = False,
                                           scale_ue8m0: bool = False,
                                           fuse_silu_and_mul: bool = False,
                                           masked_m: Optional[torch.Tensor] = None,
                                           enable_v2: Optional[bool] = None):
    """api/mxfp4.py:63-90: forwards to the FP4 wrapper."""
    return omo_per_token_group_quant_fp4_warpper(
        x=x, group_size=group_size, eps=eps, column_major_scales=column_major_scales,
        scale_tma_aligned=scale_tma_aligned, scale_ue8m0=scale_ue8m0,
        fuse_silu_and_mul=fuse_silu_and_mul, masked_m=masked_m, enable_v2=enable_v2)


def omo_per_token_group_quant_mxfp4(x: torch.Tensor):
    """Rowwise MXFP4 quantize (api/mxfp4.py:164-202): codes [..., K/2] uint8 and
    E8M0 scales [rows, K/32] uint8 (leading dimensions flattened into rows)."""
    group_size = 32
    assert x.shape[-1] % group_size == 0, \
        "the last dimension of `x` cannot be divisible by `group_size`"
    assert x.is_contiguous(), "`x` is not contiguous"
    out_shape = (*x.shape[:-1], x.shape[-1] // 2)
    rows = x.numel() // x.shape[-1] if x.shape[-1] else 0
    x_q = torch.empty(out_shape, device=x.device, dtype=uint8_type)
    x_s = torch.empty((rows, x.shape[-1] // 32), device=x.device, dtype=torch.uint8)
    if x.shape[0] > 0:
        omo_per_token_group_quant_fp4(x, x_q, x_s, group_size, 1e-10, mxfp4_min, mxfp4_max, False)
    return x_q, x_s


def omo_per_token_group_quant_mxfp4_rowcol(x: torch.Tensor, rowwise: bool = True,
                                           swizzled_scales: bool = False):
    """Rowwise and columnwise MXFP4 quantize of a 2-D tensor in one pass.

    Same bytes as `omo_per_token_group_quant_mxfp4(x)` plus
    `omo_per_token_group_quant_mxfp4(x.T.contiguous())` (the Transformer Engine
    quantize, transformer_engine-2.8.diff:1464-1466), without the transpose copy.
    Returns (codes_row, scales_row, codes_col, scales_col[, scales_row_swizzled]);
    the row pair is None when rowwise=False."""
    assert x.dim() == 2 and x.is_contiguous()
    M, K = x.shape
    dev = x.device
    cr = torch.empty((M, K // 2), device=dev, dtype=torch.uint8) if rowwise else \
        torch.empty(0, device=dev, dtype=torch.uint8)
    sr = torch.empty((M, K // 32), device=dev, dtype=torch.uint8) if rowwise else \
        torch.empty(0, device=dev, dtype=torch.uint8)
    cc = torch.empty((K, M // 2), device=dev, dtype=torch.uint8)
    sc = torch.empty((K, M // 32), device=dev, dtype=torch.uint8)
    swz = torch.empty((align(M, 128), align(K // 32, 4)), device=dev, dtype=torch.uint8) \
        if swizzled_scales else None
    omo_quant_mxfp4_rowcol(x, cr, sr, cc, sc, swz)
    out = (cr if rowwise else None, sr if rowwise else None, cc, sc)
    return out + (swz,) if swizzled_scales else out


def omo_per_token_group_quant_mxfp4_fused_fp8(x: torch.Tensor):
    """Rowwise MXFP4 quantize and its rowwise FP8 conversion in one pass (the op
    the reference binds as omo_per_token_group_quant_fp4_fused_ToFp8, ops.cu:34,
    without a shipped wrapper).  Returns (codes [M, K/2] uint8, E8M0 scales
    [M, K/32] uint8, FP8 [M, K], FP32 group scales [K/128, M]); K % 128 == 0."""
    assert x.dim() == 2 and x.is_contiguous(), "`x` must be a contiguous 2-D tensor"
    M, K = x.shape
    dev = x.device
    x_q = torch.empty((M, K // 2), device=dev, dtype=uint8_type)
    x_s = torch.empty((M, K // 32), device=dev, dtype=uint8_type)
    y = torch.empty((M, K), device=dev, dtype=fp8_type_)
    y_s = torch.empty((K // 128, M), device=dev, dtype=torch.float)
    if M > 0:
        omo_per_token_group_quant_fp4_fused_ToFp8(x, x_q, x_s, y, y_s, 32, 1e-10, mxfp4_min,
                                                  mxfp4_max, False)
    return x_q, x_s, y, y_s


def omo_swiglu_quant_mxfp4(x: torch.Tensor):
    """Megatron's SwiGLU with fp4_input_store in one pass (megatron-0.15.0rc7.diff:164-193):
    returns (silu(x[..., :H]) * x[..., H:] as BF16 [..., H], the rowwise MXFP4 of x: codes
    [..., H] uint8 and E8M0 scales [rows, 2H/32] uint8)."""
    assert x.is_contiguous() and x.shape[-1] % 64 == 0, "`x` must be contiguous with 2H % 64 == 0"
    H = x.shape[-1] // 2
    rows = x.numel() // x.shape[-1] if x.shape[-1] else 0
    y = torch.empty((*x.shape[:-1], H), device=x.device, dtype=torch.bfloat16)
    q = torch.empty((*x.shape[:-1], H), device=x.device, dtype=uint8_type)
    s = torch.empty((rows, x.shape[-1] // 32), device=x.device, dtype=uint8_type)
    if rows > 0:
        _swiglu_op(x, y, q, s)
    return y, q, s


def omo_moe_permute_mxfp4(codes: torch.Tensor, scales: torch.Tensor, dst: torch.Tensor,
                          num_out: int):
    """MoE permute of MXFP4 rows (the MXFP4 branch of TE's moe_permute,
    transformer_engine-2.8.diff:253-261,338-356): row i of codes [rows, H/2] and scales
    [rows, H/32] goes to output rows dst[i, k] (int32 [rows, topk]; -1 = none) of the
    returned (codes [num_out, H/2], scales [num_out, H/32])."""
    oc = torch.empty((num_out, codes.shape[1]), device=codes.device, dtype=uint8_type)
    os_ = torch.empty((num_out, scales.shape[1]), device=codes.device, dtype=uint8_type)
    _permute_op(codes.contiguous(), scales.contiguous(), dst.to(torch.int32).contiguous(), oc, os_)
    return oc, os_


def omo_gemm_mxfp4(a_codes: torch.Tensor, a_scales: torch.Tensor, b_codes: torch.Tensor,
                   b_scales: torch.Tensor) -> torch.Tensor:
    """C = A . B^T in BF16 on the tcgen05 tensor cores from MXFP4 operands as the rowwise
    quantizer returns them (codes [rows, K/2], E8M0 scales [rows, K/32]); the scales are
    swizzled into the 128x4 block-scale layout here.  M % 128, N % 256, K % 256 == 0."""
    M, N = a_codes.shape[0], b_codes.shape[0]
    sa = torch.empty((align(M, 128), align(a_scales.shape[1], 4)), device=a_codes.device,
                     dtype=uint8_type)
    sb = torch.empty((align(N, 128), align(b_scales.shape[1], 4)), device=b_codes.device,
                     dtype=uint8_type)
    omo_swizzle_scales(a_scales.contiguous(), sa)
    omo_swizzle_scales(b_scales.contiguous(), sb)
    c = torch.empty((M, N), device=a_codes.device, dtype=torch.bfloat16)
    _gemm_op(a_codes.contiguous(), sa, b_codes.contiguous(), sb, c)
    return c
