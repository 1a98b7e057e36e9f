"""MXFP4 dequantize / convert wrappers (reference: code/kernel/api/mxfp4_dequant.py),
plus the two wrappers the reference's Transformer Engine patch imports but the
reference does not ship (transformer_engine-2.8.diff:70,199)."""
from __future__ import annotations

import torch
import torch.nn.functional as F

import mxfp4_b200  # noqa: F401
from omo import (omo_per_token_Mxfp4RowToBf16ToFp8Col, omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit,
                 omo_per_token_Mxfp4ToBf16_dequant, omo_per_token_Mxfp4ToBf16ToFp8,
                 omo_per_token_Mxfp4ToFp8, omo_per_token_Mxfp4ToFp8_col)

fp8_type_ = torch.float8_e4m3fn
uint8_type = torch.uint8
fp8_max = torch.finfo(fp8_type_).max
fp8_min = -fp8_max
mxfp4_max = 6.0
mxfp4_min = -mxfp4_max
FLOAT4_E2M1_MAX = 6.0
FLOAT8_E4M3_MAX = torch.finfo(torch.float8_e4m3fn).max


def pad_to_multiple(x, multiple=128):
    """Zero-pad the last dimension up to a multiple (api/mxfp4_dequant.py:15-29)."""
    last_dim = x.shape[-1]
    pad_amount = (multiple - (last_dim % multiple)) % multiple
    return (F.pad(x, (0, pad_amount)) if pad_amount > 0 else x), last_dim


def unpad_from_multiple(x_padded, original_size):
    return x_padded[..., :original_size]


def omo_per_token_mxfp4ToBf16_dequant_wrapper(x: torch.Tensor, x_in_s: torch.Tensor, dtype):
    """MXFP4 -> BF16, returned as `dtype` (api/mxfp4_dequant.py:39-76)."""
    assert x.shape[-1] % 32 == 0, "the last dimension of `x` cannot be divisible by `group_size`"
    assert x.is_contiguous(), "`x` is not contiguous"
    out_shape = (*x.shape[:-1], x.shape[-1] * 2)
    scale_shape = (*x.shape[:-1], x.shape[-1] * 2 // 128)
    x_q = torch.empty(out_shape, device=x.device, dtype=torch.bfloat16)
    x_s = torch.empty(scale_shape, device=x.device, dtype=torch.float)
    if x.shape[0] > 0:
        omo_per_token_Mxfp4ToBf16_dequant(x, x_in_s, x_q, x_s, 32, 1e-10, mxfp4_min, mxfp4_max,
                                          False)
    return x_q.to(dtype)


def omo_per_token_mxfp4ToBf16ToFp8_wrapper(x: torch.Tensor, x_in_s: torch.Tensor):
    """MXFP4 -> FP8 with 1x128 groups (api/mxfp4_dequant.py:79-121).  The code
    row is padded to 64 bytes and the scales to 4 columns, which the group
    layout needs."""
    assert x.is_contiguous(), "`x` is not contiguous"
    x_padded, original_w = pad_to_multiple(x, multiple=64)
    x_in_s_pad, _ = pad_to_multiple(x_in_s, multiple=4)
    out_shape = (*x_padded.shape[:-1], x_padded.shape[-1] * 2)
    scale_shape = ((x_padded.shape[-1] * 2 // 128), *x_padded.shape[:-1])
    x_q = torch.empty(out_shape, device=x.device, dtype=fp8_type_)
    x_s = torch.empty(scale_shape, device=x.device, dtype=torch.float)
    if x.shape[0] > 0:
        omo_per_token_Mxfp4ToBf16ToFp8(x_padded.contiguous(), x_in_s_pad.contiguous(), x_q, x_s,
                                       128, 1e-10, mxfp4_min, mxfp4_max, False)
    return x_q[:, :original_w * 2], x_s


def omo_per_token_mxfp4ToFp8_wrapper(x: torch.Tensor, x_in_s: torch.Tensor, m_splits=None):
    """MXFP4 -> FP8 (1x128 groups), split by rows into m_splits
    (api/mxfp4_dequant.py:122-187).  Returns (tuple of FP8 [m_i, K], tuple of
    FP32 scales [K/128, m_i]); with m_splits=None the unsplit pair."""
    assert x.is_contiguous(), "`x` is not contiguous"
    x_padded, original_w = pad_to_multiple(x, multiple=64)
    x_in_s_pad, original_w_scale = pad_to_multiple(x_in_s, multiple=4)
    out_shape = (*x_padded.shape[:-1], x_padded.shape[-1] * 2)
    scale_shape = ((x_padded.shape[-1] * 2 // 128), *x_padded.shape[:-1])
    x_q = torch.empty(out_shape, device=x.device, dtype=fp8_type_)
    x_s = torch.empty(scale_shape, device=x.device, dtype=torch.float)
    if x.shape[0] > 0:
        omo_per_token_Mxfp4ToFp8(x_padded.contiguous(), x_in_s_pad.contiguous(), x_q, x_s, 128,
                                 1e-10, mxfp4_min, mxfp4_max, False)
    x_q = x_q[:, :original_w * 2]
    x_s = x_s[:original_w_scale, :]
    if m_splits is None:
        return x_q, x_s
    return torch.split(x_q, m_splits, dim=0), torch.split(x_s, m_splits, dim=1)


def omo_per_token_mxfp4ToFp8_col_wrapper(x: torch.Tensor, x_in_s: torch.Tensor):
    """MXFP4 -> transposed FP8 [2K, M] with [M/128, 2K] scales
    (api/mxfp4_dequant.py:189-237)."""
    assert x.is_contiguous(), "`x` is not contiguous"
    x_padded, original_w = pad_to_multiple(x, multiple=16)
    out_shape = (x_padded.shape[-1] * 2, *x_padded.shape[:-1])
    scale_shape = ((x_padded.shape[0] // 128), x_padded.shape[-1] * 2)
    x_q = torch.empty(out_shape, device=x.device, dtype=fp8_type_)
    x_s = torch.empty(scale_shape, device=x.device, dtype=torch.float)
    if x.shape[0] > 0:
        omo_per_token_Mxfp4ToFp8_col(x_padded.contiguous(), x_in_s, x_q, x_s, 128, 1e-10,
                                     mxfp4_min, mxfp4_max, False)
    return x_q[..., :original_w * 2], x_s


def omo_per_token_mxfp4RowToBf16ToFp8Col_wrapper(x: torch.Tensor, x_in_s: torch.Tensor,
                                                 eps: float = 1e-10):
    """MXFP4 (rowwise) -> columnwise FP8 [N, M] with amax/448 scales
    [ceil(M/128), N]: the wgrad operand of _Linear.backward
    (transformer_engine-2.8.diff:259; kernel per_token_Mxfp4RowToBf16ToFp8Col.cu)."""
    assert x.dim() == 2 and x.is_contiguous(), "`x` must be a contiguous 2-D tensor"
    M, N = x.shape[0], x.shape[1] * 2
    y = torch.empty((N, M), device=x.device, dtype=fp8_type_)
    s = torch.empty(((M + 127) // 128, N), device=x.device, dtype=torch.float)
    if M > 0:
        omo_per_token_Mxfp4RowToBf16ToFp8Col(x, x_in_s.contiguous(), y, s, eps)
    return y, s


def msplit_offsets(m_splits):
    """(split_offsets, scale_offsets, max_split_len) for the msplit kernel."""
    so, sco, acc, accs = [], [], 0, 0
    for m in m_splits:
        so.append(acc)
        sco.append(accs)
        acc += int(m)
        accs += (int(m) + 127) // 128
    return so, sco, (max(int(m) for m in m_splits) if len(m_splits) else 0), accs


def omo_per_token_mxfp4RowToBf16ToFp8Col_msplit_wrapper(x: torch.Tensor, x_in_s: torch.Tensor,
                                                        m_splits, eps: float = 1e-10):
    """Grouped-GEMM wgrad operand (transformer_engine-2.8.diff:159-163; kernel
    per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu): rows split into m_splits, each
    split quantized columnwise with power-of-two scales.  Returns (list of FP8
    [N, m_i], list of FP32 1/scale [ceil(m_i/128), N])."""
    assert x.dim() == 2 and x.is_contiguous(), "`x` must be a contiguous 2-D tensor"
    M, N = x.shape[0], x.shape[1] * 2
    m_splits = [int(m) for m in m_splits]
    assert sum(m_splits) == M, "m_splits must sum to the number of rows"
    so, sco, max_len, nblk = msplit_offsets(m_splits)
    out = torch.empty((N * M,), device=x.device, dtype=fp8_type_)
    scales = torch.empty((nblk, N), device=x.device, dtype=torch.float)
    if M > 0 and len(m_splits) > 0:
        dev = x.device
        t = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731
        omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit(x, x_in_s.contiguous(), out, scales,
                                                    t(m_splits), t(so), t(sco), max_len, eps)
    ys, ss = [], []
    for m, o, sb in zip(m_splits, so, sco):
        ys.append(out[o * N:(o + m) * N].view(N, m))
        ss.append(scales[sb:sb + (m + 127) // 128])
    return ys, ss
