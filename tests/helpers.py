"""Test helpers: call the C ABI with torch CUDA tensors, convert results."""
import numpy as np
import torch

from mxfp4_b200 import capi


def ptr(t):
    return torch.tensor([], dtype=torch.uint8) if t is None else t


def stream():
    return torch.cuda.current_stream().cuda_stream


def dp(t):
    return None if t is None else t.data_ptr()


def np_u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def np_u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def np_f32(t):
    return t.detach().cpu().contiguous().float().numpy()


def bf16_from_bits(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def quant_rows(x, eps=1e-10, fmin=-6.0, fmax=6.0):
    M, K = x.shape
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    s = torch.empty(M, K // 32, dtype=torch.uint8, device=x.device)
    capi.call("mxb_per_token_group_quant_fp4", dp(x), M, K, K, dp(q), dp(s), 32, eps, fmin, fmax,
              0, stream())
    return q, s


def quant_fused_fp8(x, eps=1e-10, fmin=-6.0, fmax=6.0):
    """Q-row and its rowwise FP8 conversion in one launch."""
    M, K = x.shape
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    s = torch.empty(M, K // 32, dtype=torch.uint8, device=x.device)
    f = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    fs = torch.empty(K // 128, M, dtype=torch.float32, device=x.device)
    capi.call("mxb_per_token_group_quant_fp4_fused_ToFp8", dp(x), M, K, K, dp(q), dp(s), dp(f),
              dp(fs), 32, eps, fmin, fmax, 0, stream())
    return q, s, f, fs


def swiglu_quant(x, eps=1e-10, fmin=-6.0, fmax=6.0):
    """silu(x[:, :H]) * x[:, H:] and the rowwise MXFP4 of x, one launch."""
    M, K = x.shape
    Hh = K // 2
    y = torch.empty(M, Hh, dtype=torch.bfloat16, device=x.device)
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    s = torch.empty(M, K // 32, dtype=torch.uint8, device=x.device)
    capi.call("mxb_swiglu_quant_mxfp4", dp(x), M, Hh, dp(y), dp(q), dp(s), eps, fmin, fmax,
              stream())
    return y, q, s


def quant_rowcol(x, rows=True, swz=False, eps=1e-10, fmin=-6.0, fmax=6.0):
    M, K = x.shape
    dev = x.device
    cr = torch.empty(M, K // 2, dtype=torch.uint8, device=dev) if rows else None
    sr = torch.empty(M, K // 32, dtype=torch.uint8, device=dev) if rows else None
    cc = torch.empty(K, M // 2, dtype=torch.uint8, device=dev)
    sc = torch.empty(K, M // 32, dtype=torch.uint8, device=dev)
    sw = torch.empty((M + 127) // 128 * 128, (K // 32 + 3) // 4 * 4, dtype=torch.uint8,
                     device=dev) if swz else None
    capi.call("mxb_quant_mxfp4_rowcol", dp(x), M, K, K, dp(cr), dp(sr), dp(cc), dp(sc), dp(sw),
              eps, fmin, fmax, stream())
    return cr, sr, cc, sc, sw


def quantize(x, rows=True, cols=False, swz=False, rule=0):
    """mxb_quantize_mxfp4: rowwise and/or columnwise with a scale rule
    (0 reference, 1 OCP)."""
    M, K = x.shape
    dev = x.device
    cr = torch.empty(M, K // 2, dtype=torch.uint8, device=dev) if rows else None
    sr = torch.empty(M, K // 32, dtype=torch.uint8, device=dev) if rows else None
    cc = torch.empty(K, M // 2, dtype=torch.uint8, device=dev) if cols else None
    sc = torch.empty(K, M // 32, dtype=torch.uint8, device=dev) if cols else None
    sw = torch.empty((M + 127) // 128 * 128, (K // 32 + 3) // 4 * 4, dtype=torch.uint8,
                     device=dev) if swz else None
    capi.call("mxb_quantize_mxfp4", dp(x), M, K, K, dp(cr), dp(sr), dp(cc), dp(sc), dp(sw), rule,
              stream())
    return cr, sr, cc, sc, sw


def to_fp8_rowscale(codes, scales, eps=1e-10):
    """MXFP4 -> FP8 with one FP32 scale per row."""
    M, Kb = codes.shape
    q = torch.empty(M, 2 * Kb, dtype=torch.float8_e4m3fn, device=codes.device)
    s = torch.empty(M, dtype=torch.float32, device=codes.device)
    capi.call("mxb_per_token_Mxfp4ToFp8_rowscale", dp(codes), dp(scales), M, Kb, dp(q), dp(s), eps,
              stream())
    return q, s


def dequant_bf16(codes, scales):
    M, Kb = codes.shape
    out = torch.empty(M, 2 * Kb, dtype=torch.bfloat16, device=codes.device)
    capi.call("mxb_per_token_Mxfp4ToBf16_dequant", dp(codes), dp(scales), M, Kb, dp(out), stream())
    return out


def to_fp8_rows(codes, scales, name="mxb_per_token_Mxfp4ToFp8"):
    M, Kb = codes.shape
    q = torch.empty(M, 2 * Kb, dtype=torch.float8_e4m3fn, device=codes.device)
    s = torch.empty(Kb // 64, M, dtype=torch.float32, device=codes.device)
    capi.call(name, dp(codes), dp(scales), M, Kb, dp(q), dp(s), stream())
    return q, s


def to_fp8_cols(codes, scales):
    M, Kb = codes.shape
    q = torch.empty(2 * Kb, M, dtype=torch.float8_e4m3fn, device=codes.device)
    s = torch.empty(M // 128, 2 * Kb, dtype=torch.float32, device=codes.device)
    capi.call("mxb_per_token_Mxfp4ToFp8_col", dp(codes), dp(scales), M, Kb, dp(q), dp(s), stream())
    return q, s


def to_fp8_colT(codes, scales, eps=1e-10):
    M, Kb = codes.shape
    N = 2 * Kb
    q = torch.empty(N, M, dtype=torch.float8_e4m3fn, device=codes.device)
    s = torch.empty((M + 127) // 128, N, dtype=torch.float32, device=codes.device)
    capi.call("mxb_per_token_Mxfp4RowToBf16ToFp8Col", dp(codes), dp(scales), M, N, dp(q), dp(s),
              eps, stream())
    return q, s


def to_fp8_colT_split(codes, scales, m_splits, eps=1e-10):
    M, Kb = codes.shape
    N = 2 * Kb
    so, sco, acc, accs = [], [], 0, 0
    for m in m_splits:
        so.append(acc); sco.append(accs)
        acc += m; accs += (m + 127) // 128
    dev = codes.device
    t = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731
    ms, sot, scot = t(m_splits), t(so), t(sco)
    q = torch.empty(N * M, dtype=torch.float8_e4m3fn, device=dev)
    s = torch.empty(max(accs, 1), N, dtype=torch.float32, device=dev)
    capi.call("mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit", dp(codes), dp(scales), M, N, dp(q),
              dp(s), dp(ms), dp(sot), dp(scot), len(m_splits), max(m_splits) if m_splits else 0,
              eps, stream())
    return q, s[:accs]


def quant_fp8(x, eps=1e-10):
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    capi.call("mxb_per_token_quant_fp8", dp(x), M, K, dp(q), dp(s), eps, stream())
    return q, s


def dequant_fp8(q, s):
    M, K = q.shape
    out = torch.empty(M, K, dtype=torch.bfloat16, device=q.device)
    capi.call("mxb_per_token_dequant_fp8", dp(q), dp(s), M, K, dp(out), stream())
    return out


def assert_bytes_equal(a, b, what=""):
    a = np.asarray(a)
    b = np.asarray(b)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    av = a.view(np.uint8) if a.dtype != np.uint8 else a
    bv = b.view(np.uint8) if b.dtype != np.uint8 else b
    if not np.array_equal(av, bv):
        d = np.argwhere(a != b) if a.dtype == b.dtype else np.argwhere(av != bv)
        raise AssertionError(f"{what}: {len(d)} mismatches, first at {d[:5].tolist()}: "
                             f"got {a[tuple(d[0])]} want {b[tuple(d[0])]}")
