"""The drop-in boundary: the `omo` operators (code/kernel/ops.cu:27-43) and the
`omo_python_api` wrappers (code/kernel/api/mxfp4.py, api/mxfp4_dequant.py, plus the
two wrappers the Transformer Engine patch imports) called the way the reference's
callers call them, against the CPU oracle.  Error behaviour follows the reference:
a RuntimeError from the operator, an AssertionError from a wrapper."""
import numpy as np
import pytest
import torch

import helpers as H
from mxfp4_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api(cuda):
    import omo
    from omo_python_api import mxfp4, mxfp4_dequant
    return omo, mxfp4, mxfp4_dequant


def _codes(M, Kb, seed, lo=110, hi=140):
    c, s = syn.config3(M, Kb, seed=seed, lo=lo, hi=hi)
    return c, s


# ------------------------------------------------------------------ quantize
@pytest.mark.parametrize("shape", [(256, 512), (3, 7, 256)])
def test_quant_mxfp4_wrapper(cuda, orc, api, shape):
    _, mx, _ = api
    x = syn.config1(int(np.prod(shape[:-1])), shape[-1], seed=21).reshape(shape)
    q, s = mx.omo_per_token_group_quant_mxfp4(x.to(cuda))
    rq, rs = orc.quant_rows(H.np_u16(x.reshape(-1, shape[-1])))
    assert tuple(q.shape) == (*shape[:-1], shape[-1] // 2)
    H.assert_bytes_equal(H.np_u8(q).reshape(rq.shape), rq, "codes")
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")


def test_quant_fp4_warppers(cuda, orc, api):
    _, mx, _ = api
    x = syn.config1(128, 1024, seed=22)
    rq, rs = orc.quant_rows(H.np_u16(x))
    for fn in (lambda t: mx.omo_per_token_group_quant_fp4_warpper(t, 32),
               lambda t: mx.omo_per_token_group_quant_4bit_warpper(t, 32, torch.uint8)):
        q, s = fn(x.to(cuda))
        H.assert_bytes_equal(H.np_u8(q), rq, "codes")
        # as on the reference, the scale tensor is sized from the code shape and
        # the scales fill its first numel/32 bytes (per_token_quant_mxfp4.cu:161)
        assert tuple(s.shape) == tuple(q.shape)
        H.assert_bytes_equal(H.np_u8(s).reshape(-1)[:rs.size], rs.reshape(-1), "scales")


def test_quant_rowcol_wrapper(cuda, orc, api):
    _, mx, _ = api
    x = syn.config2(256, 512, seed=23)
    xb = H.np_u16(x)
    cr, sr, cc, sc, swz = mx.omo_per_token_group_quant_mxfp4_rowcol(x.to(cuda),
                                                                   swizzled_scales=True)
    rq, rs = orc.quant_rows(xb)
    rcq, rcs = orc.quant_cols(xb)
    H.assert_bytes_equal(H.np_u8(cr), rq, "row codes")
    H.assert_bytes_equal(H.np_u8(sr), rs, "row scales")
    H.assert_bytes_equal(H.np_u8(cc), rcq, "col codes")
    H.assert_bytes_equal(H.np_u8(sc), rcs, "col scales")
    H.assert_bytes_equal(H.np_u8(swz), orc.swizzle_scales(rs), "swizzled scales")


def test_fused_to_fp8_op_and_wrapper(cuda, orc, api):
    omo, mx, _ = api
    x = syn.config1(64, 2048, seed=24)
    xb = H.np_u16(x)
    rq, rs = orc.quant_rows(xb)
    rf, rfs = orc.mxfp4_to_fp8_rows(rq, rs)
    q, s, f, fs = mx.omo_per_token_group_quant_mxfp4_fused_fp8(x.to(cuda))
    for a, b, what in ((q, rq, "codes"), (s, rs, "scales"), (f, rf, "fp8")):
        H.assert_bytes_equal(H.np_u8(a), b, what)
    H.assert_bytes_equal(H.np_f32(fs).view(np.uint32), rfs.view(np.uint32), "fp8 scales")


def test_quant_op_errors(cuda, api):
    omo, _, _ = api
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    q = torch.empty(4, 32, dtype=torch.uint8, device=cuda)
    s = torch.empty(4, 2, dtype=torch.uint8, device=cuda)
    with pytest.raises(RuntimeError):  # the reference's host assert on scale_ue8m0
        omo.omo_per_token_group_quant_fp4(x, q, s, 32, 1e-10, -6.0, 6.0, True)
    with pytest.raises(RuntimeError):  # BF16 input only
        omo.omo_per_token_group_quant_fp4(x.float(), q, s, 32, 1e-10, -6.0, 6.0, False)


# ------------------------------------------------------------------ dequantize / convert
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_dequant_bf16_wrapper(cuda, orc, api, dtype):
    _, _, dq = api
    c, s = _codes(64, 256, seed=25, lo=0, hi=255)
    y = dq.omo_per_token_mxfp4ToBf16_dequant_wrapper(c.to(cuda), s.to(cuda), dtype)
    ref = orc.dequant_bf16(c.numpy(), s.numpy())
    assert y.dtype == dtype
    H.assert_bytes_equal(H.np_u16(y.to(torch.bfloat16)), ref, "bf16")


@pytest.mark.parametrize("Kb", [128, 80])  # 80: the wrappers pad the code row to 64 bytes
def test_fp8_row_wrappers(cuda, orc, api, Kb):
    _, _, dq = api
    M = 48
    c, s = _codes(M, Kb, seed=26)
    pad = (-Kb) % 64
    cp = np.pad(c.numpy(), ((0, 0), (0, pad)))
    sp = np.pad(s.numpy(), ((0, 0), (0, (-(Kb // 16)) % 4)))
    rf, rfs = orc.mxfp4_to_fp8_rows(cp, sp[:, :cp.shape[1] // 16])
    rf = rf[:, :2 * Kb]
    for fn in (dq.omo_per_token_mxfp4ToBf16ToFp8_wrapper, dq.omo_per_token_mxfp4ToFp8_wrapper):
        f, fs = fn(c.to(cuda), s.to(cuda))
        H.assert_bytes_equal(H.np_u8(f), rf, "fp8")
        H.assert_bytes_equal(H.np_f32(fs).view(np.uint32)[:, :M],
                             rfs[:fs.shape[0]].view(np.uint32), "scales")
    fsp, ssp = dq.omo_per_token_mxfp4ToFp8_wrapper(c.to(cuda), s.to(cuda), m_splits=[16, 32])
    assert [t.shape[0] for t in fsp] == [16, 32] and [t.shape[1] for t in ssp] == [16, 32]
    H.assert_bytes_equal(np.concatenate([H.np_u8(t) for t in fsp]), rf, "split fp8")


def test_fp8_col_wrapper(cuda, orc, api):
    _, _, dq = api
    c, s = _codes(256, 128, seed=27)
    f, fs = dq.omo_per_token_mxfp4ToFp8_col_wrapper(c.to(cuda), s.to(cuda))
    rf, rfs = orc.mxfp4_to_fp8_cols(c.numpy(), s.numpy())
    H.assert_bytes_equal(H.np_u8(f), rf, "fp8")
    H.assert_bytes_equal(H.np_f32(fs).view(np.uint32), rfs.view(np.uint32), "scales")


def test_colT_wrappers(cuda, orc, api):
    _, _, dq = api
    c, s = _codes(300, 96, seed=28)
    f, fs = dq.omo_per_token_mxfp4RowToBf16ToFp8Col_wrapper(c.to(cuda), s.to(cuda))
    rf, rfs = orc.mxfp4_to_fp8_colT(c.numpy(), s.numpy())
    H.assert_bytes_equal(H.np_u8(f), rf, "colT fp8")
    H.assert_bytes_equal(H.np_f32(fs).view(np.uint32), rfs.view(np.uint32), "colT scales")
    splits = [100, 0, 77, 123]
    ys, ss = dq.omo_per_token_mxfp4RowToBf16ToFp8Col_msplit_wrapper(c.to(cuda), s.to(cuda), splits)
    rq, rs = orc.mxfp4_to_fp8_colT_split(c.numpy(), s.numpy(), splits)
    N = 2 * c.shape[1]
    assert [tuple(y.shape) for y in ys] == [(N, m) for m in splits]
    H.assert_bytes_equal(np.concatenate([H.np_u8(y).reshape(-1) for y in ys]), rq.reshape(-1),
                         "split fp8")
    H.assert_bytes_equal(np.concatenate([H.np_f32(t).view(np.uint32) for t in ss]),
                         rs.view(np.uint32), "split scales")


def test_wrapper_rejects_non_contiguous(cuda, api):
    _, _, dq = api
    c, s = _codes(64, 128, seed=29)
    with pytest.raises(AssertionError):
        dq.omo_per_token_mxfp4ToBf16_dequant_wrapper(c.to(cuda).t(), s.to(cuda), torch.bfloat16)


# ------------------------------------------------------------------ next rows of the path
def test_swiglu_quant_wrapper(cuda, orc, api):
    _, mx, _ = api
    x = syn.config1(96, 1024, seed=51)
    y, q, s = mx.omo_swiglu_quant_mxfp4(x.to(cuda))
    rq, rs = orc.quant_rows(H.np_u16(x))
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    xf = x.float()
    ref = (torch.nn.functional.silu(xf[:, :512]) * xf[:, 512:]).to(torch.bfloat16)
    assert np.abs(H.np_u16(y).astype(np.int32) - H.np_u16(ref).astype(np.int32)).max() <= 1


def test_moe_permute_wrapper(cuda, api):
    _, mx, _ = api
    g = np.random.default_rng(52)
    rows, Hd, topk = 64, 1024, 4
    codes = torch.from_numpy(g.integers(0, 256, (rows, Hd // 2), dtype=np.uint8)).to(cuda)
    scales = torch.from_numpy(g.integers(100, 150, (rows, Hd // 32), dtype=np.uint8)).to(cuda)
    dst = torch.from_numpy(g.permutation(rows * topk).astype(np.int32).reshape(rows, topk)).to(cuda)
    oc, os_ = mx.omo_moe_permute_mxfp4(codes, scales, dst, rows * topk)
    inv = torch.empty(rows * topk, dtype=torch.long, device=cuda)
    inv[dst.reshape(-1).long()] = torch.arange(rows, device=cuda).repeat_interleave(topk)
    assert torch.equal(oc, codes[inv]) and torch.equal(os_, scales[inv])


def test_gemm_wrapper(cuda, api):
    _, mx, _ = api
    from test_gemm_gpu import dequant_np
    a = syn.config2(256, 512, seed=53)
    b = syn.config2(256, 512, seed=54)
    qa, sa = mx.omo_per_token_group_quant_mxfp4(a.to(cuda))
    qb, sb = mx.omo_per_token_group_quant_mxfp4(b.to(cuda))
    c = mx.omo_gemm_mxfp4(qa, sa, qb, sb)
    ref = dequant_np(H.np_u8(qa), H.np_u8(sa)) @ dequant_np(H.np_u8(qb), H.np_u8(sb)).T
    scale = np.maximum(np.abs(ref).max(axis=1, keepdims=True), 1e-30)
    assert (np.abs(c.float().cpu().numpy() - ref) / scale).max() < 2 ** -7
