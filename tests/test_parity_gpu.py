"""Parity of the sm_100a kernels (called through the C ABI) with the CPU oracle.

Bit-exact for every output: MXFP4 codes, E8M0 scales, BF16 / FP8 bytes and
FP32 scales.  Inputs are seeded; sizes are those the oracle finishes in
seconds, plus the full BASELINE shapes where the oracle is fast enough.
"""
import numpy as np
import pytest
import torch

import helpers as H
from mxfp4_b200 import capi
from mxfp4_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _bits(x):
    return syn.bf16_bits(x)


# ------------------------------------------------------------------ inputs
def special_block_input():
    """Rows exercising zero blocks, -0, bf16 subnormals, Inf, NaN, ties."""
    rows = []
    z = np.zeros(64, np.uint16)
    rows.append(z.copy())                                   # all +0
    r = z.copy(); r[:] = 0x8000; rows.append(r)             # all -0
    r = z.copy(); r[0:32] = np.arange(1, 33); rows.append(r)  # subnormals
    r = z.copy(); r[3] = 0x7F80; r[40] = 0xFF80; rows.append(r)  # +Inf / -Inf
    r = z.copy(); r[5] = 0x7FC0; r[6] = 0x3F80; r[33] = 0xFFC1; r[34] = 0xC000; rows.append(r)  # NaN
    r = z.copy(); r[:32] = 0x40C0; r[32:] = 0xC0C0; rows.append(r)  # +-6 exact
    ties = np.array([0x3E80, 0x3F40, 0x3FA0, 0x3FE0, 0x4020, 0x4060, 0x40A0, 0x40B0], np.uint16)
    r = z.copy(); r[:8] = ties; r[8:16] = ties | 0x8000; r[16] = 0x40C0; r[32:40] = ties; rows.append(r)
    r = z.copy(); r[:] = 0x7F7F; rows.append(r)             # bf16 max
    r = z.copy(); r[0] = 0x0001; r[1] = 0x8001; rows.append(r)
    return np.stack(rows)


def scale_kat_input():
    """KAT (b): one block per positive finite BF16 amax value (32767 blocks)."""
    v = np.arange(1, 0x7F80, dtype=np.uint16)
    x = np.zeros((len(v), 32), np.uint16)
    x[:, 0] = v
    x[:, 17] = v | 0x8000  # the same magnitude, negative
    return x


def encode_kat_input():
    """KAT (c): every BF16 value of magnitude <= 6 * 2^k as an element of a block
    whose amax is pinned to 6 * 2^k, for several k."""
    blocks = []
    for k in (-33, -20, -3, 0, 5, 40, 120):
        lim = np.float32(6.0) * np.float32(2.0) ** k
        allv = np.arange(0, 0x10000, dtype=np.uint32).astype(np.uint16)
        f = (allv.astype(np.uint32) << 16).view(np.float32)
        ok = np.isfinite(f) & (np.abs(f) <= lim)
        vals = allv[ok]
        pad = (-len(vals)) % 31
        vals = np.concatenate([vals, np.zeros(pad, np.uint16)]).reshape(-1, 31)
        head = np.full((vals.shape[0], 1), (np.array([lim], np.float32).view(np.uint32) >> 16)[0],
                       np.uint16)
        blocks.append(np.concatenate([head, vals], axis=1))
    x = np.concatenate(blocks)
    pad = (-x.shape[0]) % 4
    x = np.concatenate([x, np.zeros((pad, 32), np.uint16)])
    return x.reshape(-1, 128)


def to_dev_bf16(bits, cuda):
    return H.bf16_from_bits(bits).to(cuda)


# ------------------------------------------------------------------ Q-row
@pytest.mark.parametrize("shape", [(1, 32), (3, 96), (256, 4096), (4096, 4096)])
def test_quant_rows_config1(cuda, orc, shape):
    x = syn.config1(*shape, seed=0)
    q, s = H.quant_rows(x.to(cuda))
    rq, rs = orc.quant_rows(_bits(x))
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")


def test_quant_rows_special_values(cuda, orc):
    xb = special_block_input()
    q, s = H.quant_rows(to_dev_bf16(xb, cuda))
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")


def test_quant_rows_scale_kat_exhaustive(cuda, orc):
    xb = scale_kat_input()
    q, s = H.quant_rows(to_dev_bf16(xb, cuda))
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")


def test_quant_rows_encode_kat(cuda, orc):
    xb = encode_kat_input()
    q, s = H.quant_rows(to_dev_bf16(xb, cuda))
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")


@pytest.mark.parametrize("eps,fmin,fmax", [(1e-3, -6.0, 6.0), (1e-10, -4.0, 4.0),
                                           (1e-10, -6.0, 8.0), (0.5, -6.0, 6.0)])
def test_quant_rows_generic_params(cuda, orc, eps, fmin, fmax):
    x = syn.config1(128, 512, seed=7)
    xb = np.concatenate([_bits(x), special_block_input()[:, :512 // 8].repeat(8, 1)[:, :512]])
    q, s = H.quant_rows(to_dev_bf16(xb, cuda), eps, fmin, fmax)
    rq, rs = orc.quant_rows(xb, eps, fmin, fmax)
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")


# -------------------------------------------- SwiGLU fused with Q-row
@pytest.mark.parametrize("M,hid", [(64, 512), (3, 4096), (200, 7168)])
def test_swiglu_quant(cuda, orc, M, hid):
    """The MXFP4 of the input is bit-exact with Q-row; silu(g) * u (f32, one BF16
    rounding) is within one BF16 ulp of torch's f32 evaluation."""
    x = syn.config1(M, 2 * hid, seed=19)
    y, q, s = H.swiglu_quant(x.to(cuda))
    rq, rs = orc.quant_rows(_bits(x))
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")
    xf = x.float()
    ref = (torch.nn.functional.silu(xf[:, :hid]) * xf[:, hid:]).to(torch.bfloat16)
    a = H.np_u16(y).astype(np.int32)
    b = H.np_u16(ref).astype(np.int32)
    # same-sign BF16 patterns: ulp distance is the integer difference
    assert np.abs(a - b).max() <= 1, f"max ulp difference {np.abs(a - b).max()}"


def test_swiglu_quant_special_values(cuda, orc):
    """Quantization of Inf / NaN / subnormal / tie inputs through the fused kernel."""
    sp = special_block_input()
    xb = np.concatenate([sp, sp[:, ::-1]], axis=1)  # 2H = 128
    y, q, s = H.swiglu_quant(to_dev_bf16(xb, cuda))
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")


# -------------------------------------------- rowcol on host buffers (pipelined)
@pytest.mark.parametrize("M,K,chunk", [(4192, 1024, 512), (4096, 512, 0), (96, 256, 128)])
def test_quant_rowcol_host(cuda, M, K, chunk):
    """The host-buffer entry point equals the device call byte for byte, including a
    partial last chunk (M not a multiple of chunk_rows)."""
    from mxfp4_b200 import capi
    x = syn.config2(M, K, seed=17)
    cr, sr, cc, sc, _ = H.quant_rowcol(x.to(cuda))
    xh = x.pin_memory()
    outs = [torch.full(tuple(t.shape), 0x77, dtype=torch.uint8).pin_memory() for t in (cr, sr, cc, sc)]
    L = capi.load()
    wb = int(L.mxb_quant_mxfp4_rowcol_host_workspace(M, K, chunk))
    ws = torch.empty(wb, dtype=torch.uint8, device=cuda)
    capi.call("mxb_quant_mxfp4_rowcol_host", xh.data_ptr(), M, K, *[t.data_ptr() for t in outs],
              ws.data_ptr(), wb, chunk, 1e-10, -6.0, 6.0, H.stream())
    torch.cuda.synchronize()
    for got, want, what in zip(outs, (cr, sr, cc, sc), ("codes_row", "scales_row", "codes_col",
                                                        "scales_col")):
        H.assert_bytes_equal(got.numpy(), H.np_u8(want), what)


# -------------------------------------------- fused Q-row + rowwise FP8
def _fused_cases():
    x = syn.config1(64, 1024, seed=8)
    sp = special_block_input()
    sp128 = np.concatenate([sp, sp[:, ::-1]], axis=1)  # 128 columns: 1x128 FP8 groups
    return {
        "config1": (_bits(x), (1e-10, -6.0, 6.0)),
        "special": (sp128, (1e-10, -6.0, 6.0)),
        "generic": (np.concatenate([_bits(x), sp128.repeat(8, 1)]), (1e-3, -4.0, 4.0)),
        "deep_exponents": (_bits(syn.config2(32, 7168, seed=9)), (1e-10, -6.0, 6.0)),
    }


@pytest.mark.parametrize("case", ["config1", "special", "generic", "deep_exponents"])
def test_quant_fused_fp8(cuda, orc, case):
    """One pass equals Q-row followed by the rowwise FP8 convert, byte for byte,
    against the oracle and against the two separate launches."""
    xb, (eps, fmin, fmax) = _fused_cases()[case]
    q, s, f, fs = H.quant_fused_fp8(to_dev_bf16(xb, cuda), eps, fmin, fmax)
    rq, rs = orc.quant_rows(xb, eps, fmin, fmax)
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")
    rf, rfs = orc.mxfp4_to_fp8_rows(rq, rs)
    H.assert_bytes_equal(H.np_u8(f), rf, "fp8")
    H.assert_bytes_equal(H.np_f32(fs).view(np.uint32), rfs.view(np.uint32), "fp8 scales")
    q2, s2 = H.quant_rows(to_dev_bf16(xb, cuda), eps, fmin, fmax)
    f2, fs2 = H.to_fp8_rows(q2, s2)
    H.assert_bytes_equal(H.np_u8(f), H.np_u8(f2), "fp8 vs two launches")


def test_quant_fused_fp8_rejects_k_not_128(cuda):
    from mxfp4_b200 import capi
    x = torch.zeros(4, 96, dtype=torch.bfloat16, device=cuda)
    st = capi.status_of("mxb_per_token_group_quant_fp4_fused_ToFp8", x.data_ptr(), 4, 96, 96,
                        x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 32, 1e-10, -6.0,
                        6.0, 0, H.stream())
    assert st == 1 and "128" in capi.last_error()


def test_quant_rows_strided_input(cuda, orc):
    from mxfp4_b200 import capi
    x = syn.config2(64, 512, seed=5)
    big = torch.zeros(64, 640, dtype=torch.bfloat16)
    big[:, :512] = x
    bd = big.to(cuda)
    q = torch.empty(64, 256, dtype=torch.uint8, device=cuda)
    s = torch.empty(64, 16, dtype=torch.uint8, device=cuda)
    capi.call("mxb_per_token_group_quant_fp4", bd.data_ptr(), 64, 512, 640, q.data_ptr(),
              s.data_ptr(), 32, 1e-10, -6.0, 6.0, 0, H.stream())
    rq, rs = orc.quant_rows(_bits(x))
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")


def test_quant_rows_deterministic(cuda):
    x = syn.config2(512, 2048, seed=9).to(cuda)
    a = H.quant_rows(x)
    b = H.quant_rows(x)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


# ------------------------------------------------------------------ fused row + col
@pytest.mark.parametrize("shape", [(32, 32), (96, 160), (256, 384), (1024, 2048)])
@pytest.mark.parametrize("swz", [False, True])
def test_quant_rowcol(cuda, orc, shape, swz):
    x = syn.config2(*shape, seed=1)
    cr, sr, cc, sc, sw = H.quant_rowcol(x.to(cuda), swz=swz)
    xb = _bits(x)
    rq, rs = orc.quant_rows(xb)
    cq, cs = orc.quant_cols(xb)
    H.assert_bytes_equal(H.np_u8(cr), rq, "row codes")
    H.assert_bytes_equal(H.np_u8(sr), rs, "row scales")
    H.assert_bytes_equal(H.np_u8(cc), cq, "col codes")
    H.assert_bytes_equal(H.np_u8(sc), cs, "col scales")
    if swz:
        H.assert_bytes_equal(H.np_u8(sw), orc.swizzle_scales(rs), "swizzled scales")


def test_quant_rowcol_cols_only_and_specials(cuda, orc):
    sb = special_block_input()                      # [9, 64]
    xb = np.concatenate([sb, sb[::-1], sb, sb[:5]])  # [32, 64]
    xb = np.concatenate([xb, xb], axis=1)            # [32, 128]
    _, _, cc, sc, _ = H.quant_rowcol(to_dev_bf16(xb, cuda), rows=False)
    cq, cs = orc.quant_cols(xb)
    H.assert_bytes_equal(H.np_u8(cc), cq, "col codes")
    H.assert_bytes_equal(H.np_u8(sc), cs, "col scales")
    cr, sr, cc2, sc2, _ = H.quant_rowcol(to_dev_bf16(xb, cuda), eps=1e-3, fmin=-4.0, fmax=4.0)
    rq, rs = orc.quant_rows(xb, 1e-3, -4.0, 4.0)
    cq, cs = orc.quant_cols(xb, 1e-3, -4.0, 4.0)
    H.assert_bytes_equal(H.np_u8(cr), rq, "row codes generic")
    H.assert_bytes_equal(H.np_u8(cc2), cq, "col codes generic")
    H.assert_bytes_equal(H.np_u8(sc2), cs, "col scales generic")


@pytest.mark.slow
def test_quant_rowcol_config2_full(cuda, orc):
    x = syn.config2()
    cr, sr, cc, sc, _ = H.quant_rowcol(x.to(cuda))
    xb = _bits(x)
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(sr), rs, "row scales")
    H.assert_bytes_equal(H.np_u8(cr), rq, "row codes")
    del rq, rs
    cq, cs = orc.quant_cols(xb)
    H.assert_bytes_equal(H.np_u8(sc), cs, "col scales")
    H.assert_bytes_equal(H.np_u8(cc), cq, "col codes")


def test_swizzle_scales(cuda, orc):
    g = torch.Generator().manual_seed(3)
    for M, S in [(1, 1), (130, 7), (256, 256)]:
        s = torch.randint(0, 256, (M, S), generator=g, dtype=torch.uint8)
        from mxfp4_b200 import capi
        out = torch.full(((M + 127) // 128 * 128, (S + 3) // 4 * 4), 7, dtype=torch.uint8,
                         device=cuda)
        sd = s.to(cuda)
        capi.call("mxb_swizzle_scales", sd.data_ptr(), M, S, out.data_ptr(), H.stream())
        H.assert_bytes_equal(H.np_u8(out), orc.swizzle_scales(s.numpy()), f"swizzle {M}x{S}")


# ------------------------------------------------------------------ dequant
def dq_exhaustive_input():
    """Every code byte under every E8M0 byte: row e holds bytes 0..255 twice."""
    codes = np.tile(np.arange(256, dtype=np.uint8), (256, 2))
    scales = np.repeat(np.arange(256, dtype=np.uint8)[:, None], 512 // 16, axis=1)
    return codes, scales


def test_dequant_bf16_exhaustive(cuda, orc):
    c, s = dq_exhaustive_input()
    out = H.dequant_bf16(torch.from_numpy(c).to(cuda), torch.from_numpy(s).to(cuda))
    H.assert_bytes_equal(H.np_u16(out), orc.dequant_bf16(c, s), "bf16")


@pytest.mark.parametrize("shape", [(1, 16), (7, 48), (1024, 4096)])
def test_dequant_bf16_config3(cuda, orc, shape):
    c, s = syn.config3(*shape)
    out = H.dequant_bf16(c.to(cuda), s.to(cuda))
    H.assert_bytes_equal(H.np_u16(out), orc.dequant_bf16(c.numpy(), s.numpy()), "bf16")


def test_roundtrip_config1(cuda, orc):
    x = syn.config1()
    xd = x.to(cuda)
    q, s = H.quant_rows(xd)
    out = H.dequant_bf16(q, s)
    rq, rs = orc.quant_rows(_bits(x))
    H.assert_bytes_equal(H.np_u16(out), orc.dequant_bf16(rq, rs), "round trip")
    # size-independent property: every element is within half an E2M1 step of x
    err = (out.float() - xd.float()).abs()
    scale = torch.pow(2.0, s.float() - 127.0).repeat_interleave(32, dim=1)
    assert bool((err <= scale * 1.0 + 1e-30).all())


def fp8_row_exhaustive_input():
    """All (group max, block exponent) pairs: rows [max, e1, e2, e3] with every nibble."""
    pairs = []
    for mx in range(256):
        es = list(range(mx + 1))
        for i in range(0, len(es), 3):
            trip = es[i:i + 3]
            trip += [trip[-1]] * (3 - len(trip))
            pairs.append([mx] + trip)
    if len(pairs) % 2:  # the reference launcher needs numel % 128 == 0
        pairs.append(pairs[-1])
    scales = np.array(pairs, np.uint8)
    blk = np.array([0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE] * 2, np.uint8)
    codes = np.tile(blk, (len(pairs), 4))
    return codes, scales


def test_mxfp4_to_fp8_rows_exhaustive(cuda, orc):
    c, s = fp8_row_exhaustive_input()
    q, so = H.to_fp8_rows(torch.from_numpy(c).to(cuda), torch.from_numpy(s).to(cuda))
    rq, rso = orc.mxfp4_to_fp8_rows(c, s)
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")


@pytest.mark.parametrize("name", ["mxb_per_token_Mxfp4ToFp8", "mxb_per_token_Mxfp4ToBf16ToFp8"])
@pytest.mark.parametrize("shape", [(3, 64), (512, 2048)])
def test_mxfp4_to_fp8_rows_config3(cuda, orc, name, shape):
    c, s = syn.config3(*shape)
    q, so = H.to_fp8_rows(c.to(cuda), s.to(cuda), name)
    rq, rso = orc.mxfp4_to_fp8_rows(c.numpy(), s.numpy())
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")


@pytest.mark.parametrize("shape,lo,hi", [((128, 128), 0, 255), ((256, 256), 110, 140),
                                         ((1024, 1024), 117, 137)])
def test_mxfp4_to_fp8_cols(cuda, orc, shape, lo, hi):
    c, s = syn.config3(*shape, seed=11, lo=lo, hi=hi)
    q, so = H.to_fp8_cols(c.to(cuda), s.to(cuda))
    rq, rso = orc.mxfp4_to_fp8_cols(c.numpy(), s.numpy())
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")


@pytest.mark.parametrize("shape,lo,hi", [((1, 16), 117, 137), ((300, 208), 100, 150),
                                         ((128, 128), 0, 255), ((1024, 1024), 117, 137)])
def test_mxfp4_to_fp8_colT(cuda, orc, shape, lo, hi):
    c, s = syn.config3(*shape, seed=12, lo=lo, hi=hi)
    q, so = H.to_fp8_colT(c.to(cuda), s.to(cuda))
    rq, rso = orc.mxfp4_to_fp8_colT(c.numpy(), s.numpy())
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")


@pytest.mark.parametrize("splits,code_bytes", [([128], 80), ([5, 128, 200, 0, 77], 80),
                                               ([1, 1, 1], 80), ([300, 129], 80),
                                               ([1000, 3, 517, 256, 130], 256),
                                               ([250, 127, 383, 120, 1], 96)])
@pytest.mark.parametrize("lo,hi", [(117, 137), (0, 255)])
def test_mxfp4_to_fp8_colT_split(cuda, orc, splits, code_bytes, lo, hi):
    M = sum(splits)
    c, s = syn.config3(M, code_bytes, seed=13, lo=lo, hi=hi)
    q, so = H.to_fp8_colT_split(c.to(cuda), s.to(cuda), splits)
    rq, rso = orc.mxfp4_to_fp8_colT_split(c.numpy(), s.numpy(), splits)
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")


# ------------------------------------------------------------------ per-token FP8
@pytest.mark.parametrize("shape", [(1, 8), (33, 7168), (64, 20480), (512, 7168)])
def test_fp8_token_quant_dequant(cuda, orc, shape):
    x = syn.config4(*shape)
    xb = _bits(x)
    if shape[0] > 3:
        xb[1, 5] = 0x7FC0      # NaN
        xb[2, 9] = 0x7F80      # Inf
        xb[3, :] = 0           # all-zero row
    xd = to_dev_bf16(xb, cuda)
    q, s = H.quant_fp8(xd)
    rq, rs = orc.fp8_quant_rows(xb)
    H.assert_bytes_equal(H.np_f32(s).view(np.uint32), rs.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")
    out = H.dequant_fp8(q, s)
    H.assert_bytes_equal(H.np_u16(out), orc.fp8_dequant_rows(rq, rs), "dequant")


def test_fp8_dequant_all_codes(cuda, orc):
    q = np.tile(np.arange(256, dtype=np.uint8), (4, 1))
    s = np.array([1.0, 3.5e-3, 1e30, 0.0], np.float32)
    out = H.dequant_fp8(torch.from_numpy(q).view(torch.float8_e4m3fn).to(cuda),
                        torch.from_numpy(s).to(cuda))
    H.assert_bytes_equal(H.np_u16(out), orc.fp8_dequant_rows(q, s), "dequant")


def test_no_pipeline_wait_gave_up(cuda):
    """Every mbarrier wait of the kernels above (quantizers, column and split
    converters) finished in time: the library-wide counter is still zero."""
    torch.cuda.synchronize()
    assert capi.wait_timeouts() == 0
