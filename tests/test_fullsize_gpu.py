"""Every kernel at its exact BASELINE shape, byte for byte against the oracle
(OpenMP over the host's cores).  The benchmark times these shapes; these
tests check the bytes the timed launches write, including the 64-bit index
arithmetic of the grid-stride and persistent tile walks that only full sizes
reach.  Config 2: BF16 [16384, 8192]; config 3: codes [16384, 8192] with
scales [16384, 512] (K = 16384 elements); config 4: BF16 [32768, 7168]."""
import numpy as np
import pytest
import torch

import helpers as H
from mxfp4_b200 import capi
from mxfp4_b200 import synthetic as syn

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(scope="module")
def config3(cuda):
    c, s = syn.config3()
    return c.numpy(), s.numpy(), c.to(cuda), s.to(cuda)


@pytest.fixture(scope="module")
def config2(cuda):
    x = syn.config2()
    return syn.bf16_bits(x), x.to(cuda)


# ------------------------------------------------------------ config 3
def test_dequant_bf16_config3(orc, config3):
    c, s, cd, sd = config3
    out = H.dequant_bf16(cd, sd)
    H.assert_bytes_equal(H.np_u16(out), orc.dequant_bf16(c, s), "bf16")


def test_fp8_rows_config3(orc, config3):
    c, s, cd, sd = config3
    q, so = H.to_fp8_rows(cd, sd)
    rq, rso = orc.mxfp4_to_fp8_rows(c, s)
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")


def test_fp8_rowscale_config3(orc, config3):
    c, s, cd, sd = config3
    q, so = H.to_fp8_rowscale(cd, sd)
    rq, rso = orc.mxfp4_to_fp8_rowscale(c, s)
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")


def test_fp8_col_config3(orc, config3):
    c, s, cd, sd = config3
    q, so = H.to_fp8_cols(cd, sd)
    rq, rso = orc.mxfp4_to_fp8_cols(c, s)
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")


def test_fp8_colT_config3(orc, config3):
    c, s, cd, sd = config3
    q, so = H.to_fp8_colT(cd, sd)
    rq, rso = orc.mxfp4_to_fp8_colT(c, s)
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")


@pytest.mark.parametrize("multiple", [1, 128])
def test_fp8_colT_split8_config3(orc, config3, multiple):
    """The bench's 8-segment split: ragged sizes, then multiples of 128."""
    c, s, cd, sd = config3
    splits = syn.config3_splits(c.shape[0], 8, multiple)
    q, so = H.to_fp8_colT_split(cd, sd, splits)
    rq, rso = orc.mxfp4_to_fp8_colT_split(c, s, splits)
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), rso.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")


# ------------------------------------------------------------ config 2
def test_quant_rows_config2(orc, config2):
    xb, xd = config2
    q, s = H.quant_rows(xd)
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")


def test_quant_fused_fp8_config2(orc, config2):
    xb, xd = config2
    q, s, f, fs = H.quant_fused_fp8(xd)
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    rf, rfs = orc.mxfp4_to_fp8_rows(rq, rs)
    H.assert_bytes_equal(H.np_f32(fs).view(np.uint32), rfs.view(np.uint32), "fp8 scales")
    H.assert_bytes_equal(H.np_u8(f), rf, "fp8")


def test_swiglu_quant_config2(orc, config2):
    """Config 2's tensor as Megatron's [M, 2H] SwiGLU input: codes and scales
    bit-exact; the activation within one BF16 ulp of torch's float32 SwiGLU."""
    xb, xd = config2
    y, q, s = H.swiglu_quant(xd)
    rq, rs = orc.quant_rows(xb)
    H.assert_bytes_equal(H.np_u8(q), rq, "codes")
    H.assert_bytes_equal(H.np_u8(s), rs, "scales")
    Hh = xd.shape[1] // 2
    g, u = xd[:, :Hh].float(), xd[:, Hh:].float()
    ref = (torch.nn.functional.silu(g) * u).to(torch.bfloat16)
    def ordered(t):  # BF16 patterns -> integers in value order (+0 and -0 both 0)
        b = t.view(torch.int16).to(torch.int32) & 0xFFFF
        mag = b & 0x7FFF
        return torch.where(b >= 0x8000, -mag, mag)
    assert int((ordered(y) - ordered(ref)).abs().max()) <= 1


# ------------------------------------------------------------ config 4
def test_fp8_token_config4(cuda, orc):
    x = syn.config4()
    xb = syn.bf16_bits(x)
    q, s = H.quant_fp8(x.to(cuda))
    rq, rs = orc.fp8_quant_rows(xb)
    H.assert_bytes_equal(H.np_f32(s).view(np.uint32), rs.view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), rq, "fp8")
    out = H.dequant_fp8(q, s)
    H.assert_bytes_equal(H.np_u16(out), orc.fp8_dequant_rows(rq, rs), "dequant")


def test_no_wait_gave_up_at_full_size():
    torch.cuda.synchronize()
    assert capi.wait_timeouts() == 0
