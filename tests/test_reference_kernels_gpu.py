"""Byte parity with the reference's own kernels on the same device.

`omo_ref` is the reference's code/kernel/*.cu compiled unmodified for sm_100a
(oracle/build_ref.py).  Each test feeds the same seeded inputs to the
reference launcher and to this library's C ABI and requires identical bytes.
The reference's RowToBf16ToFp8Col kernel has a missing barrier (its column
amax may read shared memory before every warp stored its tile), so that one
is compared against the race-free CPU oracle in test_parity_gpu.py and only
checked here on tiles where the race cannot change the result twice in a row.
"""
import numpy as np
import pytest
import torch

import helpers as H
from mxfp4_b200 import synthetic as syn
from test_parity_gpu import (dq_exhaustive_input, encode_kat_input, fp8_row_exhaustive_input,
                             scale_kat_input, special_block_input)

pytestmark = pytest.mark.gpu


def ref_quant(ref, x):
    M, K = x.shape
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    s = torch.empty(M, K // 32, dtype=torch.uint8, device=x.device)
    ref.omo_per_token_group_quant_fp4(x, q, s, 32, 1e-10, -6.0, 6.0, False)
    return q, s


@pytest.mark.parametrize("kind", ["config1", "scale_kat", "encode_kat", "special", "config2"])
def test_ref_quant_rows(cuda, ref_kernels, kind):
    if kind == "config1":
        x = syn.config1(512, 4096).to(cuda)
    elif kind == "config2":
        x = syn.config2(1024, 8192).to(cuda)
    else:
        bits = {"scale_kat": scale_kat_input, "encode_kat": encode_kat_input,
                "special": lambda: special_block_input()[:8]}[kind]()
        x = H.bf16_from_bits(bits).to(cuda)
    rq, rs = ref_quant(ref_kernels, x)
    q, s = H.quant_rows(x)
    H.assert_bytes_equal(H.np_u8(s), H.np_u8(rs), "scales vs reference kernel")
    H.assert_bytes_equal(H.np_u8(q), H.np_u8(rq), "codes vs reference kernel")


def test_ref_quant_cols_via_transpose(cuda, ref_kernels):
    x = syn.config2(512, 1024).to(cuda)
    rq, rs = ref_quant(ref_kernels, x.t().contiguous())
    _, _, cc, sc, _ = H.quant_rowcol(x, rows=False)
    H.assert_bytes_equal(H.np_u8(sc), H.np_u8(rs), "col scales vs reference")
    H.assert_bytes_equal(H.np_u8(cc), H.np_u8(rq), "col codes vs reference")


def test_ref_dequant_bf16(cuda, ref_kernels):
    c, s = dq_exhaustive_input()
    cd, sd = torch.from_numpy(c).to(cuda), torch.from_numpy(s).to(cuda)
    out_r = torch.empty(c.shape[0], 2 * c.shape[1], dtype=torch.bfloat16, device=cuda)
    dummy = torch.empty(c.shape[0], 2 * c.shape[1] // 128, dtype=torch.float32, device=cuda)
    ref_kernels.omo_per_token_Mxfp4ToBf16_dequant(cd, sd, out_r, dummy, 32, 1e-10, -6.0, 6.0, False)
    out = H.dequant_bf16(cd, sd)
    H.assert_bytes_equal(H.np_u16(out), H.np_u16(out_r), "bf16 vs reference")


def _ref_fp8_rows(ref, cd, sd):
    M, Kb = cd.shape
    q = torch.empty(M, 2 * Kb, dtype=torch.float8_e4m3fn, device=cd.device)
    so = torch.empty(Kb // 64, M, dtype=torch.float32, device=cd.device)
    ref.omo_per_token_Mxfp4ToFp8(cd, sd, q, so, 128, 1e-10, -6.0, 6.0, False)
    return q, so


@pytest.mark.parametrize("kind", ["exhaustive", "config3"])
def test_ref_mxfp4_to_fp8_rows(cuda, ref_kernels, kind):
    if kind == "exhaustive":
        c, s = (torch.from_numpy(a) for a in fp8_row_exhaustive_input())
    else:
        c, s = syn.config3(512, 2048)
    cd, sd = c.to(cuda), s.to(cuda)
    rq, rso = _ref_fp8_rows(ref_kernels, cd, sd)
    q, so = H.to_fp8_rows(cd, sd)
    H.assert_bytes_equal(H.np_u8(q), H.np_u8(rq), "fp8 vs reference")
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), H.np_f32(rso).view(np.uint32), "scales")


@pytest.mark.parametrize("lo,hi", [(0, 255), (117, 137)])
def test_ref_mxfp4_to_fp8_cols(cuda, ref_kernels, lo, hi):
    c, s = syn.config3(256, 256, seed=21, lo=lo, hi=hi)
    cd, sd = c.to(cuda), s.to(cuda)
    M, Kb = c.shape
    rq = torch.empty(2 * Kb, M, dtype=torch.float8_e4m3fn, device=cuda)
    rso = torch.empty(M // 128, 2 * Kb, dtype=torch.float32, device=cuda)
    ref_kernels.omo_per_token_Mxfp4ToFp8_col(cd, sd, rq, rso, 128, 1e-10, -6.0, 6.0, False)
    q, so = H.to_fp8_cols(cd, sd)
    H.assert_bytes_equal(H.np_u8(q), H.np_u8(rq), "fp8 vs reference")
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32), H.np_f32(rso).view(np.uint32), "scales")


@pytest.mark.parametrize("shape,lo,hi", [((256, 128), 117, 137), ((300, 208), 100, 150),
                                          ((1024, 1024), 117, 137)])
def test_ref_mxfp4_to_fp8_colT(cuda, ref_kernels, shape, lo, hi):
    """The reference kernel races (its column amax can read shared memory before
    every warp stored the tile), so it is run several times and this library's
    bytes must equal the reference's on every byte that all runs agree on; most
    bytes are stable (the race hits a few tiles per launch)."""
    c, s = syn.config3(*shape, seed=22, lo=lo, hi=hi)
    cd, sd = c.to(cuda), s.to(cuda)
    M, Kb = c.shape
    N = 2 * Kb
    qs, ss = [], []
    for _ in range(6):
        rq = torch.empty(N, M, dtype=torch.float8_e4m3fn, device=cuda)
        rso = torch.empty((M + 127) // 128, N, dtype=torch.float32, device=cuda)
        ref_kernels.omo_per_token_Mxfp4RowToBf16ToFp8Col(cd, sd, rq, rso, 1e-10)
        qs.append(H.np_u8(rq))
        ss.append(H.np_f32(rso).view(np.uint32))
    mq = np.all([q == qs[0] for q in qs[1:]], axis=0)
    ms = np.all([x == ss[0] for x in ss[1:]], axis=0)
    # how often the reference races varies between boxes: at 256 x 256, 68-82 % of the
    # FP8 bytes and 57-76 % of the scales agreed over 6 runs in the runs measured
    assert mq.mean() > 0.3 and ms.mean() > 0.25, (mq.mean(), ms.mean())
    q, so = H.to_fp8_colT(cd, sd)
    H.assert_bytes_equal(H.np_u8(q)[mq], qs[0][mq], "fp8 vs reference (stable bytes)")
    H.assert_bytes_equal(H.np_f32(so).view(np.uint32)[ms], ss[0][ms],
                         "scales vs reference (stable bytes)")


@pytest.mark.parametrize("splits", [[128], [5, 128, 200, 0, 77]])
def test_ref_mxfp4_to_fp8_colT_split(cuda, ref_kernels, splits):
    M = sum(splits)
    c, s = syn.config3(M, 80, seed=23, lo=100, hi=150)
    cd, sd = c.to(cuda), s.to(cuda)
    N = 160
    so, sco, acc, accs = [], [], 0, 0
    for m in splits:
        so.append(acc); sco.append(accs)
        acc += m; accs += (m + 127) // 128
    t = lambda v: torch.tensor(v, dtype=torch.int32, device=cuda)  # noqa: E731
    rq = torch.empty(N * M, dtype=torch.float8_e4m3fn, device=cuda)
    rso = torch.empty(accs, N, dtype=torch.float32, device=cuda)
    ref_kernels.omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit(cd, sd, rq, rso, t(splits), t(so),
                                                           t(sco), max(splits), 1e-10)
    q, sc = H.to_fp8_colT_split(cd, sd, splits)
    H.assert_bytes_equal(H.np_f32(sc).view(np.uint32), H.np_f32(rso).view(np.uint32), "scales")
    H.assert_bytes_equal(H.np_u8(q), H.np_u8(rq), "fp8 vs reference")
