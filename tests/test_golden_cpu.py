"""Pins the CPU oracle to the reference itself.

tests/golden/ref_outputs.npz holds outputs of the reference's own kernels
(code/kernel/*.cu compiled unmodified for sm_100a) run on a B200 by
tests/golden/make_golden.py.  Inputs are regenerated here from the same seeds
and builders; the oracle must reproduce the stored bytes exactly.
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from mxfp4_b200 import synthetic as syn
from test_parity_gpu import (dq_exhaustive_input, encode_kat_input, fp8_row_exhaustive_input,
                             scale_kat_input, special_block_input)

GOLD = Path(__file__).resolve().parent / "golden" / "ref_outputs.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def _u8(a):
    return np.ascontiguousarray(a).view(np.uint8)


@pytest.mark.parametrize("name,builder", [
    ("q_scale_kat", scale_kat_input), ("q_encode_kat", encode_kat_input),
    ("q_special", lambda: special_block_input()[:8]),
    ("q_config1s", lambda: syn.bf16_bits(syn.config1(256, 4096)))])
def test_quant_rows_vs_reference(orc, gold, name, builder):
    x = builder()
    q, s = orc.quant_rows(x)
    assert np.array_equal(q, gold[name + "_codes"])
    assert np.array_equal(s, gold[name + "_scales"])


def test_config1_full_hashes(orc, gold):
    """[4096, 4096] seed 0 round trip, by SHA-256."""
    q, s = orc.quant_rows(syn.bf16_bits(syn.config1()))
    rt = orc.dequant_bf16(q, s)
    got = [hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest() for a in (q, s, rt)]
    assert got == list(gold["config1_sha256"])


def test_dequant_bf16_vs_reference(orc, gold):
    c, s = dq_exhaustive_input()
    assert np.array_equal(_u8(orc.dequant_bf16(c, s)), gold["dq_bf16_exhaustive"])


def test_fp8_rows_vs_reference(orc, gold):
    c, s = fp8_row_exhaustive_input()
    q, so = orc.mxfp4_to_fp8_rows(c, s)
    assert np.array_equal(q, gold["fp8_rows_exhaustive_q"])
    assert np.array_equal(_u8(so).reshape(1, -1), gold["fp8_rows_exhaustive_s"])


def test_fp8_cols_vs_reference(orc, gold):
    c, s = syn.config3(256, 256, seed=21, lo=0, hi=255)
    q, so = orc.mxfp4_to_fp8_cols(c.numpy(), s.numpy())
    assert np.array_equal(q, gold["fp8_cols_q"])
    assert np.array_equal(_u8(so).reshape(so.shape[0], -1), gold["fp8_cols_s"])


def test_fp8_colT_vs_reference_where_stable(orc, gold):
    """The reference's RowToBf16ToFp8Col kernel races (missing barrier); the
    oracle restates the race-free semantics and must agree on every byte that
    was identical across the reference's repeated runs."""
    if "fp8_colT_q_stable" not in gold:
        pytest.skip("fixture predates the stability masks")
    c, s = syn.config3(256, 128, seed=22, lo=117, hi=137)
    q, so = orc.mxfp4_to_fp8_colT(c.numpy(), s.numpy())
    mq, ms = gold["fp8_colT_q_stable"], gold["fp8_colT_s_stable"]
    # 96.7% of the FP8 bytes and 95.7% of the scales were identical over the
    # reference's 8 runs when the fixture was made
    assert mq.mean() > 0.95 and ms.mean() > 0.94
    assert np.array_equal(q[mq], gold["fp8_colT_q"][mq])
    so8 = _u8(so).reshape(so.shape[0], -1)
    assert np.array_equal(so8[ms], gold["fp8_colT_s"][ms])


def test_fp8_colT_split_vs_reference(orc, gold):
    c, s = syn.config3(410, 80, seed=23, lo=100, hi=150)
    q, so = orc.mxfp4_to_fp8_colT_split(c.numpy(), s.numpy(), [5, 128, 200, 0, 77])
    assert np.array_equal(q, gold["fp8_colT_split_q"])
    assert np.array_equal(_u8(so).reshape(so.shape[0], -1), gold["fp8_colT_split_s"])
