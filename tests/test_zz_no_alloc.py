"""The allocation-free split converter (mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit_noalloc):
its offsets live in a static device array instead of caller-allocated tensors.  Collected
last (file name) so that it also runs after every other test has used the library; each test
also passes alone."""
import ctypes

import numpy as np
import pytest
import torch

import helpers as H
from mxfp4_b200 import capi
from mxfp4_b200 import synthetic as syn

NAME = "mxb_per_token_Mxfp4RowToBf16ToFp8Col_msplit_noalloc"
MAX_SEGMENTS = 4096  # MXB_MSPLIT_MAX_SEGMENTS in include/mxfp4_b200.h


def _noalloc(codes, scales, m_splits, max_len):
    M, Kb = codes.shape
    N = 2 * Kb
    accs = sum((m + 127) // 128 for m in m_splits)
    dev = codes.device
    ms = torch.tensor(m_splits, dtype=torch.int32, device=dev)
    q = torch.full((N * M,), 0x55, dtype=torch.uint8, device=dev)
    s = torch.full((max(accs, 1), N), -1.0, dtype=torch.float32, device=dev)
    capi.call(NAME, H.dp(codes), H.dp(scales), M, N, H.dp(q), H.dp(s), H.dp(ms), len(m_splits),
              max_len, 1e-10, H.stream())
    return q, s[:accs]


def test_noalloc_rejects_too_many_segments():
    """Checked before any CUDA call, so it runs without a GPU."""
    L = capi.load()
    st = capi.status_of(NAME, None, None, 128, 64, None, None, None, MAX_SEGMENTS + 1, 128,
                        1e-10, None)
    assert st == 1  # MXB_ERR_INVALID_ARGUMENT
    assert b"exceeds" in L.mxb_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("splits,code_bytes", [([5, 128, 200, 0, 77], 80),
                                               ([1000, 3, 517, 256, 130], 256)])
def test_noalloc_matches_msplit_twice(cuda, splits, code_bytes):
    """Two calls in a row (the second reuses the static scratch) each equal the
    entry point that takes caller-allocated offsets."""
    M = sum(splits)
    c, s = syn.config3(M, code_bytes, seed=31, lo=110, hi=140)
    c, s = c.to(cuda), s.to(cuda)
    rq, rs = H.to_fp8_colT_split(c, s, splits)
    for max_len in (max(splits), M):  # tight bound, then the always-safe bound
        q, sc = _noalloc(c, s, splits, max_len)
        torch.cuda.synchronize()
        H.assert_bytes_equal(H.np_u8(q), H.np_u8(rq), "fp8")
        H.assert_bytes_equal(H.np_f32(sc).view(np.uint32), H.np_f32(rs).view(np.uint32), "scales")


@pytest.mark.gpu
def test_noalloc_many_segments(cuda):
    """The scan's full width: MXB_MSPLIT_MAX_SEGMENTS segments, most of them empty."""
    rng = np.random.default_rng(5)
    splits = [0] * MAX_SEGMENTS
    for i in rng.choice(MAX_SEGMENTS, 40, replace=False):
        splits[i] = int(rng.integers(1, 300))
    M = sum(splits)
    c, s = syn.config3(M, 64, seed=32, lo=115, hi=135)
    c, s = c.to(cuda), s.to(cuda)
    rq, rs = H.to_fp8_colT_split(c, s, splits)
    q, sc = _noalloc(c, s, splits, max(splits))
    torch.cuda.synchronize()
    H.assert_bytes_equal(H.np_u8(q), H.np_u8(rq), "fp8")
    H.assert_bytes_equal(H.np_f32(sc).view(np.uint32), H.np_f32(rs).view(np.uint32), "scales")
