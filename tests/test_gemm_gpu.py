"""Block-scaled MXFP4 GEMM on the tcgen05 tensor cores (next row 3 of the path): the
operands are this library's own rowwise quantize outputs with swizzled scales; the
reference is the exact product of the dequantized operands (float64) rounded to BF16."""
import numpy as np
import pytest
import torch

import helpers as H
from mxfp4_b200 import capi
from mxfp4_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6])


def dequant_np(codes, scales):
    """codes [R, K/2], scales [R, K/32] -> float64 [R, K] (element 2i = low nibble)."""
    lo, hi = codes & 0xF, codes >> 4
    v = np.empty((codes.shape[0], codes.shape[1] * 2))
    v[:, 0::2], v[:, 1::2] = E2M1[lo], E2M1[hi]
    f = np.ldexp(1.0, scales.astype(np.int64) - 127)
    return v * np.repeat(f, 32, axis=1)


def quantize(x, cuda):
    q, s = H.quant_rows(x.to(cuda))
    R, S = s.shape
    swz = torch.empty((R + 127) // 128 * 128, (S + 3) // 4 * 4, dtype=torch.uint8, device=cuda)
    capi.call("mxb_swizzle_scales", s.data_ptr(), R, S, swz.data_ptr(), H.stream())
    return q, s, swz


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (256, 512, 1024), (512, 256, 7168), (384, 768, 2048)])
def test_gemm_mxfp4(cuda, M, N, K):
    a = syn.config2(M, K, seed=41)
    b = syn.config2(N, K, seed=42)
    qa, sa, sza = quantize(a, cuda)
    qb, sb, szb = quantize(b, cuda)
    c = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    capi.call("mxb_gemm_mxfp4", qa.data_ptr(), sza.data_ptr(), qb.data_ptr(), szb.data_ptr(),
              M, N, K, c.data_ptr(), H.stream())
    torch.cuda.synchronize()
    assert capi.load().mxb_gemm_wait_timeouts() == 0
    da, db = dequant_np(H.np_u8(qa), H.np_u8(sa)), dequant_np(H.np_u8(qb), H.np_u8(sb))
    ref = da @ db.T
    absprod = np.abs(da) @ np.abs(db).T
    got = c.float().cpu().numpy().astype(np.float64)
    # per element: one BF16 rounding of the result (half an ulp, 2^-9 relative,
    # bounded here by 2^-8) plus the f32 accumulation's rounding, bounded by
    # 2^-18 of the sum of |a_k * b_k| (K / 64 partial sums of 64-element MMAs
    # at 2^-24 each, with margin); a wrong scale byte moves an element by a
    # factor of two and fails this unless its products cancel to ~2^-18
    bound = 2.0 ** -8 * np.abs(ref) + 2.0 ** -18 * absprod
    err = np.abs(got - ref)
    worst = (err / np.maximum(bound, 1e-300)).max()
    assert (err <= bound).all(), f"worst error / bound = {worst:.3f}"
