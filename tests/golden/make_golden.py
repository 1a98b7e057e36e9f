"""Generate the golden fixtures by running the REFERENCE's own kernels.

The reference ships no tests or expected outputs, so its kernels themselves
are the source of truth: this script runs code/kernel/*.cu of the reference,
compiled unmodified for sm_100a by oracle/build_ref.py (module `omo_ref`), on
seeded inputs on a B200 and stores their outputs in ref_outputs.npz.  The
inputs are not stored: they are regenerated from the same seeds by the tests
(tests/test_golden_cpu.py) through tests/test_parity_gpu.py's builders and
mxfp4_b200.synthetic.

Usage (on a GPU machine, after `python oracle/build_ref.py` on a machine that
has the reference sources):
    python tests/golden/make_golden.py [OUT.npz]
"""
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (ROOT, ROOT / "mxfp4-hopper_b200", ROOT / "tests", ROOT / "oracle" / "_ref"):
    sys.path.insert(0, str(p))

import omo_ref  # noqa: E402

from mxfp4_b200 import synthetic as syn  # noqa: E402
from test_parity_gpu import (dq_exhaustive_input, encode_kat_input, fp8_row_exhaustive_input,  # noqa: E402
                             scale_kat_input, special_block_input)

dev = torch.device("cuda:0")


def u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def quant(x):
    M, K = x.shape
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=dev)
    s = torch.empty(M, K // 32, dtype=torch.uint8, device=dev)
    omo_ref.omo_per_token_group_quant_fp4(x, q, s, 32, 1e-10, -6.0, 6.0, False)
    return u8(q), u8(s)


def dq_bf16(c, s):
    M, Kb = c.shape
    out = torch.empty(M, 2 * Kb, dtype=torch.bfloat16, device=dev)
    dummy = torch.empty(M, 2 * Kb // 128, dtype=torch.float32, device=dev)
    omo_ref.omo_per_token_Mxfp4ToBf16_dequant(torch.as_tensor(c).to(dev), torch.as_tensor(s).to(dev),
                                              out, dummy, 32, 1e-10, -6.0, 6.0, False)
    return u8(out)


def fp8_rows(c, s):
    M, Kb = c.shape
    q = torch.empty(M, 2 * Kb, dtype=torch.float8_e4m3fn, device=dev)
    so = torch.empty(Kb // 64, M, dtype=torch.float32, device=dev)
    omo_ref.omo_per_token_Mxfp4ToFp8(torch.as_tensor(c).to(dev), torch.as_tensor(s).to(dev), q, so,
                                     128, 1e-10, -6.0, 6.0, False)
    return u8(q), u8(so)


def fp8_cols(c, s):
    M, Kb = c.shape
    q = torch.empty(2 * Kb, M, dtype=torch.float8_e4m3fn, device=dev)
    so = torch.empty(M // 128, 2 * Kb, dtype=torch.float32, device=dev)
    omo_ref.omo_per_token_Mxfp4ToFp8_col(torch.as_tensor(c).to(dev), torch.as_tensor(s).to(dev), q,
                                         so, 128, 1e-10, -6.0, 6.0, False)
    return u8(q), u8(so)


def fp8_colT(c, s):
    """The reference kernel lacks a barrier (per_token_Mxfp4RowToBf16ToFp8Col.cu:126-131)
    and its output varies from run to run; eight runs are kept and the bytes
    on which all of them agree form the stability masks stored beside run 0."""
    M, Kb = c.shape
    N = 2 * Kb
    runs = []
    for _ in range(8):
        q = torch.empty(N, M, dtype=torch.float8_e4m3fn, device=dev)
        so = torch.empty((M + 127) // 128, N, dtype=torch.float32, device=dev)
        omo_ref.omo_per_token_Mxfp4RowToBf16ToFp8Col(torch.as_tensor(c).to(dev),
                                                    torch.as_tensor(s).to(dev), q, so, 1e-10)
        runs.append((u8(q), u8(so)))
    mq = np.logical_and.reduce([r[0] == runs[0][0] for r in runs])
    ms = np.logical_and.reduce([r[1] == runs[0][1] for r in runs])
    return runs[0][0], runs[0][1], mq, ms


def fp8_colT_split(c, s, splits):
    M, Kb = c.shape
    N = 2 * Kb
    so, sco, acc, accs = [], [], 0, 0
    for m in splits:
        so.append(acc); sco.append(accs)
        acc += m; accs += (m + 127) // 128
    t = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731
    q = torch.empty(N * M, dtype=torch.float8_e4m3fn, device=dev)
    sc = torch.empty(accs, N, dtype=torch.float32, device=dev)
    omo_ref.omo_per_token_Mxfp4RowToBf16ToFp8Col_msplit(
        torch.as_tensor(c).to(dev), torch.as_tensor(s).to(dev), q, sc, t(splits), t(so), t(sco),
        max(splits), 1e-10)
    return u8(q), u8(sc)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(out_path):
    g = {}
    g["q_scale_kat_codes"], g["q_scale_kat_scales"] = quant(bf16(scale_kat_input()))
    g["q_encode_kat_codes"], g["q_encode_kat_scales"] = quant(bf16(encode_kat_input()))
    g["q_special_codes"], g["q_special_scales"] = quant(bf16(special_block_input()[:8]))
    g["q_config1s_codes"], g["q_config1s_scales"] = quant(syn.config1(256, 4096).to(dev))
    # full config 1: hashes of codes, scales and the round trip
    qc, qs = quant(syn.config1().to(dev))
    rt = dq_bf16(qc, qs)
    g["config1_sha256"] = np.array([sha(qc), sha(qs), sha(rt)])
    c, s = dq_exhaustive_input()
    g["dq_bf16_exhaustive"] = dq_bf16(c, s)
    c, s = fp8_row_exhaustive_input()
    g["fp8_rows_exhaustive_q"], g["fp8_rows_exhaustive_s"] = fp8_rows(c, s)
    c, s = syn.config3(256, 256, seed=21, lo=0, hi=255)
    g["fp8_cols_q"], g["fp8_cols_s"] = fp8_cols(c.numpy(), s.numpy())
    c, s = syn.config3(256, 128, seed=22, lo=117, hi=137)
    g["fp8_colT_q"], g["fp8_colT_s"], g["fp8_colT_q_stable"], g["fp8_colT_s_stable"] = \
        fp8_colT(c.numpy(), s.numpy())
    c, s = syn.config3(410, 80, seed=23, lo=100, hi=150)
    g["fp8_colT_split_q"], g["fp8_colT_split_s"] = fp8_colT_split(c.numpy(), s.numpy(),
                                                                  [5, 128, 200, 0, 77])
    g["device"] = np.array([torch.cuda.get_device_name(0)])
    np.savez_compressed(out_path, **g)
    print("wrote", out_path, {k: v.shape for k, v in g.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "ref_outputs.npz"))
