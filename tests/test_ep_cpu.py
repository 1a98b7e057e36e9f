"""Expert-parallel dispatch / combine: routing tables and the full protocol on
CPU ranks (gloo, world size 2), with the oracle standing in for the CUDA data
kernels.  The CUDA kernels themselves are checked in test_ep_gpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mxfp4_b200 import synthetic as syn
from mxfp4_b200.ep import build_route, unpack_rowwise, wire_row_bytes


def test_wire_row_bytes_and_split():
    assert wire_row_bytes(7168) == 3808
    packed = torch.zeros(3, 3808, dtype=torch.uint8)
    c, s = unpack_rowwise(packed)
    assert c.shape == (3, 3584) and s.shape == (3, 224)
    with pytest.raises(ValueError):
        unpack_rowwise(torch.zeros(2, 100, dtype=torch.uint8))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_route_tables(world):
    _, idx, w = syn.config5(0, world, tokens=256, hidden=128, experts=64, topk=8)
    r = build_route(idx, w, world, 64)
    per = 64 // world
    dest = (idx // per).numpy()
    sl = r.slots.numpy()
    S = int(r.send_counts.sum())
    assert sorted(sl[sl >= 0].tolist()) == list(range(S))           # every row used once
    for t in range(256):
        assert set(np.nonzero(sl[t] >= 0)[0]) == set(dest[t])     # sent exactly to its ranks
    offs = np.concatenate([[0], np.cumsum(r.send_counts.numpy())[:-1]])
    for g in range(world):                                          # grouped by rank, token order
        rows = sl[sl[:, g] >= 0, g]
        assert np.array_equal(rows, np.arange(offs[g], offs[g] + len(rows)))
    st = r.src_token.numpy()
    for s_ in range(S):
        t = st[s_]
        g = np.nonzero(sl[t] == s_)[0][0]
        lt, lw = r.local_topk[s_].numpy(), r.local_w[s_].numpy()
        for j in range(8):
            if dest[t, j] == g:
                assert lt[j] == idx[t, j] - g * per and lw[j] == w[t, j]
            else:
                assert lt[j] == -1 and lw[j] == 0
    # config 5 at 8 ranks: ~5.29 distinct destination ranks per token
    _, idx8, w8 = syn.config5(0, 8, tokens=4096, hidden=128)
    r8 = build_route(idx8, w8, 8, 256)
    assert 5.0 < r8.send_counts.sum().item() / 4096 < 5.6


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, H, E, k, q):
    try:
        import sys
        from pathlib import Path
        root = Path(__file__).resolve().parent.parent
        for p in (root, root / "mxfp4-hopper_b200", root / "tests"):
            sys.path.insert(0, str(p))
        from ep_oracle import OracleKernels, expected_round, pack_rows
        from mxfp4_b200 import synthetic as syn
        from mxfp4_b200.ep import MXFP4Dispatcher

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        x, idx, w = syn.config5(rank, world, tokens=T, hidden=H, experts=E, topk=k)
        d = MXFP4Dispatcher(None, num_experts=E, hidden=H, kernels=OracleKernels())
        recv_wire, recv_topk, recv_w, h = d.dispatch(x, idx, w)
        # received rows must be the senders' oracle-quantized tokens, in rank order
        per = E // world
        exp_rows = []
        for src in range(world):
            xs, ids, _ = syn.config5(src, world, tokens=T, hidden=H, experts=E, topk=k)
            rows = pack_rows(xs)
            sel = ((ids // per) == rank).any(1).numpy()
            exp_rows.append(rows[sel])
        ok_rows = np.array_equal(recv_wire.numpy(), np.concatenate(exp_rows))
        ok_topk = bool(((recv_topk >= -1) & (recv_topk < per)).all())
        y = d.identity_experts(recv_wire, recv_w)
        out = d.combine(y, h)
        exp = expected_round(x, idx, w, world, E)
        ok_out = np.array_equal(out.view(torch.int16).numpy().view(np.uint16), exp)
        q.put((rank, ok_rows, ok_topk, ok_out))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), False, False))


@pytest.mark.parametrize("world", [2])
def test_dispatch_combine_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 48, 256, 16, 4, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok_rows, ok_topk, ok_out in sorted(res):
        assert ok_rows is True, f"rank {rank}: received rows differ ({ok_rows})"
        assert ok_topk and ok_out, f"rank {rank}: topk {ok_topk} out {ok_out}"
