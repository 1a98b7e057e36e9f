"""Expert-parallel data kernels on the GPU (through the C ABI) against the
oracle, and the full NCCL dispatch -> identity experts -> combine round on
2+ GPUs (one process per GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from ep_oracle import combine_rows, expected_round, pack_rows, unpack_rows
from mxfp4_b200 import capi
from mxfp4_b200 import synthetic as syn
from mxfp4_b200.ep import CudaKernels, build_route, weight_sums

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,T,H", [(1, 7, 128), (4, 200, 512), (8, 512, 7168)])
def test_pack_unpack_combine_kernels(cuda, world, T, H):
    x, idx, w = syn.config5(0, world, tokens=T, hidden=H)
    if T > 100:  # a few blocks with Inf / NaN / zeros
        xb = syn.bf16_bits(x).copy()
        xb[3, 5], xb[4, 70], xb[5, :] = 0x7F80, 0xFFC1, 0
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
    r = build_route(idx, w, world, 256)
    S = int(r.send_counts.sum())
    K = CudaKernels()
    wire = K.pack(x.to(cuda), r.slots.to(cuda), S)
    rows = pack_rows(x)
    assert np.array_equal(wire.cpu().numpy(), rows[r.src_token.numpy()])
    wsum = weight_sums(r.local_w)
    y = K.unpack(wire, H, wsum.to(cuda))
    y_ref = unpack_rows(wire.cpu().numpy(), H, wsum.numpy())
    assert np.array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), y_ref)
    y0 = K.unpack(wire, H, None)
    assert np.array_equal(y0.cpu().view(torch.int16).numpy().view(np.uint16),
                          unpack_rows(wire.cpu().numpy(), H))
    out = K.combine(y, r.slots.to(cuda))
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16),
                          combine_rows(y_ref, r.slots.numpy()))


@pytest.mark.parametrize("world,T", [(1, 5), (2, 1), (2, 4096), (8, 4096), (8, 3000), (64, 2500),
                                     (64, 51200), (64, 65792)])
def test_route_kernel(cuda, world, T):
    from mxfp4_b200 import capi
    from mxfp4_b200.ep import local_route
    _, idx, _ = syn.config5(3, world, tokens=T, hidden=128)
    idx = idx.to(cuda).contiguous()
    within = torch.empty(T, world, dtype=torch.int32, device=cuda)
    counts = torch.empty(world, dtype=torch.int32, device=cuda)
    capi.call("mxb_ep_route", idx.data_ptr(), T, 8, 256 // world, world, within.data_ptr(),
              counts.data_ptr(), torch.cuda.current_stream().cuda_stream)
    w_ref, c_ref, _ = local_route(idx, world, 256)
    assert torch.equal(within, w_ref) and torch.equal(counts, c_ref)


@pytest.mark.parametrize("world,T,topk,experts", [(4, 2100, 3, 64), (3, 1025, 1, 9),
                                                  (16, 700, 13, 160)])
def test_route_kernel_odd_topk(cuda, world, T, topk, experts):
    """Top-k widths that do not divide the tile, repeated experts of one rank."""
    from mxfp4_b200 import capi
    from mxfp4_b200.ep import local_route
    g = torch.Generator().manual_seed(world * 1000 + topk)
    idx = torch.randint(0, experts, (T, topk), generator=g, dtype=torch.int64).to(cuda)
    within = torch.empty(T, world, dtype=torch.int32, device=cuda)
    counts = torch.empty(world, dtype=torch.int32, device=cuda)
    capi.call("mxb_ep_route", idx.data_ptr(), T, topk, experts // world, world,
              within.data_ptr(), counts.data_ptr(), torch.cuda.current_stream().cuda_stream)
    w_ref, c_ref, _ = local_route(idx, world, experts)
    assert torch.equal(within, w_ref) and torch.equal(counts, c_ref)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        import sys
        from pathlib import Path
        root = Path(__file__).resolve().parent.parent
        for p in (root, root / "mxfp4-hopper_b200", root / "tests"):
            sys.path.insert(0, str(p))
        import torch.distributed as dist
        from ep_oracle import expected_round
        from mxfp4_b200 import synthetic as syn
        from mxfp4_b200.ep import MXFP4Dispatcher

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, device_id=dev)
        from mxfp4_b200 import capi
        from mxfp4_b200.ep import P2PDispatcher
        x, idx, w = syn.config5(rank, world, tokens=512, hidden=7168)
        exp = expected_round(x, idx, w, world, 256)
        d = MXFP4Dispatcher(None, num_experts=256, hidden=7168)
        recv_wire, recv_topk, recv_w, h = d.dispatch(x.to(dev), idx.to(dev), w.to(dev))
        out = d.combine(d.identity_experts(recv_wire, recv_w), h)
        ok_nccl = np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), exp)
        # the C-ABI dispatcher over an NCCL communicator of its own
        from mxfp4_b200.ep import NcclCDispatcher, weight_sums
        ids = [NcclCDispatcher.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        cd = NcclCDispatcher(world, rank, ids[0], tokens=512, hidden=7168, topk=8,
                             num_experts=256)
        ok_c = True
        for it in range(2):
            xs, ids_, ws = syn.config5(rank + 50 * it, world, tokens=512 - 32 * it, hidden=7168)
            rw, rt, rwt = cd.dispatch(xs.to(dev), ids_.to(dev), ws.to(dev))
            yc = d.k.unpack(rw, 7168, weight_sums(rwt))
            oc = cd.combine(yc)
            ec = expected_round(xs, ids_, ws, world, 256)
            ok_c &= np.array_equal(oc.cpu().view(torch.int16).numpy().view(np.uint16), ec)
            ok_c &= bool(((rt >= -1) & (rt < 256 // world)).all())
        cd.close()
        p2p = P2PDispatcher(None, tcap=512, hidden=7168, topk=8, num_experts=256)
        ok_p2p = True
        for it in range(3):  # several steps: parity and epochs advance
            xs, ids, ws = syn.config5(rank + 100 * it, world, tokens=512 - 64 * it, hidden=7168)
            o2 = p2p.step(xs.to(dev), ids.to(dev), ws.to(dev))
            e2 = expected_round(xs, ids, ws, world, 256)
            ok_p2p &= np.array_equal(o2.cpu().view(torch.int16).numpy().view(np.uint16), e2)
        torch.cuda.synchronize()
        ok_p2p &= capi.load().mxb_ep_wait_timeouts() == 0
        dist.barrier()
        p2p.close()
        q.put((rank, bool(ok_nccl and ok_p2p and ok_c) or f"nccl {ok_nccl} p2p {ok_p2p} c-abi {ok_c}"))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


def test_dispatch_combine_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = min(n, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok in sorted(res):
        assert ok is True, f"rank {rank}: {ok}"


# ------------------------------------------------------------------ moe_permute
def _permute_ref(codes, scales, dst, n_out, fill=0x5A):
    """out[dst[i, k]] = row i (codes and scales), destinations outside [0, n_out) skipped."""
    rows, topk = dst.shape
    oc = np.full((n_out, codes.shape[1]), fill, np.uint8)
    os_ = np.full((n_out, scales.shape[1]), fill, np.uint8)
    for i in range(rows):
        for k in range(topk):
            d = int(dst[i, k])
            if 0 <= d < n_out:
                oc[d] = codes[i]
                os_[d] = scales[i]
    return oc, os_


@pytest.mark.parametrize("rows,H,topk,wire", [(300, 7168, 8, True), (300, 7168, 8, False),
                                               (77, 128, 3, True), (5, 64, 1, False),
                                               (9, 96, 2, True)])
def test_moe_permute_mxfp4(cuda, rows, H, topk, wire):
    g = np.random.default_rng(rows + H + topk)
    codes = g.integers(0, 256, (rows, H // 2), dtype=np.uint8)
    scales = g.integers(100, 150, (rows, H // 32), dtype=np.uint8)
    n_out = rows * topk - (rows * topk) // 8 - 1
    dst = g.permutation(rows * topk).astype(np.int32).reshape(rows, topk)
    dst[dst >= n_out] = -1            # a few routed-nowhere slots
    dst[0, 0] = -1
    oc_ref, os_ref = _permute_ref(codes, scales, dst, n_out)
    if wire:  # EP receive rows: codes || scales, pitch 17H/32
        src = torch.from_numpy(np.concatenate([codes, scales], axis=1)).to(cuda)
        cptr, cp, sptr, sp = src.data_ptr(), 17 * H // 32, src.data_ptr() + H // 2, 17 * H // 32
    else:
        c_d, s_d = torch.from_numpy(codes).to(cuda), torch.from_numpy(scales).to(cuda)
        cptr, cp, sptr, sp = c_d.data_ptr(), H // 2, s_d.data_ptr(), H // 32
    d_d = torch.from_numpy(dst).to(cuda)
    oc = torch.full((n_out, H // 2), 0x5A, dtype=torch.uint8, device=cuda)
    os_ = torch.full((n_out, H // 32), 0x5A, dtype=torch.uint8, device=cuda)
    capi.call("mxb_moe_permute_mxfp4", cptr, cp, sptr, sp, rows, H, d_d.data_ptr(), topk,
              oc.data_ptr(), os_.data_ptr(), n_out, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(oc.cpu().numpy(), oc_ref)
    np.testing.assert_array_equal(os_.cpu().numpy(), os_ref)


# ------------------------------------------------------------------ bounded waits
def test_p2p_wait_gives_up_and_reports(cuda):
    """A cross-GPU wait whose peer never signals gives up after the configured
    number of polls and is counted, leaving the context usable.  The "world" is
    two ranks whose buffers are both this GPU's own buffer: rank 1 never runs,
    so its flag stays 0 and both the count exchange and the barrier run out
    (a short bounded wait on a flag that nothing sets; no peer memory, no fault)."""
    import ctypes
    L = capi.EpLayout()
    total = ctypes.c_int64()
    capi.call("mxb_ep_layout_init", 2, 0, 16, 512, 2, 4, ctypes.byref(L), ctypes.byref(total))
    buf = torch.zeros(total.value, dtype=torch.uint8, device=cuda)
    bases = torch.tensor([buf.data_ptr(), buf.data_ptr()], dtype=torch.int64, device=cuda)
    counts = torch.zeros(2, dtype=torch.int32, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    lib = capi.load()
    torch.cuda.synchronize()
    lib.mxb_ep_reset_wait_timeouts()
    try:
        capi.call("mxb_ep_set_wait_polls", 2000)
        capi.call("mxb_ep_p2p_counts", bases.data_ptr(), ctypes.byref(L), counts.data_ptr(), 0, 1, s)
        capi.call("mxb_ep_p2p_barrier", bases.data_ptr(), ctypes.byref(L), 2, s)
        torch.cuda.synchronize()
        assert lib.mxb_ep_wait_timeouts() == 2
        # the context is still usable and the own flag carries the last epoch
        sig = buf[L.sig_off:L.sig_off + 8].view(torch.int32).cpu().tolist()
        assert sig == [2, 0]
        # a wait that is satisfied does not count: raise the peer's flag by hand
        buf[L.sig_off + 4:L.sig_off + 8].view(torch.int32).fill_(3)
        capi.call("mxb_ep_p2p_barrier", bases.data_ptr(), ctypes.byref(L), 3, s)
        torch.cuda.synchronize()
        assert lib.mxb_ep_wait_timeouts() == 2
    finally:
        capi.call("mxb_ep_set_wait_polls", 0)
        torch.cuda.synchronize()
        lib.mxb_ep_reset_wait_timeouts()
    assert lib.mxb_ep_wait_timeouts() == 0


# ------------------------------------------------------------------ row_id_map permute
def _row_id_map_ref(rmap):
    """Restated Transformer Engine mask-map row_id_map: experts in order, tokens
    in order within an expert; per token its destinations, experts and count."""
    T, E = rmap.shape
    counts = rmap.sum(0)
    offs = np.concatenate([[0], np.cumsum(counts)[:-1]])
    rank = np.cumsum(rmap, 0) - 1
    rid = np.full((T, 2 * E + 1), -1, np.int32)
    for t in range(T):
        ex = np.nonzero(rmap[t])[0]
        n = len(ex)
        rid[t, :n] = offs[ex] + rank[t, ex]
        rid[t, E:E + n] = ex
        rid[t, 2 * E] = n
    return rid


@pytest.mark.parametrize("T,E,k,H,wire", [(4096, 32, 8, 7168, True), (300, 256, 8, 7168, False),
                                          (77, 64, 40, 7168, False), (77, 64, 40, 128, True),
                                          (1, 8, 8, 512, False), (5, 16, 0, 256, False)])
def test_moe_permute_row_id_map(cuda, T, E, k, H, wire):
    """TE's moe_permute on MXFP4 rows from a mask routing map: the row_id_map
    the device builds, and the permuted codes and scales, against a numpy
    restatement; more than 32 destinations per row, empty tokens included."""
    from mxfp4_b200.ep import moe_permute_mxfp4
    g = np.random.default_rng(T + E + k)
    rmap = np.zeros((T, E), bool)
    for t in range(T):
        if k:
            rmap[t, g.choice(E, size=min(k, E), replace=False)] = True
    if T > 3:
        rmap[2] = False                       # a token routed nowhere
    codes = g.integers(0, 256, (T, H // 2), dtype=np.uint8)
    scales = g.integers(100, 150, (T, H // 32), dtype=np.uint8)
    if wire:
        src = torch.from_numpy(np.concatenate([codes, scales], axis=1)).to(cuda)
        c_d, s_d = src[:, :H // 2], src[:, H // 2:]
    else:
        c_d, s_d = torch.from_numpy(codes).to(cuda), torch.from_numpy(scales).to(cuda)
    oc, os_, rid = moe_permute_mxfp4(c_d, s_d, torch.from_numpy(rmap).to(cuda))
    torch.cuda.synchronize()
    rid_ref = _row_id_map_ref(rmap.astype(np.int64))
    np.testing.assert_array_equal(rid.cpu().numpy(), rid_ref)
    n_out = int(rmap.sum())
    order = np.concatenate([np.nonzero(rmap[:, e])[0] for e in range(E)]) if n_out else \
        np.zeros(0, np.int64)
    np.testing.assert_array_equal(oc.cpu().numpy(), codes[order])
    np.testing.assert_array_equal(os_.cpu().numpy(), scales[order])
