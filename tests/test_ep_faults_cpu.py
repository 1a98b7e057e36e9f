"""Failure detection of the expert-parallel exchange, on CPU ranks (gloo,
world size 2), with the oracle standing in for the CUDA data kernels.  The
failures are made on the host: a rank that leaves between steps, a rank
that is late past the deadline, and a rank that sends an impossible count
table.  The surviving rank must raise an EPError subclass within the
deadline's order of magnitude instead of blocking."""
import socket
import time

import pytest
import torch.multiprocessing as mp

DEADLINE_S = 3.0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    for p in (root, root / "mxfp4-hopper_b200", root / "tests"):
        sys.path.insert(0, str(p))
    import torch
    import torch.distributed as dist
    from ep_oracle import OracleKernels
    from mxfp4_b200 import synthetic as syn
    from mxfp4_b200.ep import EPError, EPProtocolError, EPTimeout, MXFP4Dispatcher

    T, H, E, k = 32, 256, 16, 4
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=DEADLINE_S))
    d = MXFP4Dispatcher(None, num_experts=E, hidden=H, kernels=OracleKernels(),
                        timeout_s=DEADLINE_S, max_tokens_per_rank=T)
    if mode == "corrupt" and rank == 1:
        d._send_counts = lambda route: route.send_counts * 0 - 5  # noqa: E731
    x, idx, w = syn.config5(rank, world, tokens=T, hidden=H, experts=E, topk=k)
    outcome = "ok"
    t0 = time.monotonic()
    try:
        # step 1: every rank healthy (except a corrupting rank, from the start)
        rw, rt, rwt, h = d.dispatch(x, idx, w)
        d.combine(d.identity_experts(rw, rwt), h)
        if mode == "leave" and rank == 1:
            q.put((rank, "left", 0.0))
            q.close()
            q.join_thread()
            import os
            os._exit(0)  # leaves between steps, with no exchange in flight
        if mode == "late" and rank == 1:
            time.sleep(4 * DEADLINE_S)
        t0 = time.monotonic()
        rw, rt, rwt, h = d.dispatch(x, idx, w)
        d.combine(d.identity_experts(rw, rwt), h)
    except EPProtocolError:
        outcome = "protocol"
    except EPTimeout:
        outcome = "timeout"
    except EPError:
        outcome = "error"
    except Exception as e:  # noqa: BLE001
        outcome = f"unexpected {type(e).__name__}: {e}"
    q.put((rank, outcome, time.monotonic() - t0))
    q.close()
    q.join_thread()
    if outcome != "ok":
        try:
            d.abort()
        except Exception:  # noqa: BLE001
            pass
    import os
    os._exit(0)


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, outcome, dt = q.get(timeout=120)
        res[r] = (outcome, dt)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


def test_healthy_steps_pass():
    res = _run("healthy")
    assert res[0][0] == "ok" and res[1][0] == "ok", res


def test_rank_leaving_between_steps_is_detected():
    res = _run("leave")
    assert res[1][0] == "left"
    assert res[0][0] in ("timeout", "error"), res
    assert res[0][1] < 10 * DEADLINE_S, res


def test_late_rank_hits_the_deadline():
    res = _run("late")
    assert res[0][0] == "timeout", res
    assert res[0][1] < 3 * DEADLINE_S, res


def test_corrupt_count_table_is_rejected():
    res = _run("corrupt")
    assert res[0][0] == "protocol", res
    assert res[1][0] in ("timeout", "error", "protocol"), res
    assert res[1][1] < 10 * DEADLINE_S, res
