"""MoE expert-parallel dispatch / combine with MXFP4 payloads.

Behaviour of the reference path (megatron-0.15.0rc7.diff:290-311 with the
DeepEP 1.2.1 patch): a token is quantized to MXFP4 (`fp4_quantize`, :91-99),
its wire row `codes[H/2] || scales[H/32]` is sent once to every rank that hosts
one of its top-k experts, the receiver splits the row at 16/17 and dequantizes
it (:101-124,303-309), and the BF16 expert outputs come back through a BF16
combine that sums each token's contributions (deep_ep-1.2.1.diff:132-139).

Here the routing tables are built on the device with torch ops, the three data
kernels are this library's (`mxb_ep_pack`, `mxb_ep_unpack`, `mxb_ep_combine`),
and the exchanges are NCCL all-to-all-v collectives through torch.distributed
(one process per GPU).  The token counts are exchanged first and read on the
host to size the receive buffers, as DeepEP's layout step does.

The per-token quantize happens once per token however many ranks it goes to;
the receive side can dequantize with a per-row weight (the routing-weighted
identity expert used by the benchmark) in the same pass.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import capi


def wire_row_bytes(hidden: int) -> int:
    """Bytes of one packed MXFP4 token row: H/2 code bytes + H/32 scale bytes."""
    return hidden // 2 + hidden // 32


def unpack_rowwise(packed: torch.Tensor):
    """Split packed rows at the 16/17 ratio into (codes, scales) views
    (megatron-0.15.0rc7.diff:40-63, `_unpack_rowwise_components`)."""
    last = packed.size(-1)
    if (last * 16) % 17 != 0:
        raise ValueError(f"Cannot infer FP4 rowwise/scale split for last_dim={last}. "
                         "Dimension must be divisible by the 17/16 packing ratio.")
    w = last * 16 // 17
    return packed.narrow(-1, 0, w), packed.narrow(-1, w, last - w)


class CudaKernels:
    """The CUDA data kernels of the dispatch path, through the C ABI."""

    def pack(self, x: torch.Tensor, slots: torch.Tensor, n_slots: int) -> torch.Tensor:
        T, H = x.shape
        wire = torch.empty(n_slots, wire_row_bytes(H), dtype=torch.uint8, device=x.device)
        capi.call("mxb_ep_pack", x.data_ptr(), T, H, slots.data_ptr(), slots.shape[1],
                  wire.data_ptr(), 1e-10, torch.cuda.current_stream(x.device).cuda_stream)
        return wire

    def unpack(self, wire: torch.Tensor, hidden: int,
               weight: Optional[torch.Tensor] = None) -> torch.Tensor:
        R = wire.shape[0]
        out = torch.empty(R, hidden, dtype=torch.bfloat16, device=wire.device)
        capi.call("mxb_ep_unpack", wire.data_ptr(), R, hidden,
                  None if weight is None else weight.data_ptr(), out.data_ptr(),
                  torch.cuda.current_stream(wire.device).cuda_stream)
        return out

    def combine(self, recv: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
        T, G = slots.shape
        H = recv.shape[1]
        out = torch.empty(T, H, dtype=torch.bfloat16, device=recv.device)
        capi.call("mxb_ep_combine", recv.data_ptr(), T, H, slots.data_ptr(), G, out.data_ptr(),
                  torch.cuda.current_stream(recv.device).cuda_stream)
        return out


def moe_permute_mxfp4(codes: torch.Tensor, scales: torch.Tensor, routing_map: torch.Tensor,
                      num_out_tokens: Optional[int] = None):
    """Transformer Engine's moe_permute (mask routing map) on the rowwise MXFP4
    data of a token tensor (the branch at transformer_engine-2.8.diff:253-261,
    338-356): codes uint8 [T, H/2] and E8M0 scales uint8 [T, H/32] (any row
    pitch; wire rows too), routing_map bool [T, E].  Returns (out_codes
    [num_out_tokens, H/2], out_scales [num_out_tokens, H/32], row_id_map int32
    [T, 2E + 1]); expert 0's tokens come first, in token order."""
    T, E = routing_map.shape
    H = codes.shape[1] * 2
    dev = codes.device
    if num_out_tokens is None:
        num_out_tokens = int(routing_map.sum().item())
    rmap = routing_map.contiguous().view(torch.uint8)
    rid = torch.empty(T, 2 * E + 1, dtype=torch.int32, device=dev)
    ws = torch.empty(E, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    capi.call("mxb_moe_make_row_id_map", rmap.data_ptr(), T, E, rid.data_ptr(), ws.data_ptr(), s)
    oc = torch.empty(num_out_tokens, H // 2, dtype=torch.uint8, device=dev)
    os_ = torch.empty(num_out_tokens, H // 32, dtype=torch.uint8, device=dev)
    capi.call("mxb_moe_permute_mxfp4_row_id_map", codes.data_ptr(), codes.stride(0),
              scales.data_ptr(), scales.stride(0), T, H, rid.data_ptr(), E, oc.data_ptr(),
              os_.data_ptr(), num_out_tokens, s)
    return oc, os_, rid


@dataclass
class Route:
    """Where each token goes.  slots[t, g] is the row of the send buffer that
    carries token t to rank g (-1 if t is not sent there); rows are grouped by
    destination rank and ordered by token within a rank."""
    slots: torch.Tensor          # int32 [T, G]
    send_counts: torch.Tensor    # int64 [G]
    src_token: torch.Tensor      # int64 [S]   token of each send row
    local_topk: torch.Tensor     # int32 [S, k] expert id local to the destination, -1 if elsewhere
    local_w: torch.Tensor        # float32 [S, k] routing weight, 0 where local_topk is -1


def build_route(topk_idx: torch.Tensor, topk_w: torch.Tensor, world: int,
                num_experts: int) -> Route:
    """Routing tables for top-k expert ids (global, experts contiguous per rank)."""
    T, k = topk_idx.shape
    per_rank = num_experts // world
    dest = torch.div(topk_idx, per_rank, rounding_mode="floor")          # [T, k]
    mask = torch.zeros(T, world, dtype=torch.bool, device=topk_idx.device)
    mask.scatter_(1, dest, True)
    send_counts = mask.sum(0)
    offsets = torch.cumsum(send_counts, 0) - send_counts
    within = torch.cumsum(mask.to(torch.int64), 0) - 1
    slots = torch.where(mask, offsets[None, :] + within, torch.full_like(within, -1))
    t_idx, g_idx = mask.nonzero(as_tuple=True)                           # row-major (t, g)
    s_idx = slots[t_idx, g_idx]
    order = torch.argsort(s_idx)
    t_sorted, g_sorted = t_idx[order], g_idx[order]
    here = dest[t_sorted] == g_sorted[:, None]                           # [S, k]
    local_topk = torch.where(here, topk_idx[t_sorted] - g_sorted[:, None] * per_rank,
                             torch.full_like(topk_idx[t_sorted], -1)).to(torch.int32)
    local_w = torch.where(here, topk_w[t_sorted].float(), torch.zeros_like(topk_w[t_sorted].float()))
    return Route(slots.to(torch.int32).contiguous(), send_counts, t_sorted, local_topk.contiguous(),
                 local_w.contiguous())


def weight_sums(w: torch.Tensor) -> torch.Tensor:
    """Row sums of routing weights, added left to right in float32 (a fixed
    order, so every device and the oracle agree bit for bit)."""
    acc = w[:, 0].float().clone()
    for j in range(1, w.shape[1]):
        acc += w[:, j].float()
    return acc.contiguous()


@dataclass
class Handle:
    route: Route
    send_splits: list
    recv_splits: list


class EPError(RuntimeError):
    """The expert-parallel exchange failed; the step's outputs are invalid."""


class EPTimeout(EPError):
    """A peer did not complete an exchange within the dispatcher's deadline
    (late, hung, or gone)."""


class EPProtocolError(EPError):
    """A peer sent a count table that cannot be right (negative counts, or more
    rows than it has tokens)."""


class MXFP4Dispatcher:
    """Dispatch / combine over a process group (one rank per GPU).

    Failure detection (DeepEP's dispatch waits are bounded the same way,
    deep_ep-1.2.1.diff:455-549): with `timeout_s`, every exchange is issued
    asynchronously and waited for at most that long on the host; a peer that
    is late, hung or gone raises EPTimeout (and a peer whose connection closed
    raises EPError) instead of blocking the step forever, after which
    `abort()` tears the process group down so that no collective stays queued.
    The count table every rank receives is checked before any row moves:
    counts must be non-negative and at most `max_tokens_per_rank`
    (EPProtocolError otherwise)."""

    def __init__(self, group=None, num_experts: int = 256, hidden: int = 7168, kernels=None,
                 timeout_s: Optional[float] = None, max_tokens_per_rank: Optional[int] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.num_experts = num_experts
        self.hidden = hidden
        self.k = kernels if kernels is not None else CudaKernels()
        self.timeout_s = timeout_s
        self.max_tokens_per_rank = max_tokens_per_rank

    def _wait(self, work, what: str):
        if self.timeout_s is None:
            work.wait()
            return
        import datetime
        try:
            ok = work.wait(timeout=datetime.timedelta(seconds=self.timeout_s))
        except RuntimeError as e:  # the backends report a timeout or a lost peer this way
            msg = str(e)
            if "imed out" in msg or "imeout" in msg:
                raise EPTimeout(f"rank {self.rank}: {what} not complete within "
                                f"{self.timeout_s} s: {msg}") from e
            raise EPError(f"rank {self.rank}: {what} failed: {msg}") from e
        if ok is False:
            raise EPTimeout(f"rank {self.rank}: {what} not complete within {self.timeout_s} s")

    def _a2a(self, out, inp, out_splits, in_splits, what="all-to-all"):
        if self.timeout_s is None:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
            return
        w = dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group,
                                   async_op=True)
        self._wait(w, what)

    def abort(self) -> None:
        """Tears down the process group after a failed exchange (aborts the
        NCCL communicator, so that no queued collective waits on a dead peer)."""
        from torch.distributed import distributed_c10d as c10d
        fn = getattr(c10d, "_abort_process_group", None)
        if fn is not None:
            fn(self.group)
        else:  # older torch: destroying the group is the closest
            dist.destroy_process_group(self.group)

    def _check_counts(self, recv_counts: torch.Tensor) -> None:
        c = recv_counts.tolist()
        cap = self.max_tokens_per_rank
        bad = [(src, n) for src, n in enumerate(c) if n < 0 or (cap is not None and n > cap)]
        if bad:
            raise EPProtocolError(f"rank {self.rank}: impossible row counts from "
                                  f"(source, count) {bad} (limit {cap})")

    def dispatch(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor):
        """Returns (recv_wire [R, 17H/32] u8, recv_topk int32 [R, k] local ids,
        recv_w float32 [R, k], handle)."""
        route = build_route(topk_idx, topk_w, self.world, self.num_experts)
        recv_counts = torch.empty_like(route.send_counts)
        self._a2a(recv_counts, self._send_counts(route), None, None, "count exchange")
        self._check_counts(recv_counts)
        send_splits = route.send_counts.tolist()
        recv_splits = recv_counts.tolist()
        S, R = sum(send_splits), sum(recv_splits)
        wire = self.k.pack(x, route.slots, S)
        recv_wire = torch.empty(R, wire.shape[1], dtype=torch.uint8, device=x.device)
        self._a2a(recv_wire, wire, recv_splits, send_splits, "row dispatch")
        kk = topk_idx.shape[1]
        recv_topk = torch.empty(R, kk, dtype=torch.int32, device=x.device)
        recv_w = torch.empty(R, kk, dtype=torch.float32, device=x.device)
        self._a2a(recv_topk, route.local_topk, recv_splits, send_splits, "routing dispatch")
        self._a2a(recv_w, route.local_w, recv_splits, send_splits, "weight dispatch")
        return recv_wire, recv_topk, recv_w, Handle(route, send_splits, recv_splits)

    def _send_counts(self, route: Route) -> torch.Tensor:
        """The count table row this rank sends (a hook for fault-injection tests)."""
        return route.send_counts

    def identity_experts(self, recv_wire: torch.Tensor, recv_w: torch.Tensor) -> torch.Tensor:
        """Expert stage of the benchmark: every local expert is the identity, so
        a row's output is its dequantized token times the sum of its local
        routing weights (rounded to BF16)."""
        return self.k.unpack(recv_wire, self.hidden, weight_sums(recv_w))

    def combine(self, y: torch.Tensor, handle: Handle) -> torch.Tensor:
        """Sends expert outputs back and sums each token's contributions."""
        back = torch.empty(sum(handle.send_splits), y.shape[1], dtype=y.dtype, device=y.device)
        self._a2a(back, y, handle.send_splits, handle.recv_splits, "combine")
        return self.k.combine(back, handle.route.slots)


def local_route(topk_idx: torch.Tensor, world: int, num_experts: int):
    """Device-side routing without host synchronisation: (within int32 [T, G],
    send_counts int32 [G], slots int32 [T, G]) where within[t, g] is token t's
    index among the tokens sent to rank g (-1 if none) and slots[t, g] its row
    in this rank's send order (grouped by destination)."""
    T = topk_idx.shape[0]
    per_rank = num_experts // world
    dest = torch.div(topk_idx, per_rank, rounding_mode="floor")
    mask = torch.zeros(T, world, dtype=torch.bool, device=topk_idx.device)
    mask.scatter_(1, dest, True)
    m64 = mask.to(torch.int64)
    send_counts = m64.sum(0)
    within = torch.where(mask, torch.cumsum(m64, 0) - 1, torch.full_like(m64, -1))
    offsets = torch.cumsum(send_counts, 0) - send_counts
    slots = torch.where(mask, offsets[None, :] + within, torch.full_like(m64, -1))
    return within.to(torch.int32), send_counts.to(torch.int32), slots.to(torch.int32)


class P2PDispatcher:
    """Fused dispatch / combine over NVLink peer memory (one process per GPU).

    Each rank owns one buffer (mxb_ep_layout) mapped into every peer with CUDA
    IPC.  A step runs five kernels and no host synchronisation: count exchange,
    fused quantize + peer store of the wire rows, barrier, expert stage fused
    with the peer store of its output rows, barrier; then the local combine.
    """

    def __init__(self, group=None, tcap: int = 4096, hidden: int = 7168, topk: int = 8,
                 num_experts: int = 256):
        import ctypes

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.hidden, self.topk, self.num_experts, self.tcap = hidden, topk, num_experts, tcap
        self.layout = capi.EpLayout()
        total = ctypes.c_int64()
        capi.call("mxb_ep_layout_init", self.world, self.rank, tcap, hidden, topk,
                  num_experts // self.world, ctypes.byref(self.layout), ctypes.byref(total))
        dev = torch.device("cuda", torch.cuda.current_device())
        self.buf = torch.zeros(total.value, dtype=torch.uint8, device=dev)
        torch.cuda.synchronize(dev)
        handle = (ctypes.c_char * 64)()
        off = ctypes.c_int64()
        capi.call("mxb_ipc_export", self.buf.data_ptr(), ctypes.cast(handle, ctypes.c_void_p),
                  ctypes.byref(off))
        objs = [None] * self.world
        dist.all_gather_object(objs, (bytes(handle), off.value), group=group)
        self._imported = []
        ptrs = []
        for p, (h, o) in enumerate(objs):
            if p == self.rank:
                ptrs.append(self.buf.data_ptr())
                continue
            hb = (ctypes.c_char * 64).from_buffer_copy(h)
            ptr = ctypes.c_void_p()
            capi.call("mxb_ipc_import", ctypes.cast(hb, ctypes.c_void_p), o, ctypes.byref(ptr))
            self._imported.append((ptr.value, o))
            ptrs.append(ptr.value)
        self.bases = torch.tensor([p if p < 2**63 else p - 2**64 for p in ptrs], dtype=torch.int64,
                                  device=dev)
        self.step_no = 0
        dist.barrier(group=group)
        L = self.layout
        self.back = self.buf[L.back_off:L.back_off + self.world * tcap * hidden * 2].view(
            torch.bfloat16).view(self.world * tcap, hidden)
        self.wire = self.buf[L.wire_off:L.wire_off + self.world * tcap * wire_row_bytes(hidden)].view(
            self.world * tcap, wire_row_bytes(hidden))

    def close(self):
        for ptr, o in self._imported:
            capi.status_of("mxb_ipc_close", ptr, o)
        self._imported = []

    def _args(self):
        import ctypes
        return self.bases.data_ptr(), ctypes.byref(self.layout)

    def _dispatch_phase(self, x, topk_idx, topk_w, mark):
        """Routing, count exchange, fused quantize + peer stores, barrier."""
        T = x.shape[0]
        s = torch.cuda.current_stream(x.device).cuda_stream
        topk_idx = topk_idx.to(torch.int64).contiguous()
        within = torch.empty(T, self.world, dtype=torch.int32, device=x.device)
        send_counts = torch.empty(self.world, dtype=torch.int32, device=x.device)
        capi.call("mxb_ep_route", topk_idx.data_ptr(), T, topk_idx.shape[1],
                  self.num_experts // self.world, self.world, within.data_ptr(),
                  send_counts.data_ptr(), s)
        mark("route")
        parity = self.step_no & 1
        e = 3 * self.step_no
        bases, lp = self._args()
        capi.call("mxb_ep_p2p_counts", bases, lp, send_counts.data_ptr(), parity, e + 1, s)
        mark("counts")
        capi.call("mxb_ep_p2p_dispatch", x.data_ptr(), T, within.data_ptr(),
                  topk_idx.data_ptr(),
                  topk_w.float().contiguous().data_ptr(), bases, lp, parity, s)
        mark("dispatch")
        capi.call("mxb_ep_p2p_barrier", bases, lp, e + 2, s)
        mark("barrier1")
        return within, send_counts, parity, e

    def dispatch_only(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor,
                      mark=None) -> None:
        """The dispatch half of a step: after it every rank's receive rows
        (self.wire, grouped by source rank) hold the MXFP4 wire rows routed to
        it.  Used to time the dispatch alone; a full step() may follow."""
        self._dispatch_phase(x, topk_idx, topk_w, mark or (lambda _n: None))
        self.step_no += 1

    def step(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor,
             expert_fn=None, mark=None) -> torch.Tensor:
        """Dispatch -> experts -> combine.  Without expert_fn every expert is the
        identity and a row returns as its dequantized token times its local
        routing-weight sum (fused into the return kernel).  mark(name), if
        given, is called after each phase is enqueued (route, counts, dispatch,
        barrier1, return, barrier2, combine), e.g. to record CUDA events."""
        mark = mark or (lambda _n: None)
        T = x.shape[0]
        s = torch.cuda.current_stream(x.device).cuda_stream
        within, send_counts, parity, e = self._dispatch_phase(x, topk_idx, topk_w, mark)
        bases, lp = self._args()
        y = None if expert_fn is None else expert_fn(self.wire).contiguous()
        capi.call("mxb_ep_p2p_return", None if y is None else y.data_ptr(), bases, lp, parity, s)
        mark("return")
        capi.call("mxb_ep_p2p_barrier", bases, lp, e + 3, s)
        mark("barrier2")
        out = torch.empty(T, self.hidden, dtype=torch.bfloat16, device=x.device)
        capi.call("mxb_ep_p2p_combine", self.back.data_ptr(), T, self.hidden, within.data_ptr(),
                  send_counts.data_ptr(), self.world, out.data_ptr(), s)
        mark("combine")
        self.step_no += 1
        return out

    def check(self) -> None:
        """Raises PeerTimeout if a cross-GPU wait of this process gave up since
        the last check (a peer is late or gone, and the outputs of the steps
        since then are invalid).  Synchronises the device."""
        n = int(capi.load().mxb_ep_reset_wait_timeouts())
        if n:
            raise PeerTimeout(f"rank {self.rank}: {n} cross-GPU wait(s) gave up")


class PeerTimeout(RuntimeError):
    """A bounded cross-GPU wait of the fused dispatcher ran out."""


class NcclCDispatcher:
    """Dispatch / combine through the C ABI over an NCCL communicator of its own
    (mxb_ep_nccl_dispatch / mxb_ep_nccl_combine): the path a C or C++ caller
    holding an ncclComm_t uses, here driven from Python.  Same results as
    MXFP4Dispatcher.  `nccl_id` is the 128-byte id of rank 0's
    `NcclCDispatcher.unique_id()`, shared by any means (e.g. a store)."""

    @staticmethod
    def unique_id() -> bytes:
        import ctypes
        buf = (ctypes.c_char * 128)()
        capi.call("mxb_nccl_unique_id", ctypes.cast(buf, ctypes.c_void_p))
        return bytes(buf)

    def __init__(self, world: int, rank: int, nccl_id: bytes, tokens: int, hidden: int = 7168,
                 topk: int = 8, num_experts: int = 256):
        import ctypes
        self.world, self.rank, self.hidden, self.topk = world, rank, hidden, topk
        self.tokens, self.num_experts = tokens, num_experts
        idb = (ctypes.c_char * 128).from_buffer_copy(nccl_id)
        self.comm = ctypes.c_void_p()
        capi.call("mxb_nccl_comm_init", ctypes.byref(self.comm), world, rank,
                  ctypes.cast(idb, ctypes.c_void_p))
        dev = torch.device("cuda", torch.cuda.current_device())
        nb = int(capi.load().mxb_ep_nccl_workspace_bytes(tokens, hidden, topk, world))
        self.ws = torch.empty(nb, dtype=torch.uint8, device=dev)
        self.cap = world * tokens
        self.recv_wire = torch.empty(self.cap, wire_row_bytes(hidden), dtype=torch.uint8, device=dev)
        self.recv_meta = torch.empty(self.cap, 2 * topk, dtype=torch.int32, device=dev)
        self.handle = capi.EpHandle()

    def dispatch(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor):
        """Returns (recv_wire [R, 17H/32], recv_topk int32 [R, k], recv_w float32 [R, k])."""
        import ctypes
        T = x.shape[0]
        idx = topk_idx.to(torch.int64).contiguous()
        w = topk_w.float().contiguous()
        s = torch.cuda.current_stream(x.device).cuda_stream
        capi.call("mxb_ep_nccl_dispatch", self.comm, self.world, self.rank, x.data_ptr(), T,
                  self.hidden, idx.data_ptr(), w.data_ptr(), self.topk,
                  self.num_experts // self.world, self.ws.data_ptr(), self.ws.numel(),
                  self.recv_wire.data_ptr(), self.recv_meta.data_ptr(), self.cap,
                  ctypes.byref(self.handle), s)
        R = int(self.handle.n_recv)
        meta = self.recv_meta[:R]
        return (self.recv_wire[:R], meta[:, :self.topk],
                meta[:, self.topk:].contiguous().view(torch.float32))

    def combine(self, y: torch.Tensor) -> torch.Tensor:
        import ctypes
        T = int(self.handle.tokens)
        out = torch.empty(T, self.hidden, dtype=torch.bfloat16, device=y.device)
        capi.call("mxb_ep_nccl_combine", self.comm, ctypes.byref(self.handle),
                  y.contiguous().data_ptr(), self.ws.data_ptr(), self.ws.numel(), out.data_ptr(),
                  torch.cuda.current_stream(y.device).cuda_stream)
        return out

    def close(self):
        import ctypes
        if self.comm:
            capi.status_of("mxb_nccl_comm_destroy", self.comm)
            self.comm = ctypes.c_void_p()
