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


class MXFP4Dispatcher:
    """Dispatch / combine over a process group (one rank per GPU)."""

    def __init__(self, group=None, num_experts: int = 256, hidden: int = 7168, kernels=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.num_experts = num_experts
        self.hidden = hidden
        self.k = kernels if kernels is not None else CudaKernels()

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def dispatch(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor):
        """Returns (recv_wire [R, 17H/32] u8, recv_topk int32 [R, k] local ids,
        recv_w float32 [R, k], handle)."""
        route = build_route(topk_idx, topk_w, self.world, self.num_experts)
        recv_counts = torch.empty_like(route.send_counts)
        dist.all_to_all_single(recv_counts, route.send_counts, group=self.group)
        send_splits = route.send_counts.tolist()
        recv_splits = recv_counts.tolist()
        S, R = sum(send_splits), sum(recv_splits)
        wire = self.k.pack(x, route.slots, S)
        recv_wire = torch.empty(R, wire.shape[1], dtype=torch.uint8, device=x.device)
        self._a2a(recv_wire, wire, recv_splits, send_splits)
        kk = topk_idx.shape[1]
        recv_topk = torch.empty(R, kk, dtype=torch.int32, device=x.device)
        recv_w = torch.empty(R, kk, dtype=torch.float32, device=x.device)
        self._a2a(recv_topk, route.local_topk, recv_splits, send_splits)
        self._a2a(recv_w, route.local_w, recv_splits, send_splits)
        return recv_wire, recv_topk, recv_w, Handle(route, send_splits, recv_splits)

    def identity_experts(self, recv_wire: torch.Tensor, recv_w: torch.Tensor) -> torch.Tensor:
        """Expert stage of the benchmark: every local expert is the identity, so
        a row's output is its dequantized token times the sum of its local
        routing weights (rounded to BF16)."""
        return self.k.unpack(recv_wire, self.hidden, weight_sums(recv_w))

    def combine(self, y: torch.Tensor, handle: Handle) -> torch.Tensor:
        """Sends expert outputs back and sums each token's contributions."""
        back = torch.empty(sum(handle.send_splits), y.shape[1], dtype=y.dtype, device=y.device)
        self._a2a(back, y, handle.send_splits, handle.recv_splits)
        return self.k.combine(back, handle.route.slots)
