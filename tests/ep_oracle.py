"""TEST INFRASTRUCTURE: CPU stand-ins for the three EP data kernels, built on
the oracle, and the expected result of a dispatch -> identity experts ->
combine round.  Used by the gloo (CPU) protocol tests and as the checker of
the CUDA kernels; the product path never uses them."""
import numpy as np
import torch

from mxfp4_b200 import synthetic as syn
from mxfp4_b200.ep import wire_row_bytes
from oracle import oracle as O


def bits_to_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def pack_rows(x):
    """Oracle wire rows [T, 17H/32] of bf16 x [T, H]."""
    q, s = O.quant_rows(syn.bf16_bits(x))
    return np.concatenate([q, s], axis=1)


def unpack_rows(wire, hidden, weight=None):
    """Oracle dequant of wire rows (+ per-row weight, rounded to bf16)."""
    wire = np.ascontiguousarray(wire)
    q, s = wire[:, :hidden // 2], wire[:, hidden // 2:]
    dq = O.dequant_bf16(np.ascontiguousarray(q), np.ascontiguousarray(s))
    if weight is None:
        return dq
    f = (dq.astype(np.uint32) << 16).view(np.float32) * np.asarray(weight, np.float32)[:, None]
    return _f32_to_bf16(f)


def _f32_to_bf16(f):
    u = np.ascontiguousarray(f, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def combine_rows(recv_bits, slots):
    """out[t] = bf16(sum over g of float(recv[slots[t, g]])), g ascending."""
    T, G = slots.shape
    H = recv_bits.shape[1]
    acc = np.zeros((T, H), np.float32)
    for g in range(G):
        sel = slots[:, g] >= 0
        if sel.any():
            acc[sel] += (recv_bits[slots[sel, g]].astype(np.uint32) << 16).view(np.float32)
    return _f32_to_bf16(acc)


class OracleKernels:
    """CPU kernels with the CUDA kernels' semantics (for gloo tests)."""

    def pack(self, x, slots, n_slots):
        rows = pack_rows(x)
        wire = np.zeros((n_slots, wire_row_bytes(x.shape[1])), np.uint8)
        sl = slots.numpy()
        for g in range(sl.shape[1]):
            sel = sl[:, g] >= 0
            wire[sl[sel, g]] = rows[sel]
        return torch.from_numpy(wire)

    def unpack(self, wire, hidden, weight=None):
        w = None if weight is None else weight.numpy()
        return bits_to_bf16(unpack_rows(wire.numpy(), hidden, w))

    def combine(self, recv, slots):
        bits = recv.contiguous().view(torch.int16).numpy().view(np.uint16)
        return bits_to_bf16(combine_rows(bits, slots.numpy()))


def expected_round(x, topk_idx, topk_w, world, num_experts):
    """Expected output of dispatch -> identity experts (x local weight sum) ->
    combine for one rank's tokens, computed from that rank's inputs alone."""
    from mxfp4_b200.ep import build_route, weight_sums
    route = build_route(topk_idx, topk_w, world, num_experts)
    rows = pack_rows(x)
    H = x.shape[1]
    wsum = weight_sums(route.local_w).numpy()
    src = route.src_token.numpy()
    y = unpack_rows(rows[src], H, wsum)
    return combine_rows(y, route.slots.numpy())
