"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations.  The reference publishes no dataset for this path;
these generators stand in for it.  All draws use torch's CPU generator, so the
same seed gives the same bytes on every machine; callers copy to the GPU.

  config 1  bf16 [4096, 4096] ~ N(0,1), 0.1% of entries x100, seed 0
  config 2  bf16 [16384, 8192] ~ N(0,1) x per-row 10^U(-2, 2), seed 1
  config 3  MXFP4 codes u8 [16384, 8192] uniform, E8M0 scales uniform in
            [117, 137] (one per 16 code bytes), seed 2
  config 4  bf16 [32768, 7168] ~ N(0,1), 0.5% of entries x50, seed 3
  config 5  MoE tokens bf16 [4096, 7168] per rank, top-8 of 256 experts,
            softmax(N(0,1)) routing weights, seed 4
"""
from __future__ import annotations

import torch


def _gen(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(seed)


def _outliers(x: torch.Tensor, frac: float, factor: float, g: torch.Generator) -> torch.Tensor:
    n = x.numel()
    k = int(round(n * frac))
    idx = torch.randperm(n, generator=g)[:k]
    flat = x.view(-1)
    flat[idx] = flat[idx] * factor
    return x


def config1(rows: int = 4096, cols: int = 4096, seed: int = 0) -> torch.Tensor:
    g = _gen(seed)
    x = torch.randn(rows, cols, generator=g, dtype=torch.float32)
    return _outliers(x, 0.001, 100.0, g).to(torch.bfloat16)


def config2(rows: int = 16384, cols: int = 8192, seed: int = 1) -> torch.Tensor:
    g = _gen(seed)
    x = torch.randn(rows, cols, generator=g, dtype=torch.float32)
    row_scale = torch.pow(10.0, torch.rand(rows, 1, generator=g) * 4.0 - 2.0)
    return (x * row_scale).to(torch.bfloat16)


def config3(rows: int = 16384, code_bytes: int = 8192, seed: int = 2, lo: int = 117,
            hi: int = 137):
    """Returns (codes u8 [rows, code_bytes], scales u8 [rows, code_bytes / 16])."""
    g = _gen(seed)
    codes = torch.randint(0, 256, (rows, code_bytes), generator=g, dtype=torch.uint8)
    scales = torch.randint(lo, hi + 1, (rows, code_bytes // 16), generator=g, dtype=torch.uint8)
    return codes, scales


def config3_splits(rows: int = 16384, segments: int = 8, multiple: int = 1, seed: int = 7):
    """Seeded expert-segment sizes for the split converter (the grouped-GEMM
    wgrad operand): `segments` shares of `rows`, each a multiple of `multiple`
    (1: ragged), summing to rows."""
    wts = torch.rand(segments, generator=_gen(seed)) + 0.5
    m = ((wts / wts.sum() * rows / multiple).floor() * multiple).to(torch.int64).tolist()
    m[-1] += rows - sum(m)
    return m


def config4(rows: int = 32768, cols: int = 7168, seed: int = 3) -> torch.Tensor:
    g = _gen(seed)
    x = torch.randn(rows, cols, generator=g, dtype=torch.float32)
    return _outliers(x, 0.005, 50.0, g).to(torch.bfloat16)


def config5(rank: int, world: int, tokens: int = 4096, hidden: int = 7168, experts: int = 256,
            topk: int = 8, seed: int = 4):
    """Per-rank MoE inputs: (x bf16 [T, H], topk_idx int64 [T, k], topk_w f32 [T, k])."""
    g = _gen(seed * 1000 + rank)
    x = torch.randn(tokens, hidden, generator=g, dtype=torch.float32).to(torch.bfloat16)
    idx = torch.rand(tokens, experts, generator=g).topk(topk, dim=1).indices
    w = torch.softmax(torch.randn(tokens, topk, generator=g), dim=1)
    return x, idx, w


def bf16_bits(x: torch.Tensor):
    """BF16 tensor -> numpy uint16 bit patterns (CPU)."""
    return x.detach().cpu().contiguous().view(torch.int16).numpy().view("uint16")
