"""Seeded synthetic inputs shared by the golden-vector generator and the tests.

Two value families, both exactly representable in bf16:
  * ``normal``: N(0, 1) rounded to bf16.
  * ``grid``:   integers in [-32, 32) times 2^-5 (values in [-1, 1), the
    scale of N(0,1) data, so the bf16 attention tolerances apply as stated).
    Dot products of up to 128 terms, means over power-of-two blocks and sums
    over heads are then exact in fp32 whatever the summation order, so
    importance scores (and with them the top-k selection) are bit-identical
    across implementations.
"""
from __future__ import annotations

import torch


def gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def normal(g: torch.Generator, shape) -> torch.Tensor:
    return torch.randn(shape, generator=g).to(torch.bfloat16).float()


def grid(g: torch.Generator, shape) -> torch.Tensor:
    return torch.randint(-32, 32, shape, generator=g).float() * (1.0 / 32.0)


def make(kind: str, g: torch.Generator, shape) -> torch.Tensor:
    return grid(g, shape) if kind == "grid" else normal(g, shape)


def page_slots(g: torch.Generator, n: int, num_pages: int, page: int = 256) -> torch.Tensor:
    """Slots of n cached rows laid out like the model runner does
    (model_runner.py:257-264): consecutive rows inside pages taken from a
    random block table."""
    pages = torch.randperm(num_pages, generator=g)[: (n + page - 1) // page]
    out = []
    for j, p in enumerate(pages.tolist()):
        m = min(page, n - j * page)
        out.extend(range(p * page, p * page + m))
    return torch.tensor(out, dtype=torch.int32)


def checksum(t: torch.Tensor) -> list[float]:
    """Cheap fingerprint of a generated tensor (sum, sum of squares, first value)."""
    f = t.double().reshape(-1)
    return [float(f.sum()), float((f * f).sum()), float(f[0]) if f.numel() else 0.0]
