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


def selection_prompts(case) -> list[int]:
    """Seeded prompt lengths of a SelectionCase."""
    g = gen(1000 + case.seed)
    lo, hi = case.prompt_range
    return torch.randint(lo, hi + 1, (case.batch,), generator=g).tolist()


def margin_selection_batch(case, step: float = 64.0):
    """q, k, v [N, H/Hkv, 128] (bf16 values in fp32) for a batch of sequences
    whose current block is the first generation block, with margin-separated
    candidate keys (every fp32 summation order ranks them alike):
      * q, k, v ~ N(0, 1);
      * per KV head h two seeded dims d1, d2: every block query row of the
        head's query heads gets q[d1] = 1, q[d2] = 64, so the block mean has
        exactly 1 and 64 there; every candidate key (a token outside the
        block) gets k[d1] = 64 * (rank mod 64), k[d2] = 64 * (rank div 64) --
        all exact in bf16 -- which adds exactly 64 * rank to its raw score.
        rank is a seeded permutation of the candidates, per KV head with
        head_select and one per token shared by every head without it;
      * `scaled_heads` seeded KV heads then get their other key dims scaled
        by 3 (a 3x key norm outside the margin dims).
    The N(0,1) part of a raw score has std ~2 (~6 scaled), so distinct scores
    sit at least ~10 apart at magnitudes up to ~64 * Klen (~1e-4 relative),
    against fp32 summation-order differences of ~1e-7 relative.
    Returns (q, k, v, prompts, lens)."""
    g = gen(case.seed)
    H, Hk, D, blk = case.num_heads, case.num_kv_heads, 128, case.block_len
    G = H // Hk
    prompts = selection_prompts(case)
    lens = [p + case.gen_len for p in prompts]
    base = int(step)
    qs, ks, vs = [], [], []
    for p, L in zip(prompts, lens):
        q = normal(g, (L, H, D))
        k = normal(g, (L, Hk, D))
        v = normal(g, (L, Hk, D))
        dims = torch.stack([torch.randperm(D, generator=g)[:2] for _ in range(Hk)])   # [Hk, 2]
        if case.scaled_heads:
            hs = torch.randperm(Hk, generator=g)[:case.scaled_heads]
            k[:, hs] = (k[:, hs] * 3).to(torch.bfloat16).float()
        klen = L - blk
        cand = torch.cat([torch.arange(0, p), torch.arange(p + blk, L)])
        if case.head_select:
            rank = torch.stack([torch.randperm(klen, generator=g) for _ in range(Hk)], 1)   # [klen, Hk]
        else:
            rank = torch.randperm(klen, generator=g)[:, None].expand(klen, Hk)
        for h in range(Hk):
            d1, d2 = int(dims[h, 0]), int(dims[h, 1])
            q[p:p + blk, h * G:(h + 1) * G, d1] = 1.0
            q[p:p + blk, h * G:(h + 1) * G, d2] = float(base)
            k[cand, h, d1] = (step * (rank[:, h] % base)).float()
            k[cand, h, d2] = (step * (rank[:, h] // base)).float()
        qs.append(q), ks.append(k), vs.append(v)
    return torch.cat(qs), torch.cat(ks), torch.cat(vs), prompts, lens
