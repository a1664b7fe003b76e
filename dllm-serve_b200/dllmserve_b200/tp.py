"""Tensor-parallel head sharding around the attention path.

Rank r of a tp-way group owns query heads [r*Hq/tp, (r+1)*Hq/tp) and KV heads
[r*Hkv/tp, (r+1)*Hkv/tp) - the contiguous slices ColumnParallelLinear gives
the q/k/v projections (dllmserve/layers/linear.py:55-88) and the per-rank
cache [.., Hkv/tp, D] (model_runner.py:174). Attention needs no exchange; the
one collective is the all-reduce of the row-parallel o_proj output
(linear.py:186-190).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F


def head_slice(num_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[int, int, int, int]:
    """(q_head_begin, q_head_end, kv_head_begin, kv_head_end) of ``rank``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if num_heads % world or num_kv_heads % world:
        raise ValueError(
            f"{num_heads} query / {num_kv_heads} KV heads do not split over {world} ranks")
    hq, hk = num_heads // world, num_kv_heads // world
    return rank * hq, (rank + 1) * hq, rank * hk, (rank + 1) * hk


def row_parallel_oproj(x: torch.Tensor, weight_shard: torch.Tensor, bias: torch.Tensor | None = None,
                       rank: int = 0, group=None, chunks: int = 1) -> torch.Tensor:
    """y = x @ W_shard^T (+ bias on rank 0), summed over ranks (linear.py:186-190).

    ``chunks`` > 1 splits the rows: each chunk's GEMM is followed by an
    asynchronous all-reduce of that chunk, which runs on NCCL's stream while
    the next chunk's GEMM runs on the current one. The all-reduce is
    elementwise, so chunking changes nothing it sums; a chunk's GEMM may
    round differently from the whole one (the library picks its algorithm
    per shape)."""
    distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
    b = bias if rank == 0 else None
    if not distributed or chunks <= 1 or x.shape[0] < chunks:
        y = F.linear(x, weight_shard, b)
        if distributed:
            dist.all_reduce(y, group=group)
        return y
    y = torch.empty(x.shape[0], weight_shard.shape[0], dtype=x.dtype, device=x.device)
    bounds = [x.shape[0] * i // chunks for i in range(chunks + 1)]
    works = []
    for i in range(chunks):
        r0, r1 = bounds[i], bounds[i + 1]
        if b is not None:
            torch.addmm(b, x[r0:r1], weight_shard.t(), out=y[r0:r1])
        else:
            torch.matmul(x[r0:r1], weight_shard.t(), out=y[r0:r1])
        works.append(dist.all_reduce(y[r0:r1], group=group, async_op=True))
    for w in works:
        w.wait()
    return y
