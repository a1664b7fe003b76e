"""Drop-in ``RotaryEmbedding`` / ``get_rope`` (dllmserve/layers/rotary_embedding.py).

Same constructor, cos/sin cache (built with the same torch ops, so the same
fp32 values) and ``forward(positions, query, key) -> (query, key)`` contract as
the reference (rotary_embedding.py:19-57); the rotation runs in one native
launch for q and k together (``dllm_rope_neox``) instead of the reference's
compiled elementwise graph, with bit-identical bf16 results.
"""
from __future__ import annotations

from functools import lru_cache

import torch
from torch import nn

from .. import ops


class RotaryEmbedding(nn.Module):
    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float) -> None:
        super().__init__()
        self.head_size = head_size
        assert rotary_dim == head_size
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
        t = torch.arange(max_position_embeddings, dtype=torch.float)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1)
        self.register_buffer("cos_sin_cache", cache, persistent=False)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        n = positions.size(0)
        q = query.view(n, -1, self.head_size)
        k = key.view(n, -1, self.head_size)
        if self.cos_sin_cache.device != q.device:
            self.cos_sin_cache = self.cos_sin_cache.to(q.device)
        qo, ko = ops.rope_neox(positions.to(torch.int64).contiguous(), q, k, self.cos_sin_cache)
        return qo.view(query.shape), ko.view(key.shape)


@lru_cache(1)
def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float, rope_scaling: dict | None = None):
    assert rope_scaling is None
    return RotaryEmbedding(head_size, rotary_dim, max_position, base)
