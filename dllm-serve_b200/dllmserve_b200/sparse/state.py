"""Sparse-attention configuration and the per-request diffusion-block state machine.

Behaviour follows the reference's dllmserve/sparse/state.py:
  * ``SparseConfig`` fields and code defaults (state.py:6-16).
  * ``PerRequestSparseState.advance_step`` (state.py:77-104): per diffusion
    block of ``default_block_len`` steps, with ``delay_step == 1`` the first
    step runs full attention (state 0), the second computes and stores the
    selected K/V (state 1) and the rest reuse the cache (state 2).
  * block boundaries (state.py:44-62) and the block / prefix+suffix index
    ranges (state.py:107-136).
As in the reference, ``enabled`` is only consulted by ``get_cache_state``;
a state created for ``enabled=False`` still advances.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class SparseConfig:
    """Per-request sparse-dLLM configuration."""

    enabled: bool = False
    default_block_len: int = 32
    retention_ratio: float = 0.5
    pool_kernel: int = 3
    delay_step: int = 1
    head_select: bool = False


@dataclass
class SparseContext:
    """Per-sequence sparse context record (state.py:18-29)."""

    cache_state: int
    block_indices: torch.Tensor
    block_spans: torch.Tensor
    retention_ratio: float
    pool_kernel: int
    seq_sparse_state: Optional["PerRequestSparseState"] = None


def num_keep(num_candidates: int, retention_ratio: float) -> int:
    """Rows kept from ``num_candidates``: ``min(max(1, int(n * r)), n)``
    (attention.py:396-399, sequence.py:119-123)."""
    if num_candidates <= 0:
        return 0
    return min(max(1, int(num_candidates * retention_ratio)), num_candidates)


class PerRequestSparseState:
    """Diffusion-block cursor and cache state of one request."""

    def __init__(self, seq_id: int, config: SparseConfig, device):
        self.seq_id = seq_id
        self.config = config
        self.current_block_idx = 0
        self.step_in_block = 0
        self.cache_state = 0
        self.device = device

    # -- block geometry ------------------------------------------------------
    def compute_block_boundaries(self, prompt_len: int, total_len: int) -> tuple[int, int]:
        """(block_start, block_length) of the current block, absolute positions."""
        if total_len - prompt_len <= 0:
            return (prompt_len, 0)
        start = prompt_len + self.current_block_idx * self.block_len
        return (start, min(self.block_len, total_len - start))

    def get_cache_state(self) -> int:
        return self.cache_state if self.config.enabled else 0

    def advance_step(self):
        self.step_in_block += 1
        if self.step_in_block % self.block_len == 0:
            self.step_in_block = 0
            self.current_block_idx += 1
        d = self.config.delay_step
        s = self.step_in_block
        if d == 1:
            self.cache_state = 0 if s == 0 else (1 if s == 1 else 2)
        elif d == 0:
            self.cache_state = 1 if s == 0 else 2
        else:
            self.cache_state = 0 if s < d else (1 if s == d else 2)

    def get_block_indices(self, prompt_len, total_len) -> torch.Tensor:
        start, length = self.compute_block_boundaries(prompt_len, total_len)
        self.block_indices = torch.arange(start, start + length, dtype=torch.int64, device=self.device)
        return self.block_indices

    def get_unuse_block_indices(self, prompt_len, total_len) -> torch.Tensor:
        start, length = self.compute_block_boundaries(prompt_len, total_len)
        self.block_indices_prefix = torch.arange(0, start, dtype=torch.int64, device=self.device)
        self.block_indices_suffix = torch.arange(
            start + length, total_len, dtype=torch.int64, device=self.device
        )
        self.block_indices = torch.cat([self.block_indices_prefix, self.block_indices_suffix], dim=0)
        return self.block_indices

    def num_unused_tokens(self, prompt_len: int, total_len: int) -> int:
        """len(get_unuse_block_indices(...)) without building the tensor."""
        start, length = self.compute_block_boundaries(prompt_len, total_len)
        return max(0, start) + max(0, total_len - (start + length))

    # -- config views ----------------------------------------------------------
    @property
    def pool_kernel(self):
        return self.config.pool_kernel

    @property
    def retention_ratio(self):
        return self.config.retention_ratio

    @property
    def block_len(self):
        return self.config.default_block_len

    @property
    def should_compute_cache(self) -> bool:
        return self.cache_state == 1

    @property
    def should_reuse_cache(self) -> bool:
        return self.cache_state == 2

    @property
    def is_full_attention(self) -> bool:
        return self.cache_state == 0
