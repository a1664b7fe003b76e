"""Per-step forward context shared by the model runner and the attention layers.

Same fields, defaults and functions as the reference's side channel
(dllmserve/utils/context.py:6-68): the runner calls ``set_context`` once per
denoising step and every ``Attention.forward`` reads ``get_context()``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | list | None = None
    extra_slot_mapping: torch.Tensor | list | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    is_diffusion: bool = False
    seqs: Optional[list] = None


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(
    is_prefill,
    cu_seqlens_q=None,
    cu_seqlens_k=None,
    max_seqlen_q=0,
    max_seqlen_k=0,
    slot_mapping=None,
    extra_slot_mapping=None,
    context_lens=None,
    block_tables=None,
    is_diffusion=False,
    seqs=None,
):
    """Replace the module-global context (a new object every call, so the
    attention layers can cache per-step metadata keyed on it)."""
    global _CONTEXT
    _CONTEXT = Context(
        is_prefill=is_prefill,
        cu_seqlens_q=cu_seqlens_q,
        cu_seqlens_k=cu_seqlens_k,
        max_seqlen_q=max_seqlen_q,
        max_seqlen_k=max_seqlen_k,
        slot_mapping=slot_mapping,
        extra_slot_mapping=extra_slot_mapping,
        context_lens=context_lens,
        block_tables=block_tables,
        is_diffusion=is_diffusion,
        seqs=seqs,
    )


def use_context(ctx: Context) -> None:
    """Install an existing Context object. The attention layers cache the
    per-step device metadata on the Context, so reinstalling the same object
    for steps with identical sequence states (e.g. the reuse steps of a
    diffusion block) skips rebuilding it and keeps CUDA-graph captures free of
    host-to-device copies. A CUDA graph captured under a Context reads that
    metadata (sequence offsets, selection descriptors, slot lists) by device
    address: keep the Context object alive, and unchanged, for as long as the
    graph is replayed."""
    global _CONTEXT
    _CONTEXT = ctx


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()
