"""Drop-in ``Attention`` layer for diffusion LLMs on B200.

Keeps the reference's module contract (dllmserve/layers/attention.py:95-119):
``Attention(num_heads, head_dim, scale, num_kv_heads, causal=True)`` with the
``k_cache`` / ``v_cache`` / ``layer_id`` attributes bound by the model runner,
and ``forward(q, k, v) -> [N, num_heads * head_dim]`` reading the per-step
``Context``. Also re-exports ``store_kvcache`` / ``load_kvcache`` with the
reference's argument order and assertions (attention.py:33-92).

The diffusion path (``context.is_diffusion``, attention.py:150-306) runs as
  1. one non-causal varlen attention launch over every sequence, whose keys
     are [cached rows read from the paged cache by slot ; fresh rows] for
     "reuse" sequences (state 2), and
  2. one scoring/top-k/store launch per ``head_select`` flavour for the
     sequences in the "compute cache" state (state 1),
with all per-sequence metadata built once per step (``StepPlan``). The
reference stores the selection before it attends; the two launches touch
disjoint memory (the selection writes only state-1 sequences' cache slots,
the attention reads only state-2 ones), so the order changes no result.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..engine.step_plan import build_step_plan, selection_arrays
from ..utils import context as _context_mod

# Where the layer reads the step context from. ``integration.install`` points
# this at the reference package's ``get_context`` so a reference model runner
# drives this layer unchanged.
get_context = _context_mod.get_context

store_kvcache = ops.store_kvcache
load_kvcache = ops.load_kvcache

_PLAN_ATTR = "_dllm_b200_plans"


def _plan_for(ctx, q: torch.Tensor, num_kv_heads: int):
    plans = getattr(ctx, _PLAN_ATTR, None)
    if plans is None:
        plans = {}
        try:
            setattr(ctx, _PLAN_ATTR, plans)
        except AttributeError:  # a frozen context: rebuild per layer
            pass
    key = (q.get_device(), q.shape[0], num_kv_heads)
    plan = plans.get(key)
    if plan is None:
        plan = build_step_plan(ctx, q.device, q.shape[0], num_kv_heads)
        plans[key] = plan
    return plan


class Attention(nn.Module):
    def __init__(self, num_heads, head_dim, scale, num_kv_heads, causal=True):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.causal = causal
        self.k_cache = self.v_cache = torch.tensor([])
        self.layer_id = None
        # top_idx of the last "compute cache" launch per head_select flavour
        # (device int64); kept only when ``record_selection`` is set.
        self.record_selection = False
        self.last_selection: dict = {}
        self._cache_sig = None  # (k_cache, v_cache, k_cache ptr, validated paged-cache arguments)
        self._launch_key = ("attn", num_heads, num_kv_heads, head_dim, scale)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        context = get_context()
        if context.is_diffusion and q.dim() in (2, 3) and k.dim() == q.dim() and v.dim() == q.dim():
            # token-row layouts ([N, heads*D] or [N, heads, D]) go to the
            # launch as they are (no per-layer views)
            return self._diffusion_attention(q, k, v, context)
        q = q.view(-1, self.num_heads, self.head_dim)
        k = k.view(-1, self.num_kv_heads, self.head_dim)
        v = v.view(-1, self.num_kv_heads, self.head_dim)
        if context.is_diffusion:
            return self._diffusion_attention(q, k, v, context)
        if self.k_cache.numel() and self.v_cache.numel():
            store_kvcache(k, v, self.k_cache, self.v_cache, context.slot_mapping)
        return self._regular_attention(q, k, v, context)

    def _regular_attention(self, q, k, v, context):
        """Non-diffusion path (attention.py:121-148). Only the non-causal,
        non-paged prefill form exists on this path's kernels."""
        if self.causal or not context.is_prefill or context.block_tables is not None:
            raise NotImplementedError(
                "dllmserve_b200 implements the diffusion (non-causal) attention path only")
        o = ops.varlen_attention(q, k, v, context.cu_seqlens_q, context.cu_seqlens_k,
                                 int(context.max_seqlen_q), self.scale)
        return o.view(-1, self.num_heads * self.head_dim)

    def _diffusion_attention(self, q, k, v, context):
        """q [N, num_heads*D] or [N, num_heads, D]; k, v likewise with
        num_kv_heads; returns [N, num_heads*D]."""
        plan = _plan_for(context, q, self.num_kv_heads)
        H, Hk, D = self.num_heads, self.num_kv_heads, self.head_dim
        if self.record_selection:
            self.last_selection = {}
        out = q.new_empty((q.shape[0], H * D))
        launch = plan.scratch.get(self._launch_key)
        if launch is None:
            dev = q.device
            # step-level arguments validated once per plan, shared by the layers of this shape
            launch = ops.prepare_attention(
                plan.cu, plan.cu, plan.max_rows, plan.total_rows, H, Hk, D, self.scale, dev,
                slots=plan.slots_c, cu_seqlens_slots=plan.cu_c)
            plan.scratch[self._launch_key] = launch
        # out was made here with the launch's layout (q's dtype and device, [rows, H*D])
        res = launch(q, k, v, out, self._paged_cache_args() if plan.total_c > 0 else None, out_checked=True)
        # The selection runs after the attention: it writes only the cache slots
        # of compute-cache sequences, which no launch of this step reads, and
        # finds this layer's K/V still partly in L2.
        if plan.sel:
            dev = q.device
            qv, kv_, vv = q.view(-1, H, D), k.view(-1, Hk, D), v.view(-1, Hk, D)
            for head_select in (True, False):
                arrs = selection_arrays(plan, head_select, Hk, dev)
                if arrs is None:
                    continue
                desc, slots, max_klen, idx_total = arrs
                top_idx = None
                if self.record_selection:
                    top_idx = torch.empty(idx_total, dtype=torch.int64, device=dev)
                    self.last_selection[head_select] = top_idx
                ops.select_kv_store(qv, kv_, vv, desc, max_klen, head_select,
                                    self.k_cache, self.v_cache, slots, top_idx)
        return res

    def _paged_cache_args(self):
        """Validated pointer/size arguments of the bound paged cache, recomputed
        only when the k_cache / v_cache tensors or their storage change."""
        kc, vc = self.k_cache, self.v_cache
        cs = self._cache_sig
        if cs is None or cs[0] is not kc or cs[1] is not vc or cs[2] != kc.data_ptr():
            self._cache_sig = cs = (kc, vc, kc.data_ptr(),
                                    ops.paged_cache_args(kc, vc, self.num_kv_heads, self.head_dim))
        return cs[3]
