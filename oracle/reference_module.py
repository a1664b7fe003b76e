"""Loads the REFERENCE's own attention module (``dllmserve.layers.attention``
of chosen-ox/dLLM-Serve) and makes it runnable on CPU. TEST INFRASTRUCTURE
ONLY (see oracle/__init__.py): used by tests/golden/make_golden.py to record
golden vectors and by bench.py's ``--impl reference`` arm to time the
reference's CPU path.

The reference's GPU-only callees are replaced in its module namespace by
CPU stand-ins; everything else (the per-sequence dispatcher
``_mixed_sparse_dense_attention``, attention.py:150-306, the selection
functions, max-pool, torch.topk, the sparse state machine) is the
reference's unmodified code:
  * ``flash_attn_varlen_func`` (third-party flash-attn 2.x, call site
    attention.py:289-299, causal=False) -> per-sequence fp32
    ``F.scaled_dot_product_attention`` (GQA by repeat_interleave)
  * ``store_kvcache`` / ``load_kvcache`` (Triton kernels, attention.py:11-92)
    -> exact index copies
"""
from __future__ import annotations

import os
import sys
import types

import torch
import torch.nn.functional as F


def flash_varlen_cpu(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q=0, max_seqlen_k=0,
                     softmax_scale=None, causal=False, **_):
    """flash_attn_varlen_func(..., causal=False) semantics: softmax(q k^T *
    softmax_scale) v per sequence, computed in fp32."""
    assert not causal
    out = torch.zeros(q.shape, dtype=torch.float32)
    cq, ck = cu_seqlens_q.tolist(), cu_seqlens_k.tolist()
    for b in range(len(cq) - 1):
        qs, ks, vs = q[cq[b]:cq[b + 1]], k[ck[b]:ck[b + 1]], v[ck[b]:ck[b + 1]]
        if qs.shape[0] == 0:
            continue
        rep = qs.shape[1] // ks.shape[1]
        ks, vs = ks.repeat_interleave(rep, 1), vs.repeat_interleave(rep, 1)
        o = F.scaled_dot_product_attention(qs.transpose(0, 1).float(), ks.transpose(0, 1).float(),
                                           vs.transpose(0, 1).float(), scale=softmax_scale)
        out[cq[b]:cq[b + 1]] = o.transpose(0, 1)
    return out


def store_rows_cpu(key, value, k_cache, v_cache, slot_mapping):
    """store_kvcache: cache row slot_mapping[i] <- key[i], value[i]."""
    N, H, Dh = key.shape
    assert slot_mapping.numel() == N
    k_cache.view(-1, H * Dh)[slot_mapping.long()] = key.reshape(N, -1)
    v_cache.view(-1, H * Dh)[slot_mapping.long()] = value.reshape(N, -1)


def load_rows_cpu(key, value, k_cache, v_cache, slot_mapping):
    """load_kvcache: key[i], value[i] <- cache row slot_mapping[i]."""
    N, H, Dh = key.shape
    assert slot_mapping.numel() == N
    key.copy_(k_cache.view(-1, H * Dh)[slot_mapping.long()].view(N, H, Dh))
    value.copy_(v_cache.view(-1, H * Dh)[slot_mapping.long()].view(N, H, Dh))


def default_paths():
    """Where the reference package may be found: an install under
    baseline/_ref of this repository (it travels with the repository), then
    a source checkout named by DLLM_REFERENCE."""
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    paths = [os.path.join(repo, "baseline", "_ref")]
    if os.environ.get("DLLM_REFERENCE"):
        paths.append(os.environ["DLLM_REFERENCE"])
    return paths


def load(path: str | None = None):
    """Imports the reference package from ``path`` (or the first of
    default_paths() that holds it), installs the CPU stand-ins and returns a
    namespace with the modules the harnesses use. Raises ImportError when no
    reference package is found."""
    cands = [path] if path else default_paths()
    for p in cands:
        if p and os.path.isdir(os.path.join(p, "dllmserve")):
            if p not in sys.path:
                sys.path.insert(0, p)
            break
    else:
        raise ImportError("reference package dllmserve not found in " + ", ".join(map(str, cands)))
    import dllmserve.layers.attention as att
    import dllmserve.utils.context as ctx
    from dllmserve.engine.sequence import Sequence
    from dllmserve.layers.rotary_embedding import RotaryEmbedding, apply_rotary_emb
    from dllmserve.sparse.state import SparseConfig

    att.flash_attn_varlen_func = flash_varlen_cpu
    att.store_kvcache = store_rows_cpu
    att.load_kvcache = load_rows_cpu
    return types.SimpleNamespace(att=att, ctx=ctx, Sequence=Sequence, SparseConfig=SparseConfig,
                                 RotaryEmbedding=RotaryEmbedding, apply_rotary_emb=apply_rotary_emb,
                                 path=os.path.dirname(os.path.dirname(os.path.dirname(att.__file__))))


class _DenseSeq:
    """A dense sequence as the model runner hands it to the layer (no
    sparse state: attention.py:171)."""

    sparse_state = None

    def __init__(self, L):
        self.num_tokens = L
        self.num_prompt_tokens = L


def dense_layer_forward(R, q, k, v, lens, num_heads, num_kv_heads, head_dim, scale):
    """One dense diffusion step of one layer through the reference's
    ``Attention.forward`` (attention.py:107-119 -> 150-306) on CPU.
    q [N, Hq, D], k/v [N, Hkv, D] fp32; returns [N, Hq*D]."""
    layer = R.att.Attention(num_heads, head_dim, scale, num_kv_heads, causal=False)
    cu = [0]
    for L in lens:
        cu.append(cu[-1] + L)
    R.ctx.set_context(is_prefill=True, cu_seqlens_k=torch.tensor(cu, dtype=torch.int32),
                      is_diffusion=True, seqs=[_DenseSeq(L) for L in lens],
                      slot_mapping=[[] for _ in lens])
    try:
        return layer(q.reshape(q.shape[0], -1), k.reshape(k.shape[0], -1), v.reshape(v.shape[0], -1))
    finally:
        R.ctx.reset_context()


class SparseLayerCycle:
    """One layer of the reference's ``Attention`` driven through a diffusion
    block of head-sparse sequences on CPU, as the model runner drives it
    (model_runner.py:240-321 builds the Context; attention.py:168-304
    dispatches per sequence): every sequence at block 0 of its generation,
    state 1 (compute cache: attention over the whole sequence, then
    _select_important_head_kv / _select_important_kv and store_kvcache of the
    selected rows, attention.py:204-233) and state 2 (reuse: the block's rows
    attend to the cached selection plus the block, attention.py:235-265).

    Inputs are fp32 [tokens, heads, head_dim]; state-1 inputs cover whole
    sequences, state-2 inputs the blocks only (``rows(state)`` gives the
    count)."""

    def __init__(self, R, prompts, gen_len, num_heads, num_kv_heads, head_dim, retention_ratio,
                 head_select, block_len=32, pool_kernel=3):
        self.R = R
        cfg = R.SparseConfig(enabled=True, default_block_len=block_len, retention_ratio=retention_ratio,
                             pool_kernel=pool_kernel, delay_step=1, head_select=head_select)
        cfg_model = types.SimpleNamespace(model_type=None, torch_device=torch.device("cpu"),
                                          hf_config=types.SimpleNamespace(mask_token_id=0))
        self.seqs, self.slots, page = [], [], 0
        for p in prompts:
            s = R.Sequence([1] * p, types.SimpleNamespace(gen_length=gen_len), cfg_model, cfg)
            s.sparse_state.current_block_idx = 0
            s.sparse_state.cache_state = 1
            n = s.current_sparse_token
            self.slots.append(torch.arange(page * 256, page * 256 + n, dtype=torch.int32))
            page += (n + 255) // 256
            self.seqs.append(s)
        self.layer = R.att.Attention(num_heads, head_dim, head_dim ** -0.5, num_kv_heads, causal=False)
        self.layer.k_cache = torch.zeros(max(page, 1), 256, num_kv_heads, head_dim)
        self.layer.v_cache = torch.zeros(max(page, 1), 256, num_kv_heads, head_dim)
        self.n_keep = [s.current_sparse_token for s in self.seqs]

    def rows(self, state):
        if state == 1:
            return sum(s.num_tokens for s in self.seqs)
        return sum(s.sparse_state.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)[1]
                   for s in self.seqs)

    def forward(self, state, q, k, v):
        for s in self.seqs:
            s.sparse_state.cache_state = state
        cu = [0]
        for s in self.seqs:
            n = (s.num_tokens if state == 1 else
                 s.sparse_state.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)[1])
            cu.append(cu[-1] + n)
        self.R.ctx.set_context(is_prefill=True, cu_seqlens_k=torch.tensor(cu, dtype=torch.int32),
                               is_diffusion=True, seqs=self.seqs, slot_mapping=self.slots)
        try:
            return self.layer(q.reshape(q.shape[0], -1), k.reshape(k.shape[0], -1), v.reshape(v.shape[0], -1))
        finally:
            self.R.ctx.reset_context()
