"""Generate the golden vectors under tests/golden/ by running the REFERENCE's
own attention module (dllmserve.layers.attention of chosen-ox/dLLM-Serve) on
CPU in fp32.

Run in a container that has the reference source:
    python tests/golden/make_golden.py --reference /path/to/dLLM-Serve

The reference's GPU-only pieces are replaced in its module namespace:
  * flash_attn_varlen_func -> per-sequence fp32 F.scaled_dot_product_attention
    (non-causal, GQA by repeat_interleave)
  * store_kvcache / load_kvcache (Triton) -> exact index copies
Everything else (the per-sequence dispatcher, _select_important_head_kv,
_select_important_kv, max-pool, torch.topk, the sparse state machine and
Sequence sizing) is the reference's unmodified code. torch.topk results are
recorded through a thin proxy of the module's ``torch`` global.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import types

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import cases as C  # noqa: E402
import inputs as I  # noqa: E402
from oracle import reference_module as RM  # noqa: E402


class _TorchProxy:
    def __init__(self, real, log):
        self._real = real
        self._log = log

    def __getattr__(self, name):
        return getattr(self._real, name)

    def topk(self, *a, **kw):
        r = self._real.topk(*a, **kw)
        self._log.append(r.indices.clone())
        return r


def load_reference(path):
    """The reference's attention module with CPU stand-ins for its flash-attn
    and Triton callees (oracle/reference_module.py)."""
    return RM.load(path)


def _fake_config():
    return types.SimpleNamespace(model_type=None, torch_device=torch.device("cpu"),
                                 hf_config=types.SimpleNamespace(mask_token_id=0))


def _run_layer(R, layer, q, k, v, seqs, slots):
    cu = [0]
    for s in seqs:
        st = s.sparse_state
        if st is not None and st.should_reuse_cache:
            cu.append(cu[-1] + st.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)[1])
        else:
            cu.append(cu[-1] + s.num_tokens)
    R.ctx.set_context(is_prefill=True, cu_seqlens_k=torch.tensor(cu, dtype=torch.int32),
                      is_diffusion=True, seqs=seqs, slot_mapping=slots)
    H, Hk, Dh = layer.num_heads, layer.num_kv_heads, layer.head_dim
    out = layer(q.reshape(-1, H * Dh), k.reshape(-1, Hk * Dh), v.reshape(-1, Hk * Dh))
    R.ctx.reset_context()
    return out.view(-1, H, Dh), cu


def make_sparse_case(R, case: C.SparseCase):
    g = I.gen(case.seed)
    H, Hk, Dh = case.num_heads, case.num_kv_heads, case.head_dim
    cfg = R.SparseConfig(enabled=True, default_block_len=case.block_len,
                         retention_ratio=case.retention_ratio, pool_kernel=case.pool_kernel,
                         delay_step=1, head_select=case.head_select)
    seqs = []
    for sp in case.seqs:
        params = types.SimpleNamespace(gen_length=sp.gen_len)
        s = R.Sequence([1] * sp.prompt_len, params, _fake_config(), cfg if sp.sparse else None)
        if s.sparse_state is not None:
            s.sparse_state.current_block_idx = sp.block_idx
            s.sparse_state.cache_state = 1
        seqs.append(s)
    page_order = torch.randperm(case.num_pages, generator=g).tolist()
    slots, next_page = [], 0
    for s in seqs:
        if s.sparse_state is None:
            slots.append([])
            continue
        n = s.current_sparse_token
        npg = (n + 255) // 256
        pages = page_order[next_page:next_page + npg]
        next_page += npg
        lst = []
        for j, p in enumerate(pages):
            lst.extend(range(p * 256, p * 256 + min(256, n - j * 256)))
        slots.append(torch.tensor(lst, dtype=torch.int32))
    layer = R.att.Attention(H, Dh, Dh ** -0.5, Hk, causal=False)
    layer.k_cache = torch.zeros(case.num_pages, 256, Hk, Dh)
    layer.v_cache = torch.zeros(case.num_pages, 256, Hk, Dh)
    log = []
    R.att.torch = _TorchProxy(torch, log)
    try:
        N1 = sum(s.num_tokens for s in seqs)
        q1, k1, v1 = (I.make(case.kind, g, (N1, h, Dh)) for h in (H, Hk, Hk))
        out1, cu1 = _run_layer(R, layer, q1, k1, v1, seqs, slots)
        kc1, vc1 = layer.k_cache.clone(), layer.v_cache.clone()
        for s in seqs:
            if s.sparse_state is not None:
                s.sparse_state.cache_state = 2
        N2 = sum(s.sparse_state.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)[1]
                 if s.sparse_state is not None else s.num_tokens for s in seqs)
        q2, k2, v2 = (I.make(case.kind, g, (N2, h, Dh)) for h in (H, Hk, Hk))
        out2, cu2 = _run_layer(R, layer, q2, k2, v2, seqs, slots)
    finally:
        R.att.torch = torch
    all_slots = torch.cat([s for s in slots if isinstance(s, torch.Tensor)] or
                          [torch.zeros(0, dtype=torch.int32)])
    rows = Hk * Dh
    res = {
        "out1": out1.numpy().astype(np.float16), "out2": out2.numpy().astype(np.float16),
        "cu1": np.array(cu1, np.int32), "cu2": np.array(cu2, np.int32),
        "all_slots": all_slots.numpy(),
        "kcache_rows": kc1.view(-1, rows)[all_slots.long()].numpy().astype(np.float16),
        "vcache_rows": vc1.view(-1, rows)[all_slots.long()].numpy().astype(np.float16),
        "cache_abs_sum": np.array([float(kc1.abs().sum()), float(vc1.abs().sum())]),
        "input_checksums": np.array(I.checksum(q1) + I.checksum(k1) + I.checksum(q2) + I.checksum(v2)),
    }
    sel = [i for i, s in enumerate(seqs) if s.sparse_state is not None]
    calls = [i for i in sel if (seqs[i].num_tokens - seqs[i].sparse_state.compute_block_boundaries(
        seqs[i].num_prompt_tokens, seqs[i].num_tokens)[1]) > 0 or not case.head_select]
    assert len(calls) == len(log), (len(calls), len(log))
    for i, idx in zip(calls, log):
        res[f"top_idx_{i}"] = idx.numpy().astype(np.int64)
    meta = {"slots": {str(i): (s.tolist() if isinstance(s, torch.Tensor) else []) for i, s in enumerate(slots)},
            "n_keep": [s.current_sparse_token for s in seqs]}
    return res, meta


def make_selection_case(R, case: C.SelectionCase):
    """One compute-cache (state 1) step of the reference's Attention.forward
    on a SelectionCase batch (inputs.margin_selection_batch); records the
    reference's top_idx of every sequence (its torch.topk indices)."""
    H, Hk, Dh, blk = case.num_heads, case.num_kv_heads, 128, case.block_len
    q, k, v, prompts, lens = I.margin_selection_batch(case)
    cfg = R.SparseConfig(enabled=True, default_block_len=blk, retention_ratio=case.retention_ratio,
                         pool_kernel=case.pool_kernel, delay_step=1, head_select=case.head_select)
    seqs, slots, page = [], [], 0
    for p in prompts:
        s = R.Sequence([1] * p, types.SimpleNamespace(gen_length=case.gen_len), _fake_config(), cfg)
        s.sparse_state.current_block_idx = 0
        s.sparse_state.cache_state = 1
        n = s.current_sparse_token
        npg = (n + 255) // 256
        slots.append(torch.arange(page * 256, page * 256 + n, dtype=torch.int32))
        page += npg
        seqs.append(s)
    layer = R.att.Attention(H, Dh, Dh ** -0.5, Hk, causal=False)
    layer.k_cache = torch.zeros(page, 256, Hk, Dh)
    layer.v_cache = torch.zeros(page, 256, Hk, Dh)
    log = []
    R.att.torch = _TorchProxy(torch, log)
    try:
        _run_layer(R, layer, q, k, v, seqs, slots)
    finally:
        R.att.torch = torch
    assert len(log) == len(seqs), (len(log), len(seqs))
    res = {"input_checksums": np.array(I.checksum(q) + I.checksum(k) + I.checksum(v)),
           "lens": np.array(lens, np.int32),
           "n_keep": np.array([s.current_sparse_token for s in seqs], np.int32)}
    for i, idx in enumerate(log):
        res[f"top_idx_{i}"] = idx.numpy().astype(np.int16)
    return res


def make_c1(R):
    c = C.C1
    g = I.gen(c["seed"])
    L = c["prompt_len"] + c["gen_len"]
    H, Dh = c["num_heads"], c["head_dim"]
    q = torch.randn((L, H, Dh), generator=g)
    k = torch.randn((L, H, Dh), generator=g)
    v = torch.randn((L, H, Dh), generator=g)
    rope = R.RotaryEmbedding(Dh, Dh, L, c["rope_theta"])
    pos = torch.arange(L)
    cos, sin = rope.cos_sin_cache[pos].chunk(2, dim=-1)
    qr = R.apply_rotary_emb(q, cos, sin)
    kr = R.apply_rotary_emb(k, cos, sin)
    seq = R.Sequence([1] * c["prompt_len"], types.SimpleNamespace(gen_length=c["gen_len"]),
                     _fake_config(), None)
    layer = R.att.Attention(H, Dh, Dh ** -0.5, H, causal=False)
    out, _ = _run_layer(R, layer, qr, kr, v, [seq], [[]])
    sdpa = F.scaled_dot_product_attention(qr.transpose(0, 1), kr.transpose(0, 1), v.transpose(0, 1),
                                          scale=Dh ** -0.5).transpose(0, 1)
    assert torch.allclose(out, sdpa, atol=1e-5), float((out - sdpa).abs().max())
    return {"out": out.numpy().astype(np.float16),
            "input_checksums": np.array(I.checksum(q) + I.checksum(k) + I.checksum(v)),
            "rope_checksums": np.array(I.checksum(qr) + I.checksum(kr))}


def make_state_traces(R):
    out = []
    for delay, blen, prompt, gen_len, n in C.STATE_TRACES:
        cfg = R.SparseConfig(enabled=True, default_block_len=blen, delay_step=delay)
        seq = R.Sequence([1] * prompt, types.SimpleNamespace(gen_length=gen_len), _fake_config(), cfg)
        st = seq.sparse_state
        rows = []
        for _ in range(n):
            bs, bl = st.compute_block_boundaries(seq.num_prompt_tokens, seq.num_tokens)
            rows.append([st.cache_state, st.current_block_idx, st.step_in_block, bs, bl,
                         seq.current_sparse_token])
            st.advance_step()
        out.append(rows)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    R = load_reference(args.reference)
    meta = {"torch": torch.__version__, "cases": {}}
    np.savez_compressed(os.path.join(HERE, "c1.npz"), **make_c1(R))
    for case in C.SELECTION_CASES:
        np.savez_compressed(os.path.join(HERE, f"selection_{case.name}.npz"), **make_selection_case(R, case))
    for case in C.SPARSE_CASES:
        res, m = make_sparse_case(R, case)
        np.savez_compressed(os.path.join(HERE, f"sparse_{case.name}.npz"), **res)
        meta["cases"][case.name] = m
    meta["state_traces"] = make_state_traces(R)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
