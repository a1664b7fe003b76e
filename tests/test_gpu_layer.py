"""The drop-in Attention layer on the GPU, driven like the reference's model
runner drives it, against the golden vectors and the oracle."""
import json
import os

import numpy as np
import pytest
import torch

import cases as C
import inputs as I
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


class Seq:
    """What the layer reads from a model runner's Sequence."""

    def __init__(self, prompt_len, gen_len, sparse_state):
        self.num_prompt_tokens = prompt_len
        self.num_tokens = prompt_len + gen_len
        self.sparse_state = sparse_state


def _run(case, golden_dir, dev):
    from dllmserve_b200 import ops
    from dllmserve_b200.layers.attention import Attention
    from dllmserve_b200.sparse.state import PerRequestSparseState, SparseConfig
    from dllmserve_b200.utils.context import reset_context, set_context

    meta = json.load(open(os.path.join(golden_dir, "golden_meta.json")))["cases"][case.name]
    gold = np.load(os.path.join(golden_dir, f"sparse_{case.name}.npz"))
    H, Hk, D = case.num_heads, case.num_kv_heads, case.head_dim
    cfg = SparseConfig(enabled=True, default_block_len=case.block_len,
                       retention_ratio=case.retention_ratio, pool_kernel=case.pool_kernel,
                       delay_step=1, head_select=case.head_select)
    seqs = []
    for sp in case.seqs:
        st = PerRequestSparseState(0, cfg, dev) if sp.sparse else None
        if st is not None:
            st.current_block_idx = sp.block_idx
            st.cache_state = 1
        seqs.append(Seq(sp.prompt_len, sp.gen_len, st))
    slots = [torch.tensor(meta["slots"][str(i)], dtype=torch.int32) for i in range(len(seqs))]
    layer = Attention(H, D, D ** -0.5, Hk, causal=False)
    layer.k_cache = torch.zeros(case.num_pages, 256, Hk, D, dtype=torch.bfloat16, device=dev)
    layer.v_cache = torch.zeros_like(layer.k_cache)
    layer.record_selection = True
    kc = torch.zeros(case.num_pages, 256, Hk, D)
    vc = torch.zeros(case.num_pages, 256, Hk, D)

    g = I.gen(case.seed)
    torch.randperm(case.num_pages, generator=g)
    metas = [R.SeqMeta(1 if sp.sparse else 0, sp.prompt_len + sp.gen_len, sp.prompt_len,
                       sp.block_idx, case.block_len, case.retention_ratio, case.pool_kernel,
                       case.head_select) for sp in case.seqs]
    results = {}
    for step in (1, 2):
        n = sum(m.rows() for m in metas)
        q, k, v = (I.make(case.kind, g, (n, h, D)) for h in (H, Hk, Hk))
        rec = {}
        ref = R.diffusion_layer(q, k, v, metas, kc, vc, slots, D ** -0.5, H, Hk, record=rec)
        set_context(True, is_diffusion=True, seqs=seqs,
                    slot_mapping=[s.to(dev) if s.numel() else [] for s in slots])
        out = layer(*(t.to(dev, torch.bfloat16).reshape(n, -1) for t in (q, k, v)))
        torch.cuda.synchronize()
        reset_context()
        assert ops.read_device_status(dev) == 0
        out = out.view(n, H, D).float().cpu()
        err = (out - ref).abs()
        assert err.max() <= 2e-2 and err.mean() <= 2e-3, (step, float(err.max()), float(err.mean()))
        results[step] = (out, rec, dict(layer.last_selection))
        for s, m in zip(seqs, metas):
            if s.sparse_state is not None:
                s.sparse_state.cache_state = 2
                m.state = 2
    return layer, kc, vc, gold, results, metas


@pytest.fixture(scope="module")
def dev():
    d = torch.device("cuda:0")
    torch.cuda.set_device(d)
    return d


@pytest.mark.parametrize("case", C.SPARSE_CASES, ids=[c.name for c in C.SPARSE_CASES])
def test_layer_two_steps_vs_oracle_and_golden(case, golden_dir, dev):
    layer, kc, vc, gold, results, metas = _run(case, golden_dir, dev)
    Hk, D = case.num_kv_heads, case.head_dim
    # cache contents: bit-exact vs the oracle (same tie rule)
    assert torch.equal(layer.k_cache.float().cpu(), kc)
    assert torch.equal(layer.v_cache.float().cpu(), vc)
    # selected indices: bit-exact vs the oracle's, in the oracle's layout
    out1, rec, sel = results[1]
    flat = sel.get(case.head_select)
    pos = 0
    for i, m in enumerate(metas):
        if i in rec:
            n = rec[i].size
            got = flat[pos:pos + n].cpu().numpy().reshape(rec[i].shape)
            assert np.array_equal(got, rec[i]), i
            pos += n
    # step-1 outputs vs the reference's golden output (independent of ties)
    err = (out1 - torch.from_numpy(gold["out1"].astype(np.float32))).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3


def test_layer_dense_c1_vs_golden(golden_dir, dev):
    """Config 1 (64+32 tokens, 32 heads, RoPE) through the layer, bf16."""
    from dllmserve_b200.layers.attention import Attention
    from dllmserve_b200.utils.context import reset_context, set_context

    c = C.C1
    gold = np.load(os.path.join(golden_dir, "c1.npz"))
    L = c["prompt_len"] + c["gen_len"]
    H, D = c["num_heads"], c["head_dim"]
    g = I.gen(c["seed"])
    q, k, v = (torch.randn((L, H, D), generator=g) for _ in range(3))
    cache = R.rope_cache(D, L, c["rope_theta"])
    pos = torch.arange(L)
    qr, kr = R.apply_rope(q, pos, cache), R.apply_rope(k, pos, cache)
    layer = Attention(H, D, D ** -0.5, H, causal=False)
    set_context(True, is_diffusion=True, seqs=[Seq(c["prompt_len"], c["gen_len"], None)],
                slot_mapping=[[]])
    out = layer(*(t.to(dev, torch.bfloat16).reshape(L, -1) for t in (qr, kr, v)))
    reset_context()
    err = (out.view(L, H, D).float().cpu() - torch.from_numpy(gold["out"].astype(np.float32))).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3
