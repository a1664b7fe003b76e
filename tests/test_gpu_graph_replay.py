"""CUDA-graph replay of whole diffusion steps through the public Attention
layer: a compute-cache step (state 1: attention + selection + cache store)
and a reuse step (state 2: block queries over the paged cache + fresh keys),
each captured once and replayed twice from a zeroed cache, must write the
same output, cache rows and top_idx bits as the eager steps, and agree with
the CPU oracle within the attention tolerance.

The captured launches use the capture stream's scheduler workspace (dynamic
unit order), which the eager warm-up on that stream creates first.
"""
import pytest
import torch

import inputs as I
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu

D = 128
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


@pytest.mark.parametrize("head_select", [True, False])
def test_graph_replay_equals_eager_and_oracle(head_select):
    from dllmserve_b200 import ops
    from dllmserve_b200.layers.attention import Attention
    from dllmserve_b200.sparse.state import PerRequestSparseState, SparseConfig
    from dllmserve_b200.utils.context import Context, reset_context, use_context

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    H, Hk = 16, 4 if head_select else 16
    cfg = SparseConfig(enabled=True, retention_ratio=0.5, head_select=head_select)

    class Seq:
        def __init__(self, prompt, gen, sparse):
            self.num_prompt_tokens = prompt
            self.num_tokens = prompt + gen
            self.sparse_state = PerRequestSparseState(0, cfg, dev) if sparse else None

    specs = [(700, 128, True), (300, 64, True), (129, 32, False), (1000, 128, True), (57, 32, True)]
    seqs = [Seq(p, gn, sp) for p, gn, sp in specs]
    metas = [R.SeqMeta(1 if sp else 0, p + gn, p, head_select=head_select) for p, gn, sp in specs]
    # slots: consecutive runs inside pages, pages handed out in reverse order
    pages = sum((m.n_keep() + 255) // 256 for m in metas if m.state) + 2
    slots, nxt = [], pages - 1
    for m in metas:
        if not m.state:
            slots.append(torch.zeros(0, dtype=torch.int32))
            continue
        n, lst = m.n_keep(), []
        for j in range((n + 255) // 256):
            lst.extend(range(nxt * 256, nxt * 256 + min(256, n - j * 256)))
            nxt -= 1
        slots.append(torch.tensor(lst, dtype=torch.int32))
    layer = Attention(H, D, D ** -0.5, Hk, causal=False)
    layer.k_cache = torch.zeros(pages, 256, Hk, D, dtype=torch.bfloat16, device=dev)
    layer.v_cache = torch.zeros_like(layer.k_cache)
    layer.record_selection = True
    g = I.gen(900 + head_select)

    def inputs(step_metas):
        n = sum(m.rows() for m in step_metas)
        return [I.grid(g, (n, h, D)) for h in (H, Hk, Hk)]

    def make_ctx():
        return Context(is_prefill=True, is_diffusion=True, seqs=seqs,
                       slot_mapping=[sl.to(dev) if s.sparse_state is not None else []
                                     for s, sl in zip(seqs, slots)])

    side = torch.cuda.Stream(dev)
    steps = {}
    kc_ref = torch.zeros(pages, 256, Hk, D)
    vc_ref = torch.zeros_like(kc_ref)
    for state in (1, 2):
        for s, m in zip(seqs, metas):
            if s.sparse_state is not None:
                s.sparse_state.cache_state = state
                m.state = state
        qh, kh, vh = inputs(metas)
        ref = R.diffusion_layer(qh, kh, vh, metas, kc_ref, vc_ref, slots, D ** -0.5, H, Hk)
        q, k, v = (t.to(dev, torch.bfloat16).reshape(t.shape[0], -1) for t in (qh, kh, vh))
        ctx = make_ctx()
        # eager run on the capture stream (plan built and cached on ctx, the
        # stream's scheduler workspace created outside the capture)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            use_context(ctx)
            eager = layer(q, k, v).clone()
            reset_context()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        eager_sel = {hs: t.clone() for hs, t in layer.last_selection.items()}
        graph = torch.cuda.CUDAGraph()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            use_context(ctx)
            with torch.cuda.graph(graph, stream=side):
                captured = layer(q, k, v)
            reset_context()
        torch.cuda.current_stream().wait_stream(side)
        captured_sel = dict(layer.last_selection)
        # the graph reads q/k/v and the step metadata cached on ctx by address:
        # keep them alive with the graph
        steps[state] = (graph, captured, captured_sel, eager, eager_sel, ref, (q, k, v, ctx))
        err = (eager.float().cpu().view(ref.shape) - ref).abs()
        assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (state, float(err.max()), float(err.mean()))
    eager_cache = (layer.k_cache.clone(), layer.v_cache.clone())
    all_slots = torch.cat([sl for sl, m in zip(slots, metas) if m.state]).long()
    rows = Hk * D
    assert torch.equal(layer.k_cache.view(-1, rows)[all_slots.to(dev)].float().cpu(),
                       kc_ref.view(-1, rows)[all_slots])

    for rep in range(2):
        layer.k_cache.zero_()
        layer.v_cache.zero_()
        for state in (1, 2):
            graph, captured, captured_sel, eager, eager_sel, _, _ = steps[state]
            captured.fill_(float("nan"))
            for t in captured_sel.values():
                t.fill_(-1)
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(captured, eager), (rep, state)
            assert captured_sel.keys() == eager_sel.keys()
            for hs in eager_sel:
                assert torch.equal(captured_sel[hs], eager_sel[hs]), (rep, state, hs)
        assert torch.equal(layer.k_cache, eager_cache[0]) and torch.equal(layer.v_cache, eager_cache[1])
    assert ops.read_device_status(dev) == 0
