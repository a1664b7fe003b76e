"""integration.install() against the REAL reference package (dllmserve,
installed under baseline/_ref; skipped when absent): a reference LLaDA
decoder layer (dllmserve/models/llada.py:13-95) built after install() runs
its attention through this package's Attention and RotaryEmbedding, driven by
the reference's own Context (dllmserve.utils.context.set_context, as
ModelRunner._run_diffusion sets it, model_runner.py:310-321) and its own
Sequence / PerRequestSparseState objects, over two consecutive diffusion
steps (state 1: attention + select + cache store; state 2: block queries over
the cache).

Checked: the patched layer's attention output against the CPU oracle on the
exact q/k/v the layer produced, both steps; the rotary embedding applied to
them against the oracle bit for bit; the whole decoder layer (RMSNorm,
projections, RoPE, attention, MLP) against the unpatched reference layer run
on the CPU in fp32 with the same weights (state 1, where both attend over
every token), within bf16 tolerance.
"""
import sys
import types

import pytest
import torch

from oracle import attention_ref as R
from oracle import reference_module as RM

pytestmark = pytest.mark.gpu

D = 128


def _reference_path():
    for p in RM.default_paths():
        import os

        if os.path.isdir(os.path.join(p, "dllmserve")):
            return p
    return None


@pytest.fixture
def ref_pkg():
    path = _reference_path()
    if path is None:
        pytest.skip("reference package dllmserve not installed under baseline/_ref")
    import torch._dynamo

    old = torch._dynamo.config.disable
    torch._dynamo.config.disable = True  # the reference's torch.compile'd norms run eagerly
    ns = RM.load(path)
    import dllmserve.models.llada as llada

    ns.llada = llada
    yield ns
    torch._dynamo.config.disable = old


def test_install_drives_reference_decoder_layer(ref_pkg):
    from dllmserve_b200 import integration, ops

    Rf = ref_pkg
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = types.SimpleNamespace(d_model=512, n_heads=4, n_kv_heads=4, mlp_hidden_size=1024,
                                rms_norm_eps=1e-5, max_sequence_length=2048, rope_theta=500000.0)
    H = cfg.n_heads
    torch.manual_seed(0)
    ref_layer = Rf.llada.LLaDADecoderLayer(cfg)            # the reference's own attention (CPU stand-ins)
    with torch.no_grad():
        for p in ref_layer.parameters():
            if p.dim() == 2:
                p.normal_(0, 0.02)
    assert type(ref_layer.attn).__module__ == "dllmserve.layers.attention"

    sc = Rf.SparseConfig(enabled=True, default_block_len=32, retention_ratio=0.5, pool_kernel=3,
                         delay_step=1, head_select=True)
    fake_cfg = types.SimpleNamespace(model_type=None, torch_device=torch.device("cpu"),
                                     hf_config=types.SimpleNamespace(mask_token_id=0))
    specs = [(200, 64, True), (150, 32, False), (90, 32, True)]
    seqs = [Rf.Sequence([1] * p, types.SimpleNamespace(gen_length=gn), fake_cfg, sc if sp else None)
            for p, gn, sp in specs]
    pages = 4
    slot_lists, page = [], 0
    for s in seqs:
        if s.sparse_state is None:
            slot_lists.append([])
            continue
        s.sparse_state.cache_state = 1
        n = s.current_sparse_token
        slot_lists.append(torch.arange(page * 256, page * 256 + n, dtype=torch.int32))
        page += 1

    def step_rows():
        positions, cu = [], [0]
        for s in seqs:
            st = s.sparse_state
            if st is not None and st.should_reuse_cache:
                b0, bl = st.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)
                positions.append(torch.arange(b0, b0 + bl))
            else:
                positions.append(torch.arange(s.num_tokens))
            cu.append(cu[-1] + positions[-1].numel())
        return torch.cat(positions), cu

    g = torch.Generator().manual_seed(3)
    pos1, cu1 = step_rows()
    xs = {1: torch.randn(pos1.numel(), cfg.d_model, generator=g)}
    # the unpatched reference layer on the CPU (fp32), compute-cache step
    Rf.ctx.set_context(is_prefill=True, cu_seqlens_k=torch.tensor(cu1, dtype=torch.int32),
                       is_diffusion=True, seqs=seqs, slot_mapping=slot_lists)
    ref_layer.attn.k_cache = torch.zeros(pages, 256, H, D)
    ref_layer.attn.v_cache = torch.zeros_like(ref_layer.attn.k_cache)
    with torch.no_grad():
        y_ref1 = ref_layer(pos1, xs[1])
    Rf.ctx.reset_context()

    patched = integration.install()
    try:
        assert "dllmserve.models.llada" in patched
        layer = Rf.llada.LLaDADecoderLayer(cfg)
        from dllmserve_b200.layers.attention import Attention as OurAttention
        from dllmserve_b200.layers.rotary_embedding import RotaryEmbedding as OurRope

        assert isinstance(layer.attn, OurAttention) and isinstance(layer.rotary_emb, OurRope)
        layer.load_state_dict(ref_layer.state_dict(), strict=False)
        layer = layer.to(dev, torch.bfloat16)
        layer.rotary_emb.cos_sin_cache = ref_layer.rotary_emb.cos_sin_cache.to(dev)
        layer.attn.k_cache = torch.zeros(pages, 256, H, D, dtype=torch.bfloat16, device=dev)
        layer.attn.v_cache = torch.zeros_like(layer.attn.k_cache)
        kc_ref = torch.zeros(pages, 256, H, D)
        vc_ref = torch.zeros_like(kc_ref)

        seen = {}

        def hook(mod, args, out):
            seen["qkv"] = [a.detach().float().cpu() for a in args]
            seen["out"] = out.detach().float().cpu()

        handle = layer.attn.register_forward_hook(hook)
        for step in (1, 2):
            pos, cu = step_rows()
            x = xs[step] if step in xs else torch.randn(pos.numel(), cfg.d_model, generator=g)
            Rf.ctx.set_context(is_prefill=True, cu_seqlens_k=torch.tensor(cu, dtype=torch.int32).to(dev),
                               is_diffusion=True, seqs=seqs,
                               slot_mapping=[sl.to(dev) if isinstance(sl, torch.Tensor) else [] for sl in slot_lists])
            with torch.no_grad():
                y = layer(pos.to(dev), x.to(dev, torch.bfloat16))
            torch.cuda.synchronize()
            Rf.ctx.reset_context()
            assert torch.isfinite(y.float()).all()
            q, k, v = (t.view(t.shape[0], -1, D) for t in seen["qkv"])
            # RoPE through the patched get_rope: bit-exact against the oracle
            with torch.no_grad():
                xn = layer.attn_norm(x.to(dev, torch.bfloat16))
                q0 = layer.q_proj(xn).view(-1, H, D).cpu()
                k0 = layer.k_proj(xn).view(-1, H, D).cpu()
            cache = layer.rotary_emb.cos_sin_cache.cpu()
            assert torch.equal(R.apply_rope(q0, pos, cache).float(), q)
            assert torch.equal(R.apply_rope(k0, pos, cache).float(), k)
            # attention output against the oracle on the layer's own q/k/v
            metas = []
            for s in seqs:
                st = s.sparse_state
                state = 0 if st is None else (1 if st.should_compute_cache else 2)
                metas.append(R.SeqMeta(state, s.num_tokens, s.num_prompt_tokens, head_select=True))
            ref = R.diffusion_layer(q, k, v, metas, kc_ref, vc_ref,
                                    [sl if isinstance(sl, torch.Tensor) else torch.zeros(0, dtype=torch.int32)
                                     for sl in slot_lists], D ** -0.5, H, H)
            err = (seen["out"].view(ref.shape) - ref).abs()
            assert err.max() <= 2e-2 and err.mean() <= 2e-3, (step, float(err.max()), float(err.mean()))
            if step == 1:
                # the whole decoder layer against the unpatched reference layer (CPU, fp32)
                e = (y.float().cpu() - y_ref1).abs()
                assert e.max() <= 6e-2 and e.mean() <= 6e-3, (float(e.max()), float(e.mean()))
                for s in seqs:
                    if s.sparse_state is not None:
                        s.sparse_state.cache_state = 2
        handle.remove()
        assert ops.read_device_status(dev) == 0
    finally:
        integration.uninstall()
    assert type(Rf.llada.LLaDADecoderLayer(cfg).attn).__module__ == "dllmserve.layers.attention"
