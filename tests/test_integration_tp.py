"""CPU tests: integration.install() on a synthetic package with the reference's
module layout, and the head-sharded tensor-parallel layer on 2 gloo ranks."""
import os
import socket
import sys
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _fake_reference(name):
    pkg = types.ModuleType(name)
    pkg.__path__ = []
    layers = types.ModuleType(f"{name}.layers")
    layers.__path__ = []
    attn = types.ModuleType(f"{name}.layers.attention")

    class RefAttention:
        pass

    RefAttention.__module__ = attn.__name__
    attn.Attention = RefAttention
    attn.store_kvcache = lambda *a: "ref-store"
    attn.load_kvcache = lambda *a: "ref-load"
    utils = types.ModuleType(f"{name}.utils")
    utils.__path__ = []
    ctx = types.ModuleType(f"{name}.utils.context")
    ctx.get_context = lambda: "ref-context"
    rope = types.ModuleType(f"{name}.layers.rotary_embedding")

    class RefRotary:
        pass

    def ref_get_rope(*a, **kw):
        return "ref-rope"

    RefRotary.__module__ = ref_get_rope.__module__ = rope.__name__
    rope.RotaryEmbedding = RefRotary
    rope.get_rope = ref_get_rope
    models = types.ModuleType(f"{name}.models")
    models.__path__ = []
    llada = types.ModuleType(f"{name}.models.llada")
    llada.Attention = RefAttention
    llada.get_rope = ref_get_rope
    mods = {name: pkg, f"{name}.layers": layers, attn.__name__: attn, f"{name}.utils": utils,
            ctx.__name__: ctx, f"{name}.models": models, llada.__name__: llada, rope.__name__: rope}
    return mods, RefAttention


def test_install_patches_reference_modules(monkeypatch):
    from dllmserve_b200 import integration
    from dllmserve_b200.layers import attention as ours
    from dllmserve_b200.layers import rotary_embedding as our_rope

    mods, RefAttention = _fake_reference("fakeref")
    for k, v in mods.items():
        monkeypatch.setitem(sys.modules, k, v)
    try:
        patched = integration.install("fakeref")
        assert mods["fakeref.layers.attention"].Attention is ours.Attention
        assert mods["fakeref.models.llada"].Attention is ours.Attention
        assert mods["fakeref.layers.attention"].store_kvcache is ours.store_kvcache
        assert ours.get_context() == "ref-context"
        assert mods["fakeref.layers.rotary_embedding"].RotaryEmbedding is our_rope.RotaryEmbedding
        assert mods["fakeref.layers.rotary_embedding"].get_rope is our_rope.get_rope
        assert mods["fakeref.models.llada"].get_rope is our_rope.get_rope
        assert "fakeref.models.llada" in patched
    finally:
        integration.uninstall()
    assert mods["fakeref.layers.attention"].Attention is RefAttention
    assert mods["fakeref.models.llada"].Attention is RefAttention
    assert mods["fakeref.models.llada"].get_rope() == "ref-rope"
    assert ours.get_context() != "ref-context"


# ---------------------------------------------------------------------------
# tensor parallelism: heads sharded over 2 gloo ranks
# ---------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q, k, v, w, lens, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from dllmserve_b200.tp import head_slice, row_parallel_oproj
        from oracle import attention_ref as R

        Hq, Hkv, D = q.shape[1], k.shape[1], q.shape[2]
        h0, h1, k0, k1 = head_slice(Hq, Hkv, rank, world)
        cu = [0]
        for L in lens:
            cu.append(cu[-1] + L)
        o = R.varlen_attention(q[:, h0:h1], k[:, k0:k1], v[:, k0:k1], cu, cu, D ** -0.5)
        y = row_parallel_oproj(o.reshape(o.shape[0], -1), w[:, h0 * D:h1 * D], rank=rank)
        # rows split in 3 chunks, each all-reduced asynchronously after its GEMM
        y3 = row_parallel_oproj(o.reshape(o.shape[0], -1), w[:, h0 * D:h1 * D], rank=rank, chunks=3)
        torch.save({"rank": rank, "attn": o, "y": y, "y3": y3}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("hq,hkv", [(4, 4), (4, 2)])
def test_head_sharded_tp_matches_single_process(tmp_path, hq, hkv):
    from oracle import attention_ref as R

    g = torch.Generator().manual_seed(7)
    lens = [33, 70]
    N, D, hidden = sum(lens), 128, 64
    q = torch.randn(N, hq, D, generator=g)
    k = torch.randn(N, hkv, D, generator=g)
    v = torch.randn(N, hkv, D, generator=g)
    w = torch.randn(hidden, hq * D, generator=g) * 0.02
    world = 2
    out = str(tmp_path / "tp")
    mp.start_processes(_tp_worker, args=(world, _free_port(), q, k, v, w, lens, out), nprocs=world,
                       start_method="spawn")
    cu = [0, lens[0], N]
    full = R.varlen_attention(q, k, v, cu, cu, D ** -0.5)
    y_ref = full.reshape(N, -1) @ w.t()
    per_rank = hq // world
    for r in range(world):
        res = torch.load(f"{out}.{r}")
        # each rank's attention equals the single-process result on its head slice
        torch.testing.assert_close(res["attn"], full[:, r * per_rank:(r + 1) * per_rank])
        # the all-reduced row-parallel o_proj equals the single-process o_proj
        torch.testing.assert_close(res["y"], y_ref, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(res["y3"], y_ref, rtol=1e-4, atol=1e-4)
