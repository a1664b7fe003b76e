"""GPU tests of the rotary embedding fused into attention
(dllm_attn_varlen_rope_fwd): the decoder layer's `q, k = rotary_emb(positions,
q, k); attn(q, k, v)` (llada.py:81-84, dream.py:90-93) in one launch.

The fused result must equal the unfused one (dllm_rope_neox, then the same
attention) bit for bit, since the rotation in shared memory uses the same
separately rounded fp32 arithmetic and the same bf16 rounding; one case is also
checked end to end against the CPU restatement (oracle rotation + fp32
attention, within the attention tolerance). q and k must come back untouched.
"""
import pytest
import torch

import inputs as I
from oracle import attention_ref as R
from test_gpu_kernels import MAX_ABS, MEAN_ABS, _check_attn, _cu

pytestmark = pytest.mark.gpu

D = 128


@pytest.fixture(scope="module")
def dev():
    d = torch.device("cuda:0")
    torch.cuda.set_device(d)
    return d


def _ops():
    from dllmserve_b200 import ops

    return ops


def _positions(lens, g, max_pos):
    """Per sequence: a random prompt offset, then consecutive positions."""
    out = []
    for L in lens:
        start = int(torch.randint(0, max_pos - L + 1, (1,), generator=g))
        out.append(torch.arange(start, start + L))
    return torch.cat(out)


def _fused_vs_unfused(dev, q, k, v, lens, pos, cache, **paged):
    ops = _ops()
    cq = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    q0, k0 = q.clone(), k.clone()
    fused = ops.varlen_attention(q, k, v, cq, cq, max(lens), D ** -0.5, rope=(pos, cache), **paged)
    qr, kr = ops.rope_neox(pos, q, k, cache)
    ref = ops.varlen_attention(qr, kr, v, cq, cq, max(lens), D ** -0.5, **paged)
    torch.cuda.synchronize()
    assert torch.equal(q, q0) and torch.equal(k, k0), "inputs were modified"
    return fused, ref


@pytest.mark.parametrize("hq,hkv,lens", [
    (32, 32, [32] * 8),                      # the reuse steps' block (LLaDA)
    (28, 4, [32] * 16),                      # Dream GQA: 4 query heads packed per tile
    (8, 2, [1, 7, 64, 33, 128, 100, 2, 64]),  # ragged, one full tile
    (6, 3, [40, 17, 1]),                     # GQA group 2, 2 heads packed
])
def test_rope_attention_bit_exact(dev, hq, hkv, lens):
    g = I.gen(400 + hq + len(lens))
    n, max_pos = sum(lens), 2048
    t = lambda x: x.to(dev, torch.bfloat16)
    q, k, v = t(I.normal(g, (n, hq, D))), t(I.normal(g, (n, hkv, D))), t(I.normal(g, (n, hkv, D)))
    cache = R.rope_cache(D, max_pos, 5e5).to(dev)
    pos = _positions(lens, g, max_pos).to(dev)
    fused, ref = _fused_vs_unfused(dev, q, k, v, lens, pos, cache)
    assert torch.equal(fused, ref)
    assert _ops().read_device_status(dev) == 0


def test_rope_attention_against_oracle(dev):
    """End to end against the CPU restatement: oracle rotation, fp32 attention."""
    g = I.gen(410)
    hq, hkv, lens, max_pos = 4, 2, [32, 5, 128], 512
    n = sum(lens)
    q, k, v = I.normal(g, (n, hq, D)), I.normal(g, (n, hkv, D)), I.normal(g, (n, hkv, D))
    qb, kb, vb = (x.to(torch.bfloat16) for x in (q, k, v))
    cache = R.rope_cache(D, max_pos, 1e6)
    pos = _positions(lens, g, max_pos)
    ref = R.varlen_attention(R.apply_rope(qb, pos, cache).float(), R.apply_rope(kb, pos, cache).float(),
                             vb.float(), _cu(lens), _cu(lens), D ** -0.5)
    cq = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(qb.to(dev), kb.to(dev), vb.to(dev), cq, cq, max(lens), D ** -0.5,
                                  rope=(pos.to(dev), cache.to(dev)))
    _check_attn(out, ref, "rope+attention vs oracle")
    assert _ops().read_device_status(dev) == 0


@pytest.mark.parametrize("hq,hkv", [(32, 32), (28, 4)])
def test_rope_attention_paged_reuse_step(dev, hq, hkv):
    """A reuse step: keys = [already rotated cache rows at slots ; the block's
    fresh rows, rotated on chip]."""
    g = I.gen(420 + hkv)
    pages, max_pos = 10, 4096
    lq = [32, 32, 32, 32]
    n_c = [304, 0, 129, 600]
    kc, vc = I.normal(g, (pages, 256, hkv, D)), I.normal(g, (pages, 256, hkv, D))
    slots = torch.randperm(pages * 256, generator=g)[:sum(n_c)].to(torch.int32)
    slots[:304] = torch.arange(512, 512 + 304, dtype=torch.int32)  # one run of consecutive slots
    n = sum(lq)
    t = lambda x: x.to(dev, torch.bfloat16)
    q, k, v = t(I.normal(g, (n, hq, D))), t(I.normal(g, (n, hkv, D))), t(I.normal(g, (n, hkv, D)))
    cache = R.rope_cache(D, max_pos, 5e5).to(dev)
    pos = torch.cat([torch.arange(c, c + b) for c, b in zip(n_c, lq)]).to(dev)
    paged = dict(k_cache=t(kc), v_cache=t(vc), slots=slots.to(dev),
                 cu_seqlens_slots=torch.tensor(_cu(n_c), dtype=torch.int32, device=dev))
    fused, ref = _fused_vs_unfused(dev, q, k, v, lq, pos, cache, **paged)
    assert torch.equal(fused, ref)
    assert _ops().read_device_status(dev) == 0


def test_rope_attention_long_segments_rotate_first(dev):
    """Query segments over 128 rows take the rotate-then-attend route (same result)."""
    g = I.gen(430)
    hq, hkv, lens = 4, 4, [300, 64]
    n = sum(lens)
    t = lambda x: x.to(dev, torch.bfloat16)
    q, k, v = t(I.normal(g, (n, hq, D))), t(I.normal(g, (n, hkv, D))), t(I.normal(g, (n, hkv, D)))
    cache = R.rope_cache(D, 1024, 5e5).to(dev)
    pos = _positions(lens, g, 1024).to(dev)
    fused, ref = _fused_vs_unfused(dev, q, k, v, lens, pos, cache)
    assert torch.equal(fused, ref)
    assert _ops().read_device_status(dev) == 0


def test_rope_attention_position_out_of_range(dev):
    """A position outside the cache gives a zero row (as dllm_rope_neox does) and
    flags DLLM_DEV_POSITION_OUT_OF_RANGE."""
    g = I.gen(440)
    hq, hkv, lens, max_pos = 2, 2, [20, 12], 64
    n = sum(lens)
    t = lambda x: x.to(dev, torch.bfloat16)
    q, k, v = t(I.normal(g, (n, hq, D))), t(I.normal(g, (n, hkv, D))), t(I.normal(g, (n, hkv, D)))
    cache = R.rope_cache(D, max_pos, 5e5).to(dev)
    pos = _positions(lens, g, max_pos)
    pos[3], pos[25] = max_pos, -2
    pos = pos.to(dev)
    fused, ref = _fused_vs_unfused(dev, q, k, v, lens, pos, cache)
    assert torch.equal(fused, ref)
    assert _ops().read_device_status(dev) == 4


def test_rope_attention_rejects_bad_args(dev):
    ops = _ops()
    q = torch.zeros(8, 2, D, dtype=torch.bfloat16, device=dev)
    k = torch.zeros(8, 2, D, dtype=torch.bfloat16, device=dev)
    cq = torch.tensor([0, 8], dtype=torch.int32, device=dev)
    cache = torch.zeros(16, D, dtype=torch.float32, device=dev)
    pos = torch.arange(8, device=dev)
    with pytest.raises(ValueError):  # positions must be int64
        ops.varlen_attention(q, k, k, cq, cq, 8, rope=(pos.to(torch.int32), cache))
    with pytest.raises(ValueError):  # cache must be fp32
        ops.varlen_attention(q, k, k, cq, cq, 8, rope=(pos, cache.to(torch.bfloat16)))
    with pytest.raises(ValueError):  # one position per query row
        ops.varlen_attention(q, k, k, cq, cq, 8, rope=(pos[:7], cache))
    assert ops.read_device_status(dev) == 0
