"""GPU tests of the NeoX rotary embedding (dllm_rope_neox) against the CPU
restatement of RotaryEmbedding.forward (rotary_embedding.py:6-57): bf16
outputs bit-exact (the kernel rounds products and sums separately, like the
reference's fp32 elementwise ops)."""
import pytest
import torch

import inputs as I
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = torch.device("cuda:0")
    torch.cuda.set_device(d)
    return d


def _ops():
    from dllmserve_b200 import ops

    return ops


@pytest.mark.parametrize("hq,hkv,theta,n", [(32, 32, 5e5, 300), (28, 4, 1e6, 257), (4, 1, 1e4, 1)])
def test_rope_bit_exact(dev, hq, hkv, theta, n):
    g = I.gen(160 + hq)
    D, max_pos = 128, 4096
    q = I.normal(g, (n, hq, D)).to(torch.bfloat16)
    k = I.normal(g, (n, hkv, D)).to(torch.bfloat16)
    pos = torch.randint(0, max_pos, (n,), generator=g)
    pos[0] = max_pos - 1
    if n > 1:
        pos[1] = 0
    cache = R.rope_cache(D, max_pos, theta)
    qr, kr = R.apply_rope(q, pos, cache), R.apply_rope(k, pos, cache)
    qo, ko = _ops().rope_neox(pos.to(dev), q.to(dev), k.to(dev), cache.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(qo.cpu(), qr) and torch.equal(ko.cpu(), kr)
    assert _ops().read_device_status(dev) == 0


def test_rope_in_place_on_fused_qkv_views(dev):
    """q and k as views of one fused projection output, rotated in place; v untouched."""
    g = I.gen(170)
    D, hq, hkv, n = 128, 8, 2, 100
    qkv = I.normal(g, (n, (hq + 2 * hkv) * D)).to(torch.bfloat16)
    pos = torch.arange(n) * 3
    cache = R.rope_cache(D, 512, 5e5)
    q = qkv[:, :hq * D].reshape(n, hq, D)
    k = qkv[:, hq * D:(hq + hkv) * D].reshape(n, hkv, D)
    qr, kr = R.apply_rope(q, pos, cache), R.apply_rope(k, pos, cache)
    d = qkv.to(dev)
    qd = d[:, :hq * D].view(n, hq, D)
    kd = d[:, hq * D:(hq + hkv) * D].view(n, hkv, D)
    _ops().rope_neox(pos.to(dev), qd, kd, cache.to(dev), query_out=qd, key_out=kd)
    torch.cuda.synchronize()
    assert torch.equal(qd.cpu(), qr) and torch.equal(kd.cpu(), kr)
    assert torch.equal(d[:, (hq + hkv) * D:].cpu(), qkv[:, (hq + hkv) * D:])


def test_rope_position_out_of_range(dev):
    g = I.gen(171)
    D, n = 128, 4
    q, k = I.normal(g, (n, 2, D)).to(torch.bfloat16), I.normal(g, (n, 2, D)).to(torch.bfloat16)
    cache = R.rope_cache(D, 16, 5e5)
    pos = torch.tensor([1, 16, 3, -1])
    qo, ko = _ops().rope_neox(pos.to(dev), q.to(dev), k.to(dev), cache.to(dev))
    torch.cuda.synchronize()
    assert _ops().read_device_status(dev) == 4
    ok = torch.tensor([0, 2])
    assert torch.equal(qo.cpu()[ok], R.apply_rope(q, pos.clamp(0, 15), cache)[ok])
    assert (qo.cpu()[1] == 0).all() and (ko.cpu()[3] == 0).all()


def test_rotary_embedding_module_matches_reference_formula(dev):
    """The drop-in module: same cache values as the reference's construction and
    the same (query, key) outputs for the model's [N, H*D] inputs."""
    from dllmserve_b200.layers.rotary_embedding import get_rope

    g = I.gen(172)
    D, hq, hkv, n = 128, 28, 4, 77
    rope = get_rope(D, D, 2048, 1e6)
    assert torch.equal(rope.cos_sin_cache, R.rope_cache(D, 2048, 1e6))
    q = I.normal(g, (n, hq * D)).to(torch.bfloat16)
    k = I.normal(g, (n, hkv * D)).to(torch.bfloat16)
    pos = torch.randint(0, 2048, (n,), generator=g)
    qo, ko = rope(pos.to(dev), q.to(dev), k.to(dev))
    torch.cuda.synchronize()
    assert qo.shape == q.shape and ko.shape == k.shape
    cache = R.rope_cache(D, 2048, 1e6)
    assert torch.equal(qo.cpu(), R.apply_rope(q.view(n, hq, D), pos, cache).view(n, -1))
    assert torch.equal(ko.cpu(), R.apply_rope(k.view(n, hkv, D), pos, cache).view(n, -1))
