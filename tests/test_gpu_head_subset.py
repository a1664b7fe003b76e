"""GPU tests of the head-compacted attention launch (dllm_attn_varlen_heads_fwd
through ops.varlen_attention(heads=...)): only the listed query heads are
computed -- each against the fp32 oracle restricted to that head, within
max-abs 2e-2 / mean-abs 2e-3 -- the other heads' output rows keep their
contents, both attention kernels (query segments longer than 128 rows and
short ones) and the paged cache are covered, and an index outside the head
range sets the device status word without touching memory."""
import pytest
import torch

import inputs as I
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu
D = 128


def _cu(lens):
    c = [0]
    for L in lens:
        c.append(c[-1] + L)
    return c


@pytest.mark.parametrize("lens,H,Hk,paged", [
    ([300, 129, 700, 1], 8, 8, False),      # pair kernel, MHA
    ([257, 513, 64], 14, 2, False),         # pair kernel, GQA 7:1
    ([32, 77, 128, 5], 8, 4, False),        # split kernel, GQA 2:1 (head packing off)
    ([32, 32, 32], 8, 8, True),             # split kernel, paged cached rows
])
def test_head_subset_matches_oracle(lens, H, Hk, paged):
    from dllmserve_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = I.gen(sum(lens) + H)
    N = sum(lens)
    q, k, v = I.normal(g, (N, H, D)), I.normal(g, (N, Hk, D)), I.normal(g, (N, Hk, D))
    heads = torch.randperm(H, generator=g)[: max(1, H // 2)].to(torch.int32)
    t = lambda x: x.to(dev, torch.bfloat16)
    cu = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    kw, kc_rows, vc_rows, cuc = {}, None, None, None
    if paged:
        nc = [40, 300, 129]
        pages = (sum(nc) + 255) // 256 + 2
        kc = I.normal(g, (pages, 256, Hk, D))
        vc = I.normal(g, (pages, 256, Hk, D))
        slots = torch.randperm(pages * 256, generator=g)[: sum(nc)].to(torch.int32)
        cuc = _cu(nc)
        kw = dict(k_cache=t(kc), v_cache=t(vc), slots=slots.to(dev),
                  cu_seqlens_slots=torch.tensor(cuc, dtype=torch.int32, device=dev))
        kc_rows = kc.view(-1, Hk, D)[slots.long()]
        vc_rows = vc.view(-1, Hk, D)[slots.long()]
    out = torch.full((N, H, D), 7.0, dtype=torch.bfloat16, device=dev)
    ops.varlen_attention(t(q), t(k), t(v), cu, cu, max(lens), D ** -0.5, out=out, heads=heads.to(dev), **kw)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 0
    ref = R.varlen_attention(q, k, v, _cu(lens), _cu(lens), D ** -0.5, kc_rows, vc_rows, cuc)
    o = out.float().cpu()
    sel = set(heads.tolist())
    for h in range(H):
        if h in sel:
            err = (o[:, h] - ref[:, h]).abs()
            assert err.max() <= 2e-2 and err.mean() <= 2e-3, (h, float(err.max()), float(err.mean()))
        else:
            assert torch.all(o[:, h] == 7.0), h
    # the same heads through the all-heads launch agree bit for bit
    full = ops.varlen_attention(t(q), t(k), t(v), cu, cu, max(lens), D ** -0.5, **kw)
    for h in sel:
        assert torch.equal(out[:, h], full[:, h])


def test_head_subset_bad_index_flags_status():
    from dllmserve_b200 import _native, ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = I.gen(5)
    lens, H = [200, 50], 4
    N = sum(lens)
    q, k, v = (I.normal(g, (N, H, D)).to(dev, torch.bfloat16) for _ in range(3))
    cu = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    out = torch.full((N, H, D), 7.0, dtype=torch.bfloat16, device=dev)
    heads = torch.tensor([1, 9, -1], dtype=torch.int32, device=dev)
    ops.varlen_attention(q, k, v, cu, cu, max(lens), D ** -0.5, out=out, heads=heads)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == _native.DLLM_DEV_BAD_SEQUENCE
    o = out.float().cpu()
    assert torch.isfinite(o[:, 1]).all() and not torch.all(o[:, 1] == 7.0)
    for h in (0, 2, 3):
        assert torch.all(o[:, h] == 7.0)
