"""GPU parity tests of the native kernels against the CPU oracle.

Tolerances (from the benchmark spec): attention outputs in bf16 vs the fp32
oracle within max-abs 2e-2 and mean-abs 2e-3; KV-cache contents bit-exact;
selected indices bit-exact (same tie rule: descending score, ascending index).
"""
import os

import numpy as np
import pytest
import torch

import inputs as I
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


@pytest.fixture(scope="module")
def dev():
    d = torch.device("cuda:0")
    torch.cuda.set_device(d)
    from dllmserve_b200 import _native

    _native.lib()
    return d


def _ops():
    from dllmserve_b200 import ops

    return ops


def _status_clear(dev):
    assert _ops().read_device_status(dev) == 0


def _cu(lens):
    c = [0]
    for L in lens:
        c.append(c[-1] + L)
    return c


def _check_attn(out_gpu, ref, what=""):
    err = (out_gpu.float().cpu() - ref).abs()
    assert torch.isfinite(out_gpu.float()).all(), f"{what}: non-finite output"
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, (
        f"{what}: max {err.max().item():.3e} mean {err.mean().item():.3e}")


# ---------------------------------------------------------------------------
# KV cache store / load
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n,hkv", [(1, 32), (7, 4), (300, 32), (1000, 1), (4097, 8)])
def test_store_kvcache_bit_exact(dev, n, hkv):
    g = I.gen(n + hkv)
    D = 128
    pages = (n + 255) // 256 + 3
    key = I.normal(g, (n, hkv, D)).to(torch.bfloat16)
    val = I.normal(g, (n, hkv, D)).to(torch.bfloat16)
    slots = torch.randperm(pages * 256, generator=g)[:n].to(torch.int32)
    canary = torch.full((pages, 256, hkv, D), 7.0, dtype=torch.bfloat16)
    kc_ref, vc_ref = canary.clone(), canary.clone()
    R.store_kvcache(key, val, kc_ref, vc_ref, slots)
    kc, vc = canary.to(dev), canary.to(dev)
    _ops().store_kvcache(key.to(dev), val.to(dev), kc, vc, slots.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(kc.cpu(), kc_ref) and torch.equal(vc.cpu(), vc_ref)
    _status_clear(dev)


def test_store_kvcache_strided_rows(dev):
    """key/value as column slices of a fused qkv buffer (token stride > row)."""
    g = I.gen(5)
    n, hq, hkv, D = 333, 8, 2, 128
    qkv = I.normal(g, (n, (hq + 2 * hkv) * D)).to(torch.bfloat16).to(dev)
    k = qkv[:, hq * D:(hq + hkv) * D].view(n, hkv, D)
    v = qkv[:, (hq + hkv) * D:].view(n, hkv, D)
    slots = torch.randperm(512, generator=g)[:n].to(torch.int32)
    kc = torch.zeros(2, 256, hkv, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    _ops().store_kvcache(k, v, kc, vc, slots.to(dev))
    kr, vr = torch.zeros(2, 256, hkv, D, dtype=torch.bfloat16), torch.zeros(2, 256, hkv, D, dtype=torch.bfloat16)
    R.store_kvcache(k.cpu(), v.cpu(), kr, vr, slots)
    assert torch.equal(kc.cpu(), kr) and torch.equal(vc.cpu(), vr)


def test_load_kvcache_bit_exact(dev):
    g = I.gen(9)
    hkv, D, pages, n = 4, 128, 6, 900
    kc = I.normal(g, (pages, 256, hkv, D)).to(torch.bfloat16)
    vc = I.normal(g, (pages, 256, hkv, D)).to(torch.bfloat16)
    slots = torch.randint(0, pages * 256, (n,), generator=g).to(torch.int32)
    k_ref, v_ref = R.load_kvcache(kc, vc, slots, hkv, D)
    k = torch.full((n, hkv, D), float("nan"), dtype=torch.bfloat16, device=dev)
    v = torch.full_like(k, float("nan"))
    _ops().load_kvcache(k, v, kc.to(dev), vc.to(dev), slots.to(dev))
    assert torch.equal(k.cpu(), k_ref) and torch.equal(v.cpu(), v_ref)


def test_slot_edge_cases(dev):
    """Negative slots are skipped; slots past the cache are skipped and flagged."""
    hkv, D = 2, 128
    key = torch.ones(3, hkv, D, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(1, 256, hkv, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    ops = _ops()
    ops.store_kvcache(key, key, kc, vc, torch.tensor([-1, 5, 256], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 1
    ref = torch.zeros(256, hkv, D, dtype=torch.bfloat16)
    ref[5] = 1
    assert torch.equal(kc.cpu().view(256, hkv, D), ref)
    # empty store is a no-op
    ops.store_kvcache(key[:0], key[:0], kc, vc, torch.zeros(0, dtype=torch.int32, device=dev))
    _status_clear(dev)


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
SMALL_LENS = [[1], [2], [31], [33], [127], [128], [129], [255], [256], [257], [300], [513],
              [1, 2, 3], [129, 7, 256, 1]]


@pytest.mark.parametrize("lens", SMALL_LENS, ids=[str(x) for x in SMALL_LENS])
@pytest.mark.parametrize("hq,hkv", [(4, 4), (7, 1), (8, 2)])
def test_attention_small(dev, lens, hq, hkv):
    g = I.gen(sum(lens) * 31 + hq)
    D, N = 128, sum(lens)
    q, k, v = I.normal(g, (N, hq, D)), I.normal(g, (N, hkv, D)), I.normal(g, (N, hkv, D))
    cu = _cu(lens)
    ref = R.varlen_attention(q, k, v, cu, cu, D ** -0.5)
    cu_d = torch.tensor(cu, dtype=torch.int32, device=dev)
    out = torch.full((N, hq, D), float("nan"), dtype=torch.bfloat16, device=dev)
    _ops().varlen_attention(q.to(dev, torch.bfloat16), k.to(dev, torch.bfloat16),
                            v.to(dev, torch.bfloat16), cu_d, cu_d, max(lens), D ** -0.5, out=out)
    torch.cuda.synchronize()
    _check_attn(out, ref, f"lens={lens} hq={hq} hkv={hkv}")
    _status_clear(dev)


def test_attention_separate_q_and_k_lengths(dev):
    """Lq != Lk per sequence (flash_attn_varlen_func semantics)."""
    g = I.gen(77)
    D, hq, hkv = 128, 4, 2
    lq, lk = [5, 200, 130], [300, 1, 129]
    q = I.normal(g, (sum(lq), hq, D))
    k, v = I.normal(g, (sum(lk), hkv, D)), I.normal(g, (sum(lk), hkv, D))
    ref = R.varlen_attention(q, k, v, _cu(lq), _cu(lk), 0.1)
    out = _ops().varlen_attention(
        q.to(dev, torch.bfloat16), k.to(dev, torch.bfloat16), v.to(dev, torch.bfloat16),
        torch.tensor(_cu(lq), dtype=torch.int32, device=dev),
        torch.tensor(_cu(lk), dtype=torch.int32, device=dev), max(lq), 0.1)
    _check_attn(out, ref)


@pytest.mark.parametrize("batch", [256, 300])
def test_attention_many_sequences(dev, batch):
    """Hundreds of ragged sequences in one launch (short ones: the split
    kernel), with empty query or key segments."""
    g = I.gen(90 + batch)
    D, hq, hkv = 128, 2, 1
    lq = torch.randint(0, 300, (batch,), generator=g).tolist()
    lk = torch.randint(0, 300, (batch,), generator=g).tolist()
    lq[3], lk[5], lq[7], lk[7] = 0, 0, 0, 0
    q = I.normal(g, (sum(lq), hq, D))
    k, v = I.normal(g, (sum(lk), hkv, D)), I.normal(g, (sum(lk), hkv, D))
    ref = R.varlen_attention(q, k, v, _cu(lq), _cu(lk), D ** -0.5)
    t = lambda x: x.to(dev, torch.bfloat16)
    out = torch.full((sum(lq), hq, D), float("nan"), dtype=torch.bfloat16, device=dev)
    _ops().varlen_attention(t(q), t(k), t(v), torch.tensor(_cu(lq), dtype=torch.int32, device=dev),
                            torch.tensor(_cu(lk), dtype=torch.int32, device=dev), max(lq),
                            D ** -0.5, out=out)
    torch.cuda.synchronize()
    _check_attn(out, ref, f"batch={batch}")
    _status_clear(dev)


def test_attention_sched_workspace_matches_round_robin(dev):
    """Dynamic unit scheduling (a scheduler workspace) writes the same output
    bits as the round-robin order, twice in a row, and leaves the workspace zero."""
    import ctypes
    from dllmserve_b200 import _native
    g = I.gen(140)
    D, H = 128, 8
    lens = [419, 1087, 700, 130, 900, 256, 555, 1000, 3]
    N = sum(lens)
    q, k, v = (I.normal(g, (N, H, D)).to(dev, torch.bfloat16) for _ in range(3))
    cu = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    lib = _native.lib()

    def run(ws):
        o = torch.full_like(q, float("nan"))
        rc = lib.dllm_attn_varlen_fwd(
            q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
            o.data_ptr(), o.stride(0), cu.data_ptr(), cu.data_ptr(), len(lens), max(lens), N, N,
            H, H, D, ctypes.c_float(D ** -0.5), None if ws is None else ws.data_ptr(), None,
            torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.dllm_last_error()
        return o

    ref = run(None)
    ws = torch.zeros(_native.SCHED_WORKSPACE_INTS, dtype=torch.int32, device=dev)
    first, second = run(ws), run(ws)
    torch.cuda.synchronize()
    assert torch.equal(first, ref) and torch.equal(second, ref)
    assert int(ws.abs().sum()) == 0
    _check_attn(ref, R.varlen_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(),
                                        _cu(lens), _cu(lens), D ** -0.5))


def test_attention_two_streams_at_once(dev):
    """Launches overlapping on two streams use separate scheduler workspaces:
    both outputs equal the single-stream result bit for bit."""
    g = I.gen(141)
    D, H = 128, 8
    lens = [900, 300, 1087, 129, 640]
    N = sum(lens)
    q, k, v = (I.normal(g, (N, H, D)).to(dev, torch.bfloat16) for _ in range(3))
    cu = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    ops = _ops()
    ref = ops.varlen_attention(q, k, v, cu, cu, max(lens))
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = []
    for s in (s1, s2):
        s.wait_stream(torch.cuda.current_stream())
    for rep in range(4):
        for s in (s1, s2):
            with torch.cuda.stream(s):
                outs.append(ops.varlen_attention(q, k, v, cu, cu, max(lens)))
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, ref)
    _status_clear(dev)


def test_attention_fused_qkv_views(dev):
    """q/k/v as strided views of one fused projection output."""
    g = I.gen(78)
    D, hq, hkv, lens = 128, 8, 2, [100, 250]
    N = sum(lens)
    qkv = I.normal(g, (N, (hq + 2 * hkv) * D))
    q = qkv[:, :hq * D].reshape(N, hq, D)
    k = qkv[:, hq * D:(hq + hkv) * D].reshape(N, hkv, D)
    v = qkv[:, (hq + hkv) * D:].reshape(N, hkv, D)
    ref = R.varlen_attention(q, k, v, _cu(lens), _cu(lens), D ** -0.5)
    qd = qkv.to(dev, torch.bfloat16)
    cu = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(qd[:, :hq * D].view(N, hq, D),
                                  qd[:, hq * D:(hq + hkv) * D].view(N, hkv, D),
                                  qd[:, (hq + hkv) * D:].view(N, hkv, D), cu, cu, max(lens))
    _check_attn(out, ref)


def test_attention_large_logits(dev):
    """Rows whose max moves a lot across KV tiles exercise the rescaling path."""
    g = I.gen(79)
    D, H, L = 128, 2, 700
    q = I.normal(g, (L, H, D)) * 3
    k = I.normal(g, (L, H, D))
    k[600:] *= 4  # the largest logits arrive in the last tiles
    v = I.normal(g, (L, H, D))
    q, k = q.to(torch.bfloat16).float(), k.to(torch.bfloat16).float()
    ref = R.varlen_attention(q, k, v, [0, L], [0, L], D ** -0.5)
    cu = torch.tensor([0, L], dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(q.to(dev, torch.bfloat16), k.to(dev, torch.bfloat16),
                                  v.to(dev, torch.bfloat16), cu, cu, L)
    _check_attn(out, ref)


@pytest.mark.parametrize("hq,hkv", [(4, 4), (7, 1)])
def test_attention_cached_segments(dev, hq, hkv):
    """keys = [cached rows ; fresh rows] per sequence (the reuse state)."""
    g = I.gen(80 + hq)
    D = 128
    lq = [32, 32, 17, 200]
    lc = [304, 0, 129, 1]
    q = I.normal(g, (sum(lq), hq, D))
    k, v = I.normal(g, (sum(lq), hkv, D)), I.normal(g, (sum(lq), hkv, D))
    kc, vc = I.normal(g, (sum(lc), hkv, D)), I.normal(g, (sum(lc), hkv, D))
    ref = R.varlen_attention(q, k, v, _cu(lq), _cu(lq), D ** -0.5, kc, vc, _cu(lc))
    t = lambda x: x.to(dev, torch.bfloat16)
    cq = torch.tensor(_cu(lq), dtype=torch.int32, device=dev)
    cc = torch.tensor(_cu(lc), dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(t(q), t(k), t(v), cq, cq, max(lq), D ** -0.5,
                                  k_cached=t(kc), v_cached=t(vc), cu_seqlens_c=cc)
    _check_attn(out, ref)
    _status_clear(dev)


SPLIT_EDGE = [  # (query rows, cached rows, fresh key rows) per sequence, all query segments <= 128
    [(32, 40, 32), (1, 0, 1), (17, 1, 17), (64, 63, 64)],
    [(65, 64, 65), (128, 65, 128), (100, 129, 100), (32, 300, 32)],
    [(128, 0, 128), (5, 0, 64), (6, 0, 65), (7, 127, 1)],
]


@pytest.mark.parametrize("case", range(len(SPLIT_EDGE)), ids=[f"e{i}" for i in range(len(SPLIT_EDGE))])
@pytest.mark.parametrize("hq,hkv", [(4, 4), (7, 1)])
def test_attention_single_tile_segments(dev, case, hq, hkv):
    """Launches whose query segments fit one 128-row tile (the split kernel): key
    tiles whose second half has no valid rows (cached segments of 40/63/64 rows,
    1-64 fresh rows), a second half that stays empty for a whole sequence, and
    partial tiles at the end of the cached segment."""
    seqs = SPLIT_EDGE[case]
    lq = [s[0] for s in seqs]
    lc = [s[1] for s in seqs]
    lk = [s[2] for s in seqs]
    g = I.gen(120 + case * 7 + hq)
    D = 128
    q = I.normal(g, (sum(lq), hq, D))
    k, v = I.normal(g, (sum(lk), hkv, D)), I.normal(g, (sum(lk), hkv, D))
    kc, vc = I.normal(g, (sum(lc), hkv, D)), I.normal(g, (sum(lc), hkv, D))
    ref = R.varlen_attention(q, k, v, _cu(lq), _cu(lk), D ** -0.5, kc, vc, _cu(lc))
    t = lambda x: x.to(dev, torch.bfloat16)
    i32 = lambda x: torch.tensor(_cu(x), dtype=torch.int32, device=dev)
    out = torch.full((sum(lq), hq, D), float("nan"), dtype=torch.bfloat16, device=dev)
    _ops().varlen_attention(t(q), t(k), t(v), i32(lq), i32(lk), max(lq), D ** -0.5,
                            k_cached=t(kc), v_cached=t(vc), cu_seqlens_c=i32(lc), out=out)
    torch.cuda.synchronize()
    _check_attn(out, ref, f"case {case} hq={hq} hkv={hkv}")
    # the same keys without a cached segment
    ref2 = R.varlen_attention(q, k, v, _cu(lq), _cu(lk), D ** -0.5)
    out2 = _ops().varlen_attention(t(q), t(k), t(v), i32(lq), i32(lk), max(lq), D ** -0.5)
    _check_attn(out2, ref2, f"case {case} fresh only")
    _status_clear(dev)


def test_attention_c2_full_layer(dev):
    """A whole config-2 layer (B=16, L in [419, 1087], 32 MHA heads, 157.6
    GFLOP): every (sequence, head) pair against the fp32 oracle, each within
    max-abs 2e-2 / mean-abs 2e-3."""
    import bench

    lens = bench.workload_lengths()
    D, H = 128, 32
    N = sum(lens)
    gd = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(N, H, D, device=dev, dtype=torch.bfloat16, generator=gd)
    k = torch.randn(N, H, D, device=dev, dtype=torch.bfloat16, generator=gd)
    v = torch.randn(N, H, D, device=dev, dtype=torch.bfloat16, generator=gd)
    cu = _cu(lens)
    cud = torch.tensor(cu, dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(q, k, v, cud, cud, max(lens))
    torch.cuda.synchronize()
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    ref = R.varlen_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), cu, cu, D ** -0.5)
    err = (out.float().cpu() - ref).abs()
    worst_max = worst_mean = 0.0
    for b in range(len(lens)):
        e = err[cu[b]:cu[b + 1]]                      # [L, H, D]
        mx = e.amax(dim=(0, 2))
        mean = e.mean(dim=(0, 2))
        worst_max, worst_mean = max(worst_max, float(mx.max())), max(worst_mean, float(mean.max()))
    assert worst_max <= 2e-2 and worst_mean <= 2e-3, (worst_max, worst_mean)
    _status_clear(dev)


def _sampled_check(out, q, k, v, cu, pairs, group=1, kc=None, vc=None, cuc=None):
    """(sequence, query head) pairs of a full-size launch against the oracle;
    with kc/vc/cuc the keys of sequence b are [cached rows ; fresh rows]."""
    D = q.shape[2]
    for b, h in pairs:
        s0, s1 = cu[b], cu[b + 1]
        hk = h // group
        kk, vv = k[s0:s1, hk:hk + 1].cpu(), v[s0:s1, hk:hk + 1].cpu()
        if kc is not None:
            c0, c1 = cuc[b], cuc[b + 1]
            kk = torch.cat([kc[c0:c1, hk:hk + 1].cpu(), kk])
            vv = torch.cat([vc[c0:c1, hk:hk + 1].cpu(), vv])
        ref = R.sdpa_seq(q[s0:s1, h:h + 1].cpu(), kk, vv, D ** -0.5)
        _check_attn(out[s0:s1, h:h + 1], ref, f"seq {b} head {h}")


def test_attention_c5_dense_full_size_sampled(dev):
    """Config-5 dense step shape (B=8, L=4,608, 32 MHA heads; 2.78 TFLOP per
    layer): every output row finite, sampled pairs against the oracle."""
    D, H, lens = 128, 32, [4608] * 8
    N = sum(lens)
    gd = torch.Generator(device=dev).manual_seed(51)
    q, k, v = (torch.randn(N, H, D, device=dev, dtype=torch.bfloat16, generator=gd) for _ in range(3))
    cu = _cu(lens)
    cud = torch.tensor(cu, dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(q, k, v, cud, cud, max(lens))
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    _sampled_check(out, q, k, v, cu, [(0, 0), (5, 17), (7, 31)])
    _status_clear(dev)


def test_attention_c5_reuse_full_size_sampled(dev):
    """Config-5 reuse step (8 sequences: 1,144 selected rows read from the paged
    cache by slot + the 32-row block, 32 heads), slots scattered over pages."""
    D, H, blk, n_keep, B = 128, 32, 32, 1144, 8
    gd = torch.Generator(device=dev).manual_seed(52)
    pages = (B * n_keep + 255) // 256 + 3
    kc = torch.randn(pages, 256, H, D, device=dev, dtype=torch.bfloat16, generator=gd)
    vc = torch.randn(pages, 256, H, D, device=dev, dtype=torch.bfloat16, generator=gd)
    perm = torch.randperm(pages * 256, device=dev, generator=gd)[:B * n_keep].to(torch.int32)
    # half the sequences on consecutive slots (TMA path), half scattered (gather path)
    slots = torch.cat([torch.arange(b * n_keep, (b + 1) * n_keep, device=dev, dtype=torch.int32)
                       if b % 2 == 0 else perm[b * n_keep:(b + 1) * n_keep] for b in range(B)])
    N = B * blk
    q, k, v = (torch.randn(N, H, D, device=dev, dtype=torch.bfloat16, generator=gd) for _ in range(3))
    cu, cuc = _cu([blk] * B), _cu([n_keep] * B)
    out = _ops().varlen_attention(q, k, v, torch.tensor(cu, dtype=torch.int32, device=dev),
                                  torch.tensor(cu, dtype=torch.int32, device=dev), blk,
                                  k_cache=kc, v_cache=vc, slots=slots,
                                  cu_seqlens_slots=torch.tensor(cuc, dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    rows_k = kc.view(-1, H, D)[slots.long()]
    rows_v = vc.view(-1, H, D)[slots.long()]
    _sampled_check(out, q, k, v, cu, [(0, 3), (1, 30), (6, 11), (7, 0)], kc=rows_k, vc=rows_v, cuc=cuc)
    _status_clear(dev)


def test_attention_c4_dense_full_size_sampled(dev):
    """Config-4 dense step shape (Dream-7B GQA 28/4, B=32, prompt U[128,768] +
    256 generated tokens): sampled (sequence, query head) pairs."""
    D, Hq, Hkv = 128, 28, 4
    g = torch.Generator().manual_seed(4)
    lens = [int(p) + 256 for p in torch.randint(128, 769, (32,), generator=g)]
    N = sum(lens)
    gd = torch.Generator(device=dev).manual_seed(53)
    q = torch.randn(N, Hq, D, device=dev, dtype=torch.bfloat16, generator=gd)
    k = torch.randn(N, Hkv, D, device=dev, dtype=torch.bfloat16, generator=gd)
    v = torch.randn(N, Hkv, D, device=dev, dtype=torch.bfloat16, generator=gd)
    cu = _cu(lens)
    cud = torch.tensor(cu, dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(q, k, v, cud, cud, max(lens))
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    _sampled_check(out, q, k, v, cu, [(0, 0), (9, 6), (20, 13), (31, 27)], group=Hq // Hkv)
    _status_clear(dev)


def test_attention_rejects_bad_args(dev):
    ops = _ops()
    q = torch.zeros(4, 2, 64, dtype=torch.bfloat16, device=dev)
    cu = torch.tensor([0, 4], dtype=torch.int32, device=dev)
    with pytest.raises(NotImplementedError):
        ops.varlen_attention(q, q, q, cu, cu, 4)
    q = torch.zeros(4, 3, 128, dtype=torch.bfloat16, device=dev)
    k = torch.zeros(4, 2, 128, dtype=torch.bfloat16, device=dev)
    with pytest.raises(NotImplementedError):
        ops.varlen_attention(q, k, k, cu, cu, 4)


# ---------------------------------------------------------------------------
# scoring + top-k + store
# ---------------------------------------------------------------------------
SEL_CASES = [
    # (hq, hkv, head_select, pool, ratio, seqs[(L, blk_start, blk_len)])
    (4, 4, True, 3, 0.5, [(96, 64, 32), (134, 70, 32), (33, 1, 32)]),
    (7, 1, True, 3, 0.5, [(640, 512, 32), (97, 65, 32)]),
    (28, 4, True, 3, 0.5, [(704, 448, 32)]),
    (8, 2, False, 3, 0.5, [(77, 45, 32), (154, 90, 32)]),
    (32, 32, False, 5, 0.25, [(300, 100, 32)]),
    (4, 4, True, 1, 0.5, [(200, 50, 32)]),
    (4, 4, True, 4, 0.5, [(200, 50, 32)]),
    (4, 2, True, 3, 0.0, [(100, 10, 32)]),
    (4, 2, True, 3, 1.0, [(100, 10, 32)]),
    (32, 32, True, 3, 0.25, [(4608, 4096, 32)]),
    # shared ranking at config-5 size (radix select in the cluster leader) and a
    # GQA batch of several sequences (one cluster each)
    (32, 32, False, 3, 0.25, [(4608, 4096, 32)]),
    (28, 4, False, 3, 0.5, [(704, 448, 32), (300, 100, 32), (2600, 2000, 32)]),
]


@pytest.mark.parametrize("case", SEL_CASES, ids=[f"c{i}" for i in range(len(SEL_CASES))])
def test_select_kv_store_bit_exact(dev, case):
    hq, hkv, hs, pool, ratio, seqs = case
    D = 128
    g = I.gen(hq * 100 + len(seqs))
    N = sum(L for L, _, _ in seqs)
    q, k, v = I.grid(g, (N, hq, D)), I.grid(g, (N, hkv, D)), I.grid(g, (N, hkv, D))
    n_keeps = [R.num_keep(L - bl, ratio) for L, _, bl in seqs]
    pages = sum((n + 255) // 256 for n in n_keeps) + 2
    slots_list, off = [], 0
    order = torch.randperm(pages, generator=g).tolist()
    for n in n_keeps:
        npg = (n + 255) // 256
        lst = []
        for j, p in enumerate(order[off:off + npg]):
            lst.extend(range(p * 256, p * 256 + min(256, n - j * 256)))
        off += npg
        slots_list.append(torch.tensor(lst, dtype=torch.int32))
    kc_ref = torch.zeros(pages, 256, hkv, D)
    vc_ref = torch.zeros(pages, 256, hkv, D)
    ref_idx = []
    desc, row, slot_off, idx_off = [], 0, 0, 0
    for (L, b0, bl), n, sl in zip(seqs, n_keeps, slots_list):
        blk = torch.arange(row + b0, row + b0 + bl)
        allr = torch.arange(row, row + L)
        ps = allr[~torch.isin(allr, blk)]
        if hs:
            idx, ks, vs = R.select_important_head_kv(q[blk], k[ps], v[ps], hq, hkv, pool, ratio)
        else:
            idx = R.select_important_kv(q[blk], k[ps], hq, hkv, pool, ratio)
            ks, vs = k[ps][torch.from_numpy(idx)], v[ps][torch.from_numpy(idx)]
        R.store_kvcache(ks, vs, kc_ref, vc_ref, sl)
        ref_idx.append(idx)
        desc.append([row, L, b0, bl, n, slot_off, idx_off, pool])
        row += L
        slot_off += n
        idx_off += n * (hkv if hs else 1)
    t = lambda x: x.to(dev, torch.bfloat16)
    kc = torch.zeros(pages, 256, hkv, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    top = torch.full((idx_off,), -1, dtype=torch.int64, device=dev)
    _ops().select_kv_store(t(q), t(k), t(v), torch.tensor(desc, dtype=torch.int32, device=dev),
                           max(L - bl for L, _, bl in seqs), hs, kc, vc,
                           torch.cat(slots_list).to(dev), top)
    torch.cuda.synchronize()
    _status_clear(dev)
    top = top.cpu().numpy()
    for d, ri in zip(desc, ref_idx):
        n = d[4]
        got = top[d[6]:d[6] + n * (hkv if hs else 1)]
        assert np.array_equal(got.reshape(ri.shape), ri)
    assert torch.equal(kc.cpu().float(), kc_ref) and torch.equal(vc.cpu().float(), vc_ref)


@pytest.mark.parametrize("hq,hkv,hs", [(4, 4, True), (8, 2, False)])
def test_select_kv_store_slot_edges(dev, hq, hkv, hs):
    """A negative slot skips its selected row and a slot past the cache skips
    it and sets DLLM_DEV_SLOT_OUT_OF_RANGE; every other selected row lands as
    with valid slots, and the chosen indices do not change."""
    from dllmserve_b200 import _native

    D, L, b0, bl, ratio = 128, 200, 50, 32, 0.5
    g = I.gen(77 + hq)
    q, k, v = I.grid(g, (L, hq, D)), I.grid(g, (L, hkv, D)), I.grid(g, (L, hkv, D))
    n = R.num_keep(L - bl, ratio)
    pages = (n + 255) // 256 + 1
    num_slots = pages * 256
    good = torch.randperm(num_slots, generator=g)[:n].to(torch.int32)
    bad = good.clone()
    bad[3] = -1
    bad[7] = num_slots + 5
    t = lambda x: x.to(dev, torch.bfloat16)
    desc = torch.tensor([[0, L, b0, bl, n, 0, 0, 3]], dtype=torch.int32, device=dev)
    out = []
    for slots in (good, bad):
        kc = torch.zeros(pages, 256, hkv, D, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        top = torch.full((n * (hkv if hs else 1),), -1, dtype=torch.int64, device=dev)
        _status_clear(dev)
        _ops().select_kv_store(t(q), t(k), t(v), desc, L - bl, hs, kc, vc, slots.to(dev), top)
        torch.cuda.synchronize()
        out.append((kc.view(num_slots, -1).cpu(), vc.view(num_slots, -1).cpu(), top.cpu(),
                    _ops().read_device_status(dev)))
    (kg, vg, tg, sg), (kb, vb, tb, sb) = out
    assert sg == 0 and sb == _native.DLLM_DEV_SLOT_OUT_OF_RANGE
    assert torch.equal(tg, tb)
    keep = torch.ones(n, dtype=torch.bool)
    keep[3] = keep[7] = False
    rows = good[keep].long()
    assert torch.equal(kb[rows], kg[rows]) and torch.equal(vb[rows], vg[rows])
    skipped = good[~keep].long()
    assert not kb[skipped].any() and not vb[skipped].any()
    assert kg[skipped].any()  # the valid run did write those rows


@pytest.mark.parametrize("layout", ["pages", "random", "mixed"])
@pytest.mark.parametrize("hq,hkv", [(4, 4), (7, 1)])
def test_attention_paged_cache(dev, layout, hq, hkv):
    """keys = [cache rows at slots ; fresh rows], read straight from the paged cache
    (TMA for runs of consecutive slots, warp gather otherwise)."""
    g = I.gen(90 + hq + len(layout))
    D, pages = 128, 12
    lq = [32, 32, 17, 64]
    n_c = [304, 0, 129, 300]
    kc = I.normal(g, (pages, 256, hkv, D))
    vc = I.normal(g, (pages, 256, hkv, D))
    order = torch.randperm(pages, generator=g).tolist()
    slot_lists, off = [], 0
    for i, n in enumerate(n_c):
        if layout == "random" or (layout == "mixed" and i % 2 == 1):
            lst = torch.randperm(pages * 256, generator=g)[:n].tolist()
        else:
            npg = (n + 255) // 256
            lst = []
            for j, p in enumerate(order[off:off + npg]):
                lst.extend(range(p * 256, p * 256 + min(256, n - j * 256)))
            off += npg
        slot_lists.append(torch.tensor(lst, dtype=torch.int32))
    slots = torch.cat(slot_lists)
    q = I.normal(g, (sum(lq), hq, D))
    k, v = I.normal(g, (sum(lq), hkv, D)), I.normal(g, (sum(lq), hkv, D))
    kg, vg = R.load_kvcache(kc, vc, slots, hkv, D)
    ref = R.varlen_attention(q, k, v, _cu(lq), _cu(lq), D ** -0.5, kg, vg, _cu(n_c))
    t = lambda x: x.to(dev, torch.bfloat16)
    cq = torch.tensor(_cu(lq), dtype=torch.int32, device=dev)
    cs = torch.tensor(_cu(n_c), dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(t(q), t(k), t(v), cq, cq, max(lq), D ** -0.5,
                                  k_cache=t(kc), v_cache=t(vc), slots=slots.to(dev),
                                  cu_seqlens_slots=cs)
    _check_attn(out, ref, f"{layout} hq={hq} hkv={hkv}")
    _status_clear(dev)


def test_attention_paged_out_of_range_slot(dev):
    """An out-of-range slot reads as a zero key/value row and flags the status word."""
    g = I.gen(95)
    D, H = 128, 2
    kc = I.normal(g, (2, 256, H, D))
    vc = I.normal(g, (2, 256, H, D))
    slots = torch.tensor([3, 700, 5], dtype=torch.int32)  # 700 >= 512 slots
    q, k, v = I.normal(g, (4, H, D)), I.normal(g, (4, H, D)), I.normal(g, (4, H, D))
    kg, vg = R.load_kvcache(kc, vc, torch.tensor([3, 0, 5]), H, D)
    kg[1] = 0
    vg[1] = 0
    ref = R.varlen_attention(q, k, v, [0, 4], [0, 4], D ** -0.5, kg, vg, [0, 3])
    t = lambda x: x.to(dev, torch.bfloat16)
    c4 = torch.tensor([0, 4], dtype=torch.int32, device=dev)
    out = _ops().varlen_attention(t(q), t(k), t(v), c4, c4, 4, D ** -0.5, k_cache=t(kc),
                                  v_cache=t(vc), slots=slots.to(dev),
                                  cu_seqlens_slots=torch.tensor([0, 3], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert _ops().read_device_status(dev) == 1
    _check_attn(out, ref)
