"""Importance selection (scores, max-pool, top-k, gather into the paged
cache) at the sizes of BASELINE configs 3 and 4.

CPU (pins the oracle at this scale): on margin-separated N(0,1) inputs
(inputs.margin_selection_batch) the oracle -- in its float64-rounded form and
in the GPU kernel's fp32 summation order -- selects what the reference's own
Attention.forward selected (tests/golden/selection_*.npz, recorded by
tests/golden/make_golden.py), index for index up to the documented tie rule.

GPU (-m gpu, through the C ABI via ops.select_kv_store):
  * config 3 as specified (B=8, 512+128 tokens, 32/32 heads, r=0.5,
    head_select, pool 3, margin keys with 4 heads' keys scaled 3x) and config 4
    (Dream 28/4, B=32, U[128,768]+256, r=0.5) in both head_select modes:
    top_idx and the written cache rows bit-exact against the oracle and the
    reference's recorded indices;
  * the same shapes on plain N(0,1) data (no margins): top_idx and cache rows
    bit-exact against the oracle restated in the kernel's fp32 summation
    order (on such data a different order can flip near-ties, so only the
    order-matched restatement is a bit-exact reference).
"""
import os

import numpy as np
import pytest
import torch

import cases as C
import inputs as I
from oracle import attention_ref as R

BLK = 32


def _fixture(golden_dir, name):
    return np.load(os.path.join(golden_dir, f"selection_{name}.npz"))


def canonical(idx, scores):
    """Indices ordered by descending score, ties by ascending index."""
    key = np.lexsort((idx, -scores[idx].astype(np.float64)))
    return idx[key]


def topk_equivalent(ref_idx, ours, scores):
    """Same selected multiset; identical (canonical) indices above the cutoff;
    the cutoff's tie group drawn alike in count (torch.topk leaves its choice
    unspecified)."""
    assert len(ref_idx) == len(ours)
    v_ref = np.sort(scores[ref_idx])[::-1]
    v_our = np.sort(scores[ours])[::-1]
    assert np.array_equal(v_ref, v_our)
    cutoff = v_our[-1]
    m = int((scores[ours] > cutoff).sum())
    assert (scores > cutoff).sum() == m
    assert np.array_equal(canonical(ref_idx, scores)[:m], ours[:m])


def _sequences(prompts, lens):
    """(row offset, prompt, L) per sequence; the block is the first
    generation block [prompt, prompt + 32)."""
    out, off = [], 0
    for p, L in zip(prompts, lens):
        out.append((off, p, L))
        off += L
    return out


def _cand(off, p, L):
    return torch.cat([torch.arange(off, off + p), torch.arange(off + p + BLK, off + L)])


def _oracle_selection(case, q, k, prompts, lens, kernel_order):
    """Per sequence: (pooled scores [rows, Klen], top_idx [Hkv or 1, n_keep])."""
    res = []
    for off, p, L in _sequences(prompts, lens):
        qb = q[off + p:off + p + BLK]
        kc = k[_cand(off, p, L)]
        H, Hk = case.num_heads, case.num_kv_heads
        if kernel_order:
            s = (R.head_scores_kernel_order(qb, kc, H, Hk) if case.head_select
                 else R.shared_scores_kernel_order(qb, kc, H, Hk)[None])
        else:
            s = R.head_scores(qb, kc, H, Hk) if case.head_select else R.shared_scores(qb, kc, H, Hk)[None]
        s = R.max_pool(s, case.pool_kernel)
        idx = R.topk_desc(s, R.num_keep(L - BLK, case.retention_ratio))
        res.append((s, idx))
    return res


@pytest.mark.parametrize("case", C.SELECTION_CASES, ids=[c.name for c in C.SELECTION_CASES])
def test_oracle_selection_matches_reference_at_scale(case, golden_dir):
    fx = _fixture(golden_dir, case.name)
    q, k, v, prompts, lens = I.margin_selection_batch(case)
    assert np.allclose(fx["input_checksums"], I.checksum(q) + I.checksum(k) + I.checksum(v), rtol=1e-12)
    assert fx["lens"].tolist() == lens
    std = _oracle_selection(case, q, k, prompts, lens, kernel_order=False)
    ko = _oracle_selection(case, q, k, prompts, lens, kernel_order=True)
    for i, ((s, idx), (_, idx_k)) in enumerate(zip(std, ko)):
        # margin-separated inputs: both summation orders select the same indices
        assert np.array_equal(idx, idx_k), i
        ref = fx[f"top_idx_{i}"].astype(np.int64).reshape(idx.shape)
        assert idx.shape[1] == int(fx["n_keep"][i])
        for h in range(idx.shape[0]):
            topk_equivalent(ref[h], idx[h], s[h])


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _plain_normal_batch(case, seed):
    """Same shapes as the case, plain N(0,1) q/k/v (bf16 values)."""
    g = I.gen(seed)
    prompts = I.selection_prompts(case)
    lens = [p + case.gen_len for p in prompts]
    N = sum(lens)
    return (I.normal(g, (N, case.num_heads, 128)), I.normal(g, (N, case.num_kv_heads, 128)),
            I.normal(g, (N, case.num_kv_heads, 128)), prompts, lens)


def _run_kernel(case, q, k, v, prompts, lens, dev):
    from dllmserve_b200 import ops

    Hk = case.num_kv_heads
    seqs = _sequences(prompts, lens)
    n_keeps = [R.num_keep(L - BLK, case.retention_ratio) for _, _, L in seqs]
    desc, slots, slot_off, idx_off, page = [], [], 0, 0, 0
    for (off, p, L), nk in zip(seqs, n_keeps):
        desc.append([off, L, p, BLK, nk, slot_off, idx_off, case.pool_kernel])
        # pages in reverse order so the cache layout is not the identity
        slots.append(torch.arange(page * 256, page * 256 + nk, dtype=torch.int32))
        page += (nk + 255) // 256
        slot_off += nk
        idx_off += nk * (Hk if case.head_select else 1)
    pages = page + 1
    slots = torch.cat(slots)
    slots = (pages - 1) * 256 - 1 - slots  # distinct slots, reversed
    kc = torch.zeros(pages, 256, Hk, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    top = torch.full((idx_off,), -7, dtype=torch.int64, device=dev)
    ops.select_kv_store(q.to(dev, torch.bfloat16), k.to(dev, torch.bfloat16), v.to(dev, torch.bfloat16),
                        torch.tensor(desc, dtype=torch.int32, device=dev), max(L - BLK for L in lens),
                        case.head_select, kc, vc, slots.to(dev), top)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 0
    rows = Hk * 128
    return (top.cpu().numpy(), kc.view(-1, rows).cpu().float(), vc.view(-1, rows).cpu().float(),
            slots, n_keeps, desc)


def _check_kernel(case, q, k, v, prompts, lens, oracle, fixture=None):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    top, kc, vc, slots, n_keeps, desc = _run_kernel(case, q, k, v, prompts, lens, dev)
    Hk = case.num_kv_heads
    for i, ((off, p, L), nk, d) in enumerate(zip(_sequences(prompts, lens), n_keeps, desc)):
        s, idx = oracle[i]
        n_rows = Hk if case.head_select else 1
        got = top[d[6]:d[6] + n_rows * nk].reshape(n_rows, nk)
        assert np.array_equal(got, idx), (case.name, i)
        if fixture is not None:
            ref = fixture[f"top_idx_{i}"].astype(np.int64).reshape(idx.shape)
            for h in range(n_rows):
                topk_equivalent(ref[h], got[h], s[h])
        cand = _cand(off, p, L)
        sl = slots[d[5]:d[5] + nk].long()
        for h in range(Hk):
            sel = cand[torch.from_numpy(idx[h if case.head_select else 0])]
            assert torch.equal(kc[sl, h * 128:(h + 1) * 128], k[sel, h]), (case.name, i, h)
            assert torch.equal(vc[sl, h * 128:(h + 1) * 128], v[sel, h]), (case.name, i, h)


@pytest.mark.gpu
@pytest.mark.parametrize("case", C.SELECTION_CASES, ids=[c.name for c in C.SELECTION_CASES])
def test_kernel_selection_margin_inputs_bit_exact(case, golden_dir):
    q, k, v, prompts, lens = I.margin_selection_batch(case)
    oracle = _oracle_selection(case, q, k, prompts, lens, kernel_order=False)
    _check_kernel(case, q, k, v, prompts, lens, oracle, _fixture(golden_dir, case.name))


@pytest.mark.gpu
@pytest.mark.parametrize("case", C.SELECTION_CASES, ids=[c.name for c in C.SELECTION_CASES])
def test_kernel_selection_plain_normal_bit_exact(case):
    q, k, v, prompts, lens = _plain_normal_batch(case, 700 + case.seed)
    oracle = _oracle_selection(case, q, k, prompts, lens, kernel_order=True)
    _check_kernel(case, q, k, v, prompts, lens, oracle)
