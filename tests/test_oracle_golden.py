"""Pins the CPU oracle (oracle/attention_ref.py) to golden vectors produced by
the reference's own attention module (tests/golden/make_golden.py)."""
import json
import os

import numpy as np
import pytest
import torch

import cases as C
import inputs as I
from oracle import attention_ref as R

ATOL = 2e-3  # golden outputs are stored as fp16


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def canonical(idx: np.ndarray, scores: np.ndarray) -> np.ndarray:
    """Order indices by (descending score, ascending index). torch.topk leaves
    the order of exactly-equal scores unspecified; this is the tie rule the
    oracle and the kernels use, so the reference's order is compared after it."""
    keys = scores[idx]
    order = np.lexsort((idx, -keys.astype(np.float64)))
    return idx[order]


def test_c1_rope_dense_attention_matches_reference(golden_dir):
    c = C.C1
    gold = _load(golden_dir, "c1.npz")
    g = I.gen(c["seed"])
    L = c["prompt_len"] + c["gen_len"]
    H, D = c["num_heads"], c["head_dim"]
    q, k, v = (torch.randn((L, H, D), generator=g) for _ in range(3))
    got = np.array(I.checksum(q) + I.checksum(k) + I.checksum(v))
    assert np.allclose(got, gold["input_checksums"]), f"input checksums {got} vs {gold['input_checksums']}"
    cache = R.rope_cache(D, L, c["rope_theta"])
    pos = torch.arange(L)
    qr, kr = R.apply_rope(q, pos, cache), R.apply_rope(k, pos, cache)
    got = np.array(I.checksum(qr) + I.checksum(kr))
    assert np.allclose(got, gold["rope_checksums"], rtol=1e-6), (
        f"rope checksums {got} vs {gold['rope_checksums']}")
    out = R.varlen_attention(qr, kr, v, [0, L], [0, L], D ** -0.5)
    err = np.abs(out.numpy() - gold["out"].astype(np.float32))
    assert err.max() < ATOL, (f"max abs error {err.max():.3e} at {np.unravel_index(err.argmax(), err.shape)}, "
                              f"torch threads {torch.get_num_threads()}")


def _build_step(case, g, step):
    """Mirror make_golden.py's sequence set-up with oracle SeqMeta records."""
    metas = []
    for sp in case.seqs:
        state = 0 if not sp.sparse else step
        metas.append(R.SeqMeta(state=state, num_tokens=sp.prompt_len + sp.gen_len,
                               prompt_len=sp.prompt_len, block_idx=sp.block_idx,
                               block_len=case.block_len, ratio=case.retention_ratio,
                               pool_kernel=case.pool_kernel, head_select=case.head_select))
    return metas


@pytest.mark.parametrize("case", C.SPARSE_CASES, ids=[c.name for c in C.SPARSE_CASES])
def test_sparse_case_matches_reference(case, golden_dir):
    gold = _load(golden_dir, f"sparse_{case.name}.npz")
    meta = json.load(open(os.path.join(golden_dir, "golden_meta.json")))["cases"][case.name]
    g = I.gen(case.seed)
    H, Hk, D = case.num_heads, case.num_kv_heads, case.head_dim
    torch.randperm(case.num_pages, generator=g)  # page order draw (slots come from meta)
    slots = [torch.tensor(meta["slots"][str(i)], dtype=torch.int32) for i in range(len(case.seqs))]
    kc = torch.zeros(case.num_pages, 256, Hk, D)
    vc = torch.zeros(case.num_pages, 256, Hk, D)

    seqs1 = _build_step(case, g, 1)
    assert [s.n_keep() if s.state else 0 for s in seqs1] == [
        n if sp.sparse else 0 for n, sp in zip(meta["n_keep"], case.seqs)]
    N1 = sum(s.rows() for s in seqs1)
    q1, k1, v1 = (I.make(case.kind, g, (N1, h, D)) for h in (H, Hk, Hk))
    rec = {}
    out1 = R.diffusion_layer(q1, k1, v1, seqs1, kc, vc, slots, D ** -0.5, H, Hk, record=rec)
    assert np.abs(out1.numpy() - gold["out1"].astype(np.float32)).max() < ATOL

    # selected indices: equivalent top-k (see topk_equivalent)
    row = 0
    ref_sel = {}
    for i, s in enumerate(seqs1):
        n = s.rows()
        if s.state == 1 and f"top_idx_{i}" in gold.files:
            ref_idx = gold[f"top_idx_{i}"]
            ref_sel[i] = ref_idx
            ours = rec[i]
            b0, bl = s.block()
            blk = torch.arange(row + b0, row + b0 + bl)
            allr = torch.arange(row, row + n)
            ps = allr[~torch.isin(allr, blk)]
            if case.head_select:
                sc = R.max_pool(R.head_scores(q1[blk], k1[ps], H, Hk), case.pool_kernel)
                for h in range(Hk):
                    topk_equivalent(ref_idx[h], ours[h], sc[h])
            else:
                sc = R.max_pool(R.shared_scores(q1[blk], k1[ps], H, Hk), case.pool_kernel)
                topk_equivalent(ref_idx, ours, sc)
        row += n

    # cache contents: the reference's rows equal the oracle's gather/store of
    # the reference's own indices into the same slots (bit-exact)
    all_slots = torch.from_numpy(gold["all_slots"]).long()
    rows = Hk * D
    kc_ref = torch.zeros_like(kc)
    vc_ref = torch.zeros_like(vc)
    row = 0
    for i, s in enumerate(seqs1):
        n = s.rows()
        if i in ref_sel:
            b0, bl = s.block()
            blk = torch.arange(row + b0, row + b0 + bl)
            allr = torch.arange(row, row + n)
            ps = allr[~torch.isin(allr, blk)]
            idx = torch.from_numpy(ref_sel[i])
            if case.head_select:
                e = idx.unsqueeze(-1).expand(-1, -1, D)
                ks = torch.gather(k1[ps].permute(1, 0, 2), 1, e).transpose(0, 1)
                vs = torch.gather(v1[ps].permute(1, 0, 2), 1, e).transpose(0, 1)
            else:
                ks, vs = k1[ps][idx], v1[ps][idx]
            R.store_kvcache(ks, vs, kc_ref, vc_ref, slots[i])
        row += n
    # (rows are stored as fp16 in the fixture; compare at that precision)
    assert np.array_equal(kc_ref.view(-1, rows)[all_slots].numpy().astype(np.float16),
                          gold["kcache_rows"])
    assert np.array_equal(vc_ref.view(-1, rows)[all_slots].numpy().astype(np.float16),
                          gold["vcache_rows"])
    assert np.isclose(float(kc_ref.abs().sum()), gold["cache_abs_sum"][0], rtol=1e-6)

    # reuse step on the reference's cache
    seqs2 = _build_step(case, g, 2)
    N2 = sum(s.rows() for s in seqs2)
    q2, k2, v2 = (I.make(case.kind, g, (N2, h, D)) for h in (H, Hk, Hk))
    out2 = R.diffusion_layer(q2, k2, v2, seqs2, kc_ref, vc_ref, slots, D ** -0.5, H, Hk)
    assert np.abs(out2.numpy() - gold["out2"].astype(np.float32)).max() < ATOL


def topk_equivalent(ref_idx: np.ndarray, ours: np.ndarray, scores: np.ndarray) -> None:
    """Both are valid top-k selections of ``scores`` and agree wherever the
    answer is unique: the same multiset of selected scores, the same indices
    (in canonical order) for every score above the cutoff, and for the
    cutoff's tie group (where torch.topk's choice is unspecified) the same
    count drawn from that group."""
    assert len(ref_idx) == len(ours)
    if len(ours) == 0:
        return
    v_ref = np.sort(scores[ref_idx])[::-1]
    v_our = np.sort(scores[ours])[::-1]
    assert np.array_equal(v_ref, v_our)
    cutoff = v_our[-1]
    assert (scores > cutoff).sum() == (scores[ours] > cutoff).sum()  # nothing larger left out
    m = int((scores[ours] > cutoff).sum())
    assert np.array_equal(canonical(ref_idx, scores)[:m], ours[:m])
    assert np.all(scores[ref_idx[scores[ref_idx] == cutoff]] == cutoff)


def test_state_traces_match_reference(golden_dir):
    """Oracle block geometry + sizing vs the reference's state machine traces."""
    traces = json.load(open(os.path.join(golden_dir, "golden_meta.json")))["state_traces"]
    for (delay, blen, prompt, gen_len, n), rows in zip(C.STATE_TRACES, traces):
        L = prompt + gen_len
        for cache_state, bidx, sib, bs, bl, n_keep in rows:
            assert R.block_boundaries(prompt, L, bidx, blen) == (bs, bl)
            assert R.num_keep(L - bl, 0.5) == n_keep


def test_topk_tie_rule():
    s = np.array([1.0, 3.0, 3.0, 2.0, 3.0, -1.0], np.float32)
    assert R.topk_desc(s, 4).tolist() == [1, 2, 4, 3]


def test_max_pool_matches_torch():
    g = I.gen(3)
    for pk in (1, 2, 3, 4, 5, 7):
        for klen in (1, 2, 3, 10, 33):
            s = torch.randn(3, klen, generator=g)
            ref = s
            if pk > 1:
                ref = torch.nn.functional.max_pool1d(s.unsqueeze(1), pk, 1, pk // 2).squeeze(1)[..., :klen]
            assert np.array_equal(R.max_pool(s.numpy(), pk), ref.numpy()), (pk, klen)
