"""CPU tests of the host-side logic: sparse state machine vs the reference's
traces, per-step metadata (StepPlan), context API, tensor-parallel slicing."""
import json
import os
import types

import pytest
import torch

import cases as C
from dllmserve_b200.engine.step_plan import (STATE_COMPUTE, STATE_DENSE, STATE_REUSE,
                                             build_step_plan, selection_arrays)
from dllmserve_b200.sparse.state import PerRequestSparseState, SparseConfig, num_keep
from dllmserve_b200.tp import head_slice
from dllmserve_b200.utils import context as ctxmod


def test_sparse_config_defaults_match_reference_code():
    c = SparseConfig()
    assert (c.enabled, c.default_block_len, c.retention_ratio, c.pool_kernel, c.delay_step,
            c.head_select) == (False, 32, 0.5, 3, 1, False)


def test_state_machine_matches_reference_traces(golden_dir):
    traces = json.load(open(os.path.join(golden_dir, "golden_meta.json")))["state_traces"]
    for (delay, blen, prompt, gen_len, n), rows in zip(C.STATE_TRACES, traces):
        st = PerRequestSparseState(0, SparseConfig(enabled=True, default_block_len=blen,
                                                   delay_step=delay), torch.device("cpu"))
        L = prompt + gen_len
        for cache_state, bidx, sib, bs, bl, n_keep in rows:
            assert (st.cache_state, st.current_block_idx, st.step_in_block) == (cache_state, bidx, sib)
            assert st.compute_block_boundaries(prompt, L) == (bs, bl)
            assert num_keep(st.num_unused_tokens(prompt, L), 0.5) == n_keep
            assert len(st.get_unuse_block_indices(prompt, L)) == st.num_unused_tokens(prompt, L)
            st.advance_step()


def test_disabled_state_still_advances():
    st = PerRequestSparseState(0, SparseConfig(enabled=False), "cpu")
    st.advance_step()
    assert st.cache_state == 1 and st.get_cache_state() == 0


def test_num_keep_edges():
    assert num_keep(0, 0.5) == 0
    assert num_keep(1, 0.5) == 1
    assert num_keep(10, 0.0) == 1
    assert num_keep(10, 1.0) == 10
    assert num_keep(608, 0.5) == 304
    assert num_keep(4576, 0.25) == 1144


class _Seq:
    def __init__(self, prompt, gen, cfg=None, state=0, block_idx=0):
        self.num_prompt_tokens = prompt
        self.num_tokens = prompt + gen
        self.sparse_state = None
        if cfg is not None:
            self.sparse_state = PerRequestSparseState(0, cfg, "cpu")
            self.sparse_state.cache_state = state
            self.sparse_state.current_block_idx = block_idx


def test_step_plan_mixed_batch():
    hs = SparseConfig(enabled=True, head_select=True, pool_kernel=3)
    sh = SparseConfig(enabled=True, head_select=False, pool_kernel=5, retention_ratio=0.25)
    seqs = [_Seq(100, 64, None), _Seq(40, 32, hs, state=1), _Seq(80, 64, hs, state=2, block_idx=1),
            _Seq(70, 32, sh, state=1)]
    n1 = num_keep(72 - 32, 0.5)
    n2 = num_keep(144 - 32, 0.5)
    n3 = num_keep(102 - 32, 0.25)
    slots = [[], torch.arange(n1, dtype=torch.int32), torch.arange(n2, dtype=torch.int32) + 1000,
             torch.arange(n3, dtype=torch.int32) + 2000]
    rows = 164 + 72 + 32 + 102
    ctx = types.SimpleNamespace(seqs=seqs, slot_mapping=slots)
    plan = build_step_plan(ctx, torch.device("cpu"), rows)
    assert [i.state for i in plan.infos] == [STATE_DENSE, STATE_COMPUTE, STATE_REUSE, STATE_COMPUTE]
    assert plan.cu.tolist() == [0, 164, 236, 268, 370]
    assert plan.max_rows == 164
    assert plan.k_lens == [164, 72, 32 + n2, 102]
    assert plan.cu_c.tolist() == [0, 0, 0, n2, n2]
    assert plan.slots_c.tolist() == list(range(1000, 1000 + n2))
    desc, sl, max_klen, total = selection_arrays(plan, True, 4, torch.device("cpu"))
    assert desc.tolist() == [[164, 72, 40, 32, n1, 0, 0, 3]]
    assert max_klen == 40 and total == 4 * n1
    desc, sl, max_klen, total = selection_arrays(plan, False, 4, torch.device("cpu"))
    assert desc.tolist() == [[268, 102, 70, 32, n3, 0, 0, 5]]
    assert sl.tolist() == list(range(2000, 2000 + n3))


def test_step_plan_rejects_inconsistent_inputs():
    hs = SparseConfig(enabled=True, head_select=True)
    seqs = [_Seq(40, 32, hs, state=1)]
    ctx = types.SimpleNamespace(seqs=seqs, slot_mapping=[torch.arange(3, dtype=torch.int32)])
    with pytest.raises(ValueError, match="slot_mapping"):
        build_step_plan(ctx, torch.device("cpu"), 72)
    ctx = types.SimpleNamespace(seqs=seqs, slot_mapping=[torch.arange(20, dtype=torch.int32)])
    with pytest.raises(ValueError, match="rows"):
        build_step_plan(ctx, torch.device("cpu"), 71)
    bad = _Seq(40, 32, hs, state=1)
    bad.sparse_state.cache_state = 7
    with pytest.raises(ValueError, match="unrecognized"):
        build_step_plan(types.SimpleNamespace(seqs=[bad], slot_mapping=[[]]), torch.device("cpu"), 72)


def test_context_api_roundtrip():
    ctxmod.set_context(True, cu_seqlens_k=torch.tensor([0, 3]), is_diffusion=True, seqs=[1])
    c = ctxmod.get_context()
    assert c.is_prefill and c.is_diffusion and c.seqs == [1] and c.max_seqlen_q == 0
    ctxmod.reset_context()
    assert not ctxmod.get_context().is_diffusion


def test_head_slice():
    assert head_slice(32, 32, 1, 4) == (8, 16, 8, 16)
    assert head_slice(28, 4, 3, 4) == (21, 28, 3, 4)
    with pytest.raises(ValueError):
        head_slice(28, 4, 0, 8)  # Dream's 4 KV heads do not split 8 ways


def test_step_plan_matches_oracle_rules_on_random_batches():
    """Property test: for random batches of dense, compute-cache and reuse
    sequences, the step plan's rows, offsets, cached-row counts, slot order and
    selection descriptors equal those the oracle's restatement of the
    reference's per-sequence rules (SeqMeta, attention.py:168-304) gives."""
    hypothesis = pytest.importorskip("hypothesis")
    from hypothesis import given, settings, strategies as st
    from oracle import attention_ref as R

    seq_st = st.tuples(
        st.integers(1, 300),                      # prompt length
        st.sampled_from([16, 32]),                # block length
        st.integers(1, 4),                        # generated blocks
        st.sampled_from([None, 1, 2]),            # None: no sparse state (dense); else cache state
        st.integers(0, 3),                        # current block index (clamped below)
        st.sampled_from([0.0, 0.25, 0.5, 1.0]),   # retention ratio
        st.sampled_from([1, 3, 4, 5]),            # pool kernel
        st.booleans(),                            # head_select
    )

    @settings(max_examples=200, deadline=None)
    @given(st.lists(seq_st, min_size=1, max_size=8), st.sampled_from([1, 2, 4, 8]))
    def check(specs, hkv):
        seqs, metas, slots = [], [], []
        base = 0
        for prompt, blen, nblk, state, bidx, ratio, pool, hs in specs:
            gen = blen * nblk
            bidx = min(bidx, nblk - 1)
            if state is None:
                s = _Seq(prompt, gen, None)
                m = R.SeqMeta(state=0, num_tokens=prompt + gen, prompt_len=prompt)
            else:
                cfg = SparseConfig(enabled=True, default_block_len=blen, retention_ratio=ratio,
                                   pool_kernel=pool, head_select=hs)
                s = _Seq(prompt, gen, cfg, state=state, block_idx=bidx)
                m = R.SeqMeta(state=state, num_tokens=prompt + gen, prompt_len=prompt, block_idx=bidx,
                              block_len=blen, ratio=ratio, pool_kernel=pool, head_select=hs)
            n = m.n_keep() if m.state else 0
            slots.append(torch.arange(base, base + n, dtype=torch.int32) if m.state else [])
            base += n
            seqs.append(s)
            metas.append(m)
        rows = sum(m.rows() for m in metas)
        plan = build_step_plan(types.SimpleNamespace(seqs=seqs, slot_mapping=slots), torch.device("cpu"), rows)
        cu = [0]
        for m in metas:
            cu.append(cu[-1] + m.rows())
        assert plan.cu.tolist() == cu
        assert plan.max_rows == max(m.rows() for m in metas)
        reuse = [i for i, m in enumerate(metas) if m.state == 2]
        if reuse:
            cc = [0]
            for m in metas:
                cc.append(cc[-1] + (m.n_keep() if m.state == 2 else 0))
            assert plan.cu_c.tolist() == cc
            assert plan.slots_c.tolist() == [x for i in reuse for x in slots[i].tolist()]
        else:
            assert plan.cu_c is None and plan.total_c == 0
        for hs in (True, False):
            idx = [i for i, m in enumerate(metas) if m.state == 1 and m.head_select == hs]
            arrs = selection_arrays(plan, hs, hkv, torch.device("cpu"))
            if not idx:
                assert arrs is None
                continue
            desc, sl, max_klen, total = arrs
            want, slot_off, idx_off = [], 0, 0
            for i in idx:
                m = metas[i]
                bs, bl = m.block()
                want.append([cu[i], m.num_tokens, bs, bl, m.n_keep(), slot_off, idx_off, m.pool_kernel])
                slot_off += m.n_keep()
                idx_off += m.n_keep() * (hkv if hs else 1)
            assert desc.tolist() == want
            assert total == idx_off
            assert max_klen == max(metas[i].num_tokens - metas[i].block()[1] for i in idx)
            assert sl.tolist() == [x for i in idx for x in slots[i].tolist()]

    check()
