"""GPU tests of the device-side step-metadata builder (dllm_build_step_plan):
on random batches of dense, compute-cache and reuse sequences (block lengths,
block indices, retention ratios, pool kernels, head_select both ways, several
KV-head counts) the plan built by one device launch equals the plan the host
assembles from the same per-sequence rules -- row offsets, cached-row
offsets, concatenated slot lists and selection descriptors -- and a wrong slot
count handed to the C ABI sets the device status word instead of faulting."""
import ctypes
import struct
import types

import pytest
import torch

from dllmserve_b200.engine.step_plan import build_step_plan, selection_arrays
from dllmserve_b200.sparse.state import SparseConfig
from test_host_logic import _Seq

pytestmark = pytest.mark.gpu


def _batch(rng, n):
    seqs, slots_cpu = [], []
    base = 0
    for _ in range(n):
        prompt = int(rng.integers(1, 301))
        blen = int(rng.choice([16, 32]))
        nblk = int(rng.integers(1, 5))
        state = rng.choice([None, 1, 2])
        bidx = min(int(rng.integers(0, 4)), nblk - 1)
        ratio = float(rng.choice([0.0, 0.25, 0.5, 0.6, 1.0]))
        pool = int(rng.choice([1, 3, 4, 5]))
        hs = bool(rng.integers(0, 2))
        if state is None:
            s = _Seq(prompt, blen * nblk, None)
            need = 0
        else:
            cfg = SparseConfig(enabled=True, default_block_len=blen, retention_ratio=ratio,
                               pool_kernel=pool, head_select=hs)
            s = _Seq(prompt, blen * nblk, cfg, state=int(state), block_idx=bidx)
            st = s.sparse_state
            b0, bl = st.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)
            from dllmserve_b200.sparse.state import num_keep

            need = num_keep(st.num_unused_tokens(s.num_prompt_tokens, s.num_tokens), ratio)
        seqs.append(s)
        slots_cpu.append(torch.randperm(4096)[:need].to(torch.int32) + base if need else [])
        base += 4096
    rows = 0
    for s in seqs:
        st = s.sparse_state
        rows += (st.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)[1]
                 if st is not None and st.cache_state == 2 else s.num_tokens)
    return seqs, slots_cpu, rows


def test_device_plan_equals_host_plan_on_random_batches():
    import numpy as np

    from dllmserve_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(7)
    checked = 0
    for trial in range(150):
        n = int(rng.integers(1, 40)) if trial % 10 else int(rng.integers(200, 1025))
        hkv = int(rng.choice([1, 2, 4, 8]))
        seqs, slots_cpu, rows = _batch(rng, n)
        ctx_h = types.SimpleNamespace(seqs=seqs, slot_mapping=slots_cpu)
        ctx_d = types.SimpleNamespace(seqs=seqs, slot_mapping=[s.to(dev) if isinstance(s, torch.Tensor) else s
                                                              for s in slots_cpu])
        host = build_step_plan(ctx_h, torch.device("cpu"), rows)
        devp = build_step_plan(ctx_d, dev, rows, hkv)
        torch.cuda.synchronize()
        assert ops.read_device_status(dev) == 0
        assert devp.cu.cpu().tolist() == host.cu.tolist()
        assert devp.max_rows == host.max_rows and devp.total_c == host.total_c
        if host.total_c:
            assert devp.cu_c.cpu().tolist() == host.cu_c.tolist()
            assert devp.slots_c.cpu().tolist() == host.slots_c.tolist()
        else:
            assert devp.cu_c is None and devp.slots_c is None
        for hs in (True, False):
            a = selection_arrays(host, hs, hkv, torch.device("cpu"))
            b = selection_arrays(devp, hs, hkv, dev)
            if a is None:
                assert b is None
                continue
            assert b[0].cpu().tolist() == a[0].tolist()
            assert b[1].cpu().tolist() == a[1].tolist()
            assert b[2:] == a[2:]
            checked += 1
    assert checked > 50


def test_device_plan_flags_wrong_slot_count():
    from dllmserve_b200 import _native, ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _native.lib()
    slots = torch.arange(100, dtype=torch.int32, device=dev)
    ratio = struct.unpack("<q", struct.pack("<d", 0.5))[0]
    # a compute-cache sequence of 96 tokens (block 64..95): n_keep = 32, but 100 slots given
    rows = torch.tensor([[1, 96, 64, 0, 32, ratio, 3 | (1 << 32), slots.data_ptr(), 100, 0]],
                        dtype=torch.int64, device=dev)
    B, D8 = 1, _native.SEQ_DESC_INTS
    layout = (ctypes.c_int64 * _native.PLAN_LAYOUT_INTS)(
        2 * (B + 1) + D8 + 32, B + 1, 2 * (B + 1), 1, 2 * (B + 1) + D8, 0,
        2 * (B + 1) + D8, 0, 2 * (B + 1) + D8, 32, 2 * (B + 1) + D8 + 32, 0)
    out = torch.full((2 * (B + 1) + D8 + 32,), -5, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.dllm_build_step_plan(rows.data_ptr(), B, 4, out.data_ptr(), layout, status.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == _native.DLLM_DEV_BAD_SEQUENCE
    assert out[2 * (B + 1) + D8:].tolist() == [-5] * 32  # nothing gathered from the mismatched list
    # an overlapping layout is refused on the host
    bad = (ctypes.c_int64 * _native.PLAN_LAYOUT_INTS)(*layout)
    bad[2] = 1
    assert lib.dllm_build_step_plan(rows.data_ptr(), B, 4, out.data_ptr(), bad, status.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream) == _native.DLLM_ERR_INVALID_ARG
    assert ops.read_device_status(dev, reset=True) in (0, _native.DLLM_DEV_BAD_SEQUENCE)
