"""GPU tests of dllm_attn_varlen_fwd_static_ws, the attention entry point for
callers that cannot allocate device memory (a plugin whose host application
owns all device memory, or a launch loop that must not call cudaMalloc because
it can synchronise the device). Its scheduler workspace is a static array of
the library instead of a caller buffer.

Checked through the C ABI: two calls in a row write the same output bits as
dllm_attn_varlen_fwd with a caller workspace (and as the round-robin order)
and agree with the CPU oracle within the attention tolerance; a launch of
another shape afterwards is still correct (each call clears the static words
on its stream, and the kernel leaves them at zero); the short-query path (max_seqlen_q <= 128) gives the same result as
the caller-workspace entry. This file sorts last, so a run that stops at the
first failure has run every other test before it, and it also passes alone
in a fresh process.
"""
import ctypes

import pytest
import torch

import inputs as I

pytestmark = pytest.mark.gpu

D = 128
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3


def _cu(lens):
    c = [0]
    for L in lens:
        c.append(c[-1] + L)
    return c


def _setup():
    from dllmserve_b200 import _native

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    return _native, _native.lib(), dev


def _case(seed, lens, H, Hk, dev):
    g = I.gen(seed)
    N = sum(lens)
    q, k, v = I.normal(g, (N, H, D)), I.normal(g, (N, Hk, D)), I.normal(g, (N, Hk, D))
    cu = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    return (q, k, v), tuple(t.to(dev, torch.bfloat16) for t in (q, k, v)), cu


def _call(lib, fn, dev_qkv, cu, lens, H, Hk, status, *ws):
    q, k, v = dev_qkv
    N = q.shape[0]
    o = torch.full_like(q, float("nan"))
    rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
            o.data_ptr(), o.stride(0), cu.data_ptr(), cu.data_ptr(), len(lens), max(lens), N, N,
            H, Hk, D, ctypes.c_float(D ** -0.5), *ws, status.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.dllm_last_error()
    return o


def _check_oracle(cpu_qkv, out, lens, seqs):
    from oracle import attention_ref as R

    q, k, v = cpu_qkv
    cu = _cu(lens)
    for b in seqs:
        sl = slice(cu[b], cu[b + 1])
        ref = R.varlen_attention(q[sl], k[sl], v[sl], [0, lens[b]], [0, lens[b]], D ** -0.5)
        err = (out[sl].float().cpu() - ref).abs()
        assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, (b, float(err.max()), float(err.mean()))


def test_static_workspace_matches_caller_workspace_and_oracle():
    native, lib, dev = _setup()
    H = 8
    lens = [419, 1087, 700, 130, 900, 256, 555, 1000, 3]  # > 128 rows: the pair kernel
    cpu_qkv, dq, cu = _case(150, lens, H, H, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(native.SCHED_WORKSPACE_INTS, dtype=torch.int32, device=dev)
    ref = _call(lib, lib.dllm_attn_varlen_fwd, dq, cu, lens, H, H, status, ws.data_ptr())
    rr = _call(lib, lib.dllm_attn_varlen_fwd, dq, cu, lens, H, H, status, None)
    first = _call(lib, lib.dllm_attn_varlen_fwd_static_ws, dq, cu, lens, H, H, status)
    second = _call(lib, lib.dllm_attn_varlen_fwd_static_ws, dq, cu, lens, H, H, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert int(ws.abs().sum()) == 0
    assert torch.isfinite(ref.float()).all()
    assert torch.equal(rr, ref)
    assert torch.equal(first, ref)
    assert torch.equal(second, ref)
    _check_oracle(cpu_qkv, second, lens, seqs=[0, 3, 8])

    # Another shape (GQA, more units than SMs) right after: every output row is
    # written, which needs the static words back at zero from the calls above.
    lens2 = [1500, 260, 777, 1200, 129, 2048]
    cpu2, dq2, cu2 = _case(151, lens2, 28, 4, dev)
    ref2 = _call(lib, lib.dllm_attn_varlen_fwd, dq2, cu2, lens2, 28, 4, status, ws.data_ptr())
    third = _call(lib, lib.dllm_attn_varlen_fwd_static_ws, dq2, cu2, lens2, 28, 4, status)
    fourth = _call(lib, lib.dllm_attn_varlen_fwd_static_ws, dq, cu, lens, H, H, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(third, ref2)
    assert torch.equal(fourth, ref)
    _check_oracle(cpu2, third, lens2, seqs=[1, 4])


def test_static_workspace_short_queries():
    """max_seqlen_q <= 128 (the reuse steps' blocks) runs the split kernel,
    which schedules round-robin; the entry point gives the same bits."""
    native, lib, dev = _setup()
    lens = [32, 128, 77, 1, 96] * 6
    cpu_qkv, dq, cu = _case(152, lens, 8, 8, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(native.SCHED_WORKSPACE_INTS, dtype=torch.int32, device=dev)
    ref = _call(lib, lib.dllm_attn_varlen_fwd, dq, cu, lens, 8, 8, status, ws.data_ptr())
    a = _call(lib, lib.dllm_attn_varlen_fwd_static_ws, dq, cu, lens, 8, 8, status)
    b = _call(lib, lib.dllm_attn_varlen_fwd_static_ws, dq, cu, lens, 8, 8, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(a, ref) and torch.equal(b, ref)
    _check_oracle(cpu_qkv, a, lens, seqs=[0, 1, 3])


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two devices")
def test_static_workspace_rejects_stream_of_other_device():
    native, lib, dev = _setup()
    lens = [200]
    _, dq, cu = _case(153, lens, 8, 8, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    other = torch.cuda.Stream(device=torch.device("cuda:1"))
    q, k, v = dq
    o = torch.empty_like(q)
    rc = lib.dllm_attn_varlen_fwd_static_ws(
        q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
        o.data_ptr(), o.stride(0), cu.data_ptr(), cu.data_ptr(), 1, 200, 200, 200, 8, 8, D,
        ctypes.c_float(D ** -0.5), status.data_ptr(), other.cuda_stream)
    assert rc == native.DLLM_ERR_INVALID_ARG
    assert b"stream" in lib.dllm_last_error()
