"""GPU test of dllm_attn_varlen_fwd_static_ws: the pair attention kernel with its
scheduler workspace in the library's static device memory instead of a caller
buffer. Two calls in a row must write the same output bits as
dllm_attn_varlen_fwd with a caller workspace (and as the round-robin order),
and report no device error. This file sorts last so it also runs after every
other GPU test has used the library.
"""
import ctypes

import pytest
import torch

import inputs as I

pytestmark = pytest.mark.gpu


def _cu(lens):
    c = [0]
    for L in lens:
        c.append(c[-1] + L)
    return c


def test_static_workspace_matches_caller_workspace():
    from dllmserve_b200 import _native

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _native.lib()
    g = I.gen(150)
    D, H = 128, 8
    lens = [419, 1087, 700, 130, 900, 256, 555, 1000, 3]  # > 128 rows: the pair kernel
    N = sum(lens)
    q, k, v = (I.normal(g, (N, H, D)).to(dev, torch.bfloat16) for _ in range(3))
    cu = torch.tensor(_cu(lens), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    scale = ctypes.c_float(D ** -0.5)

    def call(fn, *ws):
        o = torch.full_like(q, float("nan"))
        rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                o.data_ptr(), o.stride(0), cu.data_ptr(), cu.data_ptr(), len(lens), max(lens), N, N,
                H, H, D, scale, *ws, status.data_ptr(), stream)
        assert rc == 0, lib.dllm_last_error()
        return o

    ws = torch.zeros(_native.SCHED_WORKSPACE_INTS, dtype=torch.int32, device=dev)
    ref = call(lib.dllm_attn_varlen_fwd, ws.data_ptr())
    rr = call(lib.dllm_attn_varlen_fwd, None)
    first = call(lib.dllm_attn_varlen_fwd_static_ws)
    second = call(lib.dllm_attn_varlen_fwd_static_ws)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert int(ws.abs().sum()) == 0
    assert torch.isfinite(ref.float()).all()
    assert torch.equal(rr, ref)
    assert torch.equal(first, ref)
    assert torch.equal(second, ref)
