"""GPU tests of the fused row-parallel o_proj + all-reduce kernel
(dllm_oproj_allreduce, tp.OprojAllReduce): with one rank it is the tcgen05
GEMM y = x W^T, checked against torch's bf16 matmul (fp32 accumulation) on
several shapes and over repeated calls; a rank whose peer never takes part
ends its call after the bounded wait with DLLM_DEV_WAIT_TIMEOUT (no fault,
the device stays usable); the 2-rank reduction over NVLink runs in
tests/test_gpu_tp.py."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(11902, 4096, 2048), (300, 1024, 512), (129, 3584, 4096), (1, 256, 64)])
def test_single_rank_gemm_matches_torch(M, N, K):
    from dllmserve_b200 import ops
    from dllmserve_b200.tp import OprojAllReduce

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    fused = OprojAllReduce(M, N, device=dev)
    for rep in range(3):
        x = torch.randn(M, K, device=dev, dtype=torch.bfloat16, generator=g)
        w = (torch.randn(N, K, device=dev, dtype=torch.bfloat16, generator=g) * 0.02).to(torch.bfloat16)
        y = fused(x, w)
        ref = F.linear(x, w)
        torch.cuda.synchronize()
        assert ops.read_device_status(dev) == 0
        err = (y.float() - ref.float()).abs()
        scale = ref.float().abs().mean().item()
        assert err.max().item() <= 2e-2 * max(1.0, ref.float().abs().max().item()), (rep, err.max().item())
        assert err.mean().item() <= 4e-3 * max(scale, 1e-3) + 1e-4, (rep, err.mean().item(), scale)


def test_missing_peer_times_out_with_status():
    """tp=2 on one GPU with a 'peer' whose buffers are local and which never
    runs: the owned tiles' partials from rank 1 never arrive, the bounded wait
    ends the call with DLLM_DEV_WAIT_TIMEOUT, and the device stays usable."""
    from dllmserve_b200 import _native, ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _native.lib()
    M, N, K = 256, 512, 128
    tiles = ((M + 127) // 128) * (N // 256)
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
    recv = [torch.zeros(2, M, N, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    ys = [torch.zeros(M, N, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    flags = [torch.zeros(3 * tiles, device=dev, dtype=torch.int32) for _ in range(2)]
    arr = ctypes.c_void_p * 2
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.dllm_oproj_allreduce(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), M, N, K,
                                  arr(*[r.data_ptr() for r in recv]), arr(*[y.data_ptr() for y in ys]),
                                  arr(*[f.data_ptr() for f in flags]), 0, 2, 1, status.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == _native.DLLM_DEV_WAIT_TIMEOUT
    # rank 0's partials of rank 1's tiles were delivered (and flagged) before the wait
    assert int((flags[1][:tiles] == 1).sum()) == tiles // 2
    # the device still works
    y = torch.ones(4, device=dev) * 2
    assert float(y.sum()) == 8.0
    ops.read_device_status(dev)


def test_epoch_wraps_with_flag_reset():
    """The epoch counter restarts at 1 after a collective flag reset (a flag
    left from an old call must never equal a new epoch); results stay right
    and the output buffers keep alternating across the wrap."""
    from dllmserve_b200.tp import OprojAllReduce

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    M, N, K = 200, 512, 256
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    w = (torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.05).to(torch.bfloat16)
    ref = torch.nn.functional.linear(x, w).float()
    fused = OprojAllReduce(M, N, device=dev)
    fused.epoch = 0x7FFFFFF0 - 1
    y0 = fused(x, w).clone()  # epoch 0x7FFFFFF0
    assert fused.epoch == 0x7FFFFFF0
    p0 = fused(x, w).data_ptr()  # reset, epoch 1
    assert fused.epoch == 1
    y1 = fused(x, w)  # epoch 2
    torch.cuda.synchronize()
    assert p0 != y1.data_ptr()
    for y in (y0, y1):
        assert (y.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
    fused.close()
