"""Tensor-parallel head sharding on 2 GPUs (skipped with fewer): one NCCL
process per GPU, each running the attention kernel on its contiguous head
slice (tp.head_slice, as ColumnParallelLinear shards q/k/v,
dllmserve/layers/linear.py:55-88, with the per-rank cache slice of
model_runner.py:174). Checked per rank: its launch equals the single-launch
result on those heads bit for bit and the fp32 oracle within tolerance; the
all-reduced row-parallel o_proj (linear.py:186-190) equals the single-GPU
o_proj within bf16 tolerance, both through NCCL after the GEMM and through
the fused kernel that pushes GEMM tiles over NVLink (dllm_oproj_allreduce),
whose result is also identical on both ranks, call after call."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

D = 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(hq, hkv, lens, hidden):
    g = torch.Generator().manual_seed(11)
    N = sum(lens)
    q = torch.randn(N, hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(N, hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(N, hkv, D, generator=g).to(torch.bfloat16)
    w = (torch.randn(hidden, hq * D, generator=g) * 0.02).to(torch.bfloat16)
    return q, k, v, w


def _worker(rank, world, port, hq, hkv, lens, hidden, out_path):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    res = {"rank": rank}
    try:
        from dllmserve_b200 import ops
        from dllmserve_b200.tp import head_slice, row_parallel_oproj
        from oracle import attention_ref as R

        q, k, v, w = _inputs(hq, hkv, lens, hidden)
        h0, h1, k0, k1 = head_slice(hq, hkv, rank, world)
        cu = [0]
        for L in lens:
            cu.append(cu[-1] + L)
        cud = torch.tensor(cu, dtype=torch.int32, device=dev)
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        full = ops.varlen_attention(qd, kd, vd, cud, cud, max(lens))
        part = ops.varlen_attention(qd[:, h0:h1].contiguous(), kd[:, k0:k1].contiguous(),
                                    vd[:, k0:k1].contiguous(), cud, cud, max(lens))
        torch.cuda.synchronize()
        res["slice_equal"] = bool(torch.equal(part, full[:, h0:h1]))
        ref = R.varlen_attention(q[:, h0:h0 + 1].float(), k[:, k0:k0 + 1].float(), v[:, k0:k0 + 1].float(),
                                 cu, cu, D ** -0.5)
        err = (part[:, :1].float().cpu() - ref).abs()
        res["oracle_err"] = (float(err.max()), float(err.mean()))
        wd = w.to(dev)
        y = row_parallel_oproj(part.reshape(part.shape[0], -1), wd[:, h0 * D:h1 * D].contiguous(), rank=rank)
        y_ref = torch.nn.functional.linear(full.reshape(full.shape[0], -1), wd)
        torch.cuda.synchronize()
        e = (y.float() - y_ref.float()).abs()
        res["oproj_err"] = (float(e.max()), float(e.mean()), float(y_ref.float().abs().mean()))
        from dllmserve_b200.tp import OprojAllReduce

        fused = OprojAllReduce(part.shape[0], hidden, device=dev)
        ys = []
        for _ in range(3):
            yf = fused(part.reshape(part.shape[0], -1), wd[:, h0 * D:h1 * D].contiguous())
            torch.cuda.synchronize()
            ys.append(yf.clone())
        fused.close()
        e = (ys[-1].float() - y_ref.float()).abs()
        res["fused_err"] = (float(e.max()), float(e.mean()))
        res["fused_repeat_equal"] = all(torch.equal(ys[0], yy) for yy in ys[1:])
        res["fused_y"] = ys[-1].cpu()
        res["status"] = ops.read_device_status(dev)
    finally:
        torch.save(res, f"{out_path}.{rank}")
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("hq,hkv,lens", [(32, 32, [419, 1087, 130, 700]), (28, 4, [300, 800, 64])])
def test_head_sharded_tp_on_two_gpus(tmp_path, hq, hkv, lens):
    world = 2
    out = str(tmp_path / "tp")
    mp.start_processes(_worker, args=(world, _free_port(), hq, hkv, lens, 1024, out), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        res = torch.load(f"{out}.{r}")
        assert res["slice_equal"], r
        assert res["oracle_err"][0] <= 2e-2 and res["oracle_err"][1] <= 2e-3, res["oracle_err"]
        mx, mean, scale = res["oproj_err"]
        assert mx <= 2e-2 and mean <= 2e-3 * max(1.0, scale), res["oproj_err"]
        assert res["fused_err"][0] <= 2e-2 and res["fused_err"][1] <= 2e-3 * max(1.0, scale), res["fused_err"]
        assert res["fused_repeat_equal"]
        assert res["status"] == 0
    y0, y1 = (torch.load(f"{out}.{r}")["fused_y"] for r in range(world))
    assert torch.equal(y0, y1)
