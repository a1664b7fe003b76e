"""CPU restatement of the fused o_proj + all-reduce protocol of
dllm_oproj_allreduce (csrc/oproj_ar.cu), run by 2 gloo ranks whose "peer
memory" is named shared memory. It replaces RowParallelLinear.forward's
F.linear + dist.all_reduce (dllmserve/layers/linear.py:186-190).

Per call (epoch e), every rank, as the kernel does:
  A) computes its partial tiles (128 x 256) of x_r W_r^T, rounds them to bf16,
     stores each into its owner's receive region (owner = tile mod tp, slot
     `rank`) and raises the owner's flag [rank][tile] = e;
  B) concurrently (a second thread, as the kernel's reduction warps) waits
     for the tp flags of each tile it owns, sums the partials in rank order
     in fp32, rounds once to bf16, writes the result into every rank's output
     buffer (parity e & 1) and raises the final flag [tile] = e on the others;
  C) waits for the final flags of the tiles it does not own.
Checked: three calls with fresh inputs give, on both ranks, the rank-order
fp32 sum of the bf16 partials, identical on both ranks; the epochs need no
flag reset; and a rank whose peer never writes gives up after a bounded
wait instead of hanging. This pins the tile ownership, flag and epoch rules
the CUDA kernel follows; the kernel itself is tested on GPUs
(tests/test_gpu_oproj.py, tests/test_gpu_tp.py)."""
import datetime
import os
import socket
import threading
import time

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

TM, TN = 128, 256


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


class _Peer:
    """One rank's buffer, as the kernel's single allocation: receive region
    [tp, M, N], two outputs [M, N] (fp32 holding bf16 values here) and the
    flags [(tp + 1) * tiles] int32."""

    def __init__(self, shm, tp, M, N, tiles):
        off = 0
        self.recv = np.ndarray((tp, M, N), np.float32, shm.buf, off)
        off += self.recv.nbytes
        self.y = np.ndarray((2, M, N), np.float32, shm.buf, off)
        off += self.y.nbytes
        self.flags = np.ndarray(((tp + 1) * tiles,), np.int32, shm.buf, off)

    @staticmethod
    def nbytes(tp, M, N, tiles):
        return 4 * (tp * M * N + 2 * M * N + (tp + 1) * tiles)


def _wait(flags, idx, epoch, err, wait_s):
    t0 = time.monotonic()
    while flags[idx] != epoch:
        if err[0] or time.monotonic() - t0 > wait_s:
            err[0] = True  # a timeout here is the kernel's DLLM_DEV_WAIT_TIMEOUT
            return False
        time.sleep(1e-4)
    return True


def _call(rank, tp, peers, x, w, epoch, wait_s):
    """One fused o_proj + all-reduce call; returns this rank's output view or None on timeout."""
    M, N = x.shape[0], w.shape[0]
    tiles_m, tiles_n = (M + TM - 1) // TM, N // TN
    num_tiles = tiles_m * tiles_n
    fin = tp * num_tiles
    par = epoch & 1
    err = [False]
    part = x @ w.T

    def phase_b():
        for t in range(rank, num_tiles, tp):
            if not all(_wait(peers[rank].flags, src * num_tiles + t, epoch, err, wait_s) for src in range(tp)):
                return
            tm, tn = divmod(t, tiles_n)
            rs, cs = slice(tm * TM, min(M, (tm + 1) * TM)), slice(tn * TN, (tn + 1) * TN)
            acc = np.zeros((rs.stop - rs.start, TN), np.float32)
            for src in range(tp):  # rank order, fp32
                acc += peers[rank].recv[src, rs, cs]
            out = _bf16(acc)
            for p in range(tp):
                peers[p].y[par, rs, cs] = out
            for p in range(tp):
                if p != rank:
                    peers[p].flags[fin + t] = epoch

    red = threading.Thread(target=phase_b)
    red.start()
    for t in range(num_tiles):  # phase A: every tile, pushed to its owner
        owner = t % tp
        tm, tn = divmod(t, tiles_n)
        rs, cs = slice(tm * TM, min(M, (tm + 1) * TM)), slice(tn * TN, (tn + 1) * TN)
        peers[owner].recv[rank, rs, cs] = _bf16(part[rs, cs])
        peers[owner].flags[rank * num_tiles + t] = epoch
    red.join()
    for t in range(num_tiles):  # phase C
        if t % tp != rank and not _wait(peers[rank].flags, fin + t, epoch, err, wait_s):
            break
    return None if err[0] else peers[rank].y[par].copy()


def _worker(rank, world, port, M, N, K, absent, wait_s, out_path):
    from multiprocessing import shared_memory

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    tiles = ((M + TM - 1) // TM) * (N // TN)
    shm = shared_memory.SharedMemory(create=True, size=_Peer.nbytes(world, M, N, tiles))
    np.ndarray((shm.size,), np.uint8, shm.buf)[:] = 0
    names = [None] * world
    dist.all_gather_object(names, shm.name)
    others = {p: shared_memory.SharedMemory(name=n) for p, n in enumerate(names) if p != rank}
    peers = [_Peer(shm if p == rank else others[p], world, M, N, tiles) for p in range(world)]
    dist.barrier()
    res = {"outs": [], "refs": [], "timeout": False}
    try:
        g = np.random.default_rng(100 + rank)
        for epoch in (1, 2, 3):
            x = _bf16(g.standard_normal((M, K)).astype(np.float32))
            w = _bf16(0.05 * g.standard_normal((N, K)).astype(np.float32))
            # the reference result: every rank's bf16 partial, summed in rank order in fp32
            parts = [None] * world
            dist.all_gather_object(parts, _bf16(x @ w.T))
            ref = np.zeros((M, N), np.float32)
            for p in parts:
                ref += p
            res["refs"].append(_bf16(ref))
            # every rank takes the same collective steps, whatever happens in between
            if (absent and rank == 1) or res["timeout"]:
                continue  # rank 1 never writes: its peer must time out
            y = _call(rank, world, peers, x, w, epoch, wait_s)
            if y is None:
                res["timeout"] = True
            else:
                res["outs"].append(y)
        dist.barrier()
    finally:
        torch.save(res, f"{out_path}.{rank}")
        for s in others.values():
            s.close()
        shm.close()
        shm.unlink()
        dist.destroy_process_group()


def test_protocol_two_ranks_three_calls(tmp_path):
    out = str(tmp_path / "proto")
    M, N, K = 300, 512, 96  # 3 x 2 tiles, a ragged last row block
    mp.start_processes(_worker, args=(2, _free_port(), M, N, K, False, 20.0, out), nprocs=2, start_method="spawn")
    r0, r1 = (torch.load(f"{out}.{r}", weights_only=False) for r in range(2))
    assert not r0["timeout"] and not r1["timeout"]
    assert len(r0["outs"]) == len(r1["outs"]) == 3
    for y0, y1, ref in zip(r0["outs"], r1["outs"], r0["refs"]):
        assert np.array_equal(y0, y1)  # every rank holds the same bits
        assert np.array_equal(y0, ref)  # rank-order fp32 sum of the bf16 partials, rounded once


def test_protocol_missing_peer_times_out(tmp_path):
    out = str(tmp_path / "proto_absent")
    M, N, K = 128, 256, 32
    mp.start_processes(_worker, args=(2, _free_port(), M, N, K, True, 1.0, out), nprocs=2, start_method="spawn")
    r0 = torch.load(f"{out}.0", weights_only=False)
    assert r0["timeout"]  # bounded wait ended, no hang
