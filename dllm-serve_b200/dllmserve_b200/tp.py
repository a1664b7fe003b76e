"""Tensor-parallel head sharding around the attention path.

Rank r of a tp-way group owns query heads [r*Hq/tp, (r+1)*Hq/tp) and KV heads
[r*Hkv/tp, (r+1)*Hkv/tp) - the contiguous slices ColumnParallelLinear gives
the q/k/v projections (dllmserve/layers/linear.py:55-88) and the per-rank
cache [.., Hkv/tp, D] (model_runner.py:174). Attention needs no exchange; the
one collective is the all-reduce of the row-parallel o_proj output
(linear.py:186-190).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _native


def head_slice(num_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[int, int, int, int]:
    """(q_head_begin, q_head_end, kv_head_begin, kv_head_end) of ``rank``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if num_heads % world or num_kv_heads % world:
        raise ValueError(
            f"{num_heads} query / {num_kv_heads} KV heads do not split over {world} ranks")
    hq, hk = num_heads // world, num_kv_heads // world
    return rank * hq, (rank + 1) * hq, rank * hk, (rank + 1) * hk


def row_parallel_oproj(x: torch.Tensor, weight_shard: torch.Tensor, bias: torch.Tensor | None = None,
                       rank: int = 0, group=None, chunks: int = 1) -> torch.Tensor:
    """y = x @ W_shard^T (+ bias on rank 0), summed over ranks (linear.py:186-190).

    ``chunks`` > 1 splits the rows: each chunk's GEMM is followed by an
    asynchronous all-reduce of that chunk, which runs on NCCL's stream while
    the next chunk's GEMM runs on the current one. The all-reduce is
    elementwise, so chunking changes nothing it sums; a chunk's GEMM may
    round differently from the whole one (the library picks its algorithm
    per shape)."""
    distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
    b = bias if rank == 0 else None
    if not distributed or chunks <= 1 or x.shape[0] < chunks:
        y = F.linear(x, weight_shard, b)
        if distributed:
            dist.all_reduce(y, group=group)
        return y
    y = torch.empty(x.shape[0], weight_shard.shape[0], dtype=x.dtype, device=x.device)
    bounds = [x.shape[0] * i // chunks for i in range(chunks + 1)]
    works = []
    for i in range(chunks):
        r0, r1 = bounds[i], bounds[i + 1]
        if b is not None:
            torch.addmm(b, x[r0:r1], weight_shard.t(), out=y[r0:r1])
        else:
            torch.matmul(x[r0:r1], weight_shard.t(), out=y[r0:r1])
        works.append(dist.all_reduce(y[r0:r1], group=group, async_op=True))
    for w in works:
        w.wait()
    return y


class OprojAllReduce:
    """Row-parallel o_proj fused with its all-reduce in one kernel per rank
    (dllm_oproj_allreduce; replaces ``F.linear`` + ``dist.all_reduce`` of
    RowParallelLinear.forward, linear.py:186-190): the GEMM's finished tiles
    go straight over NVLink into the owning rank's receive buffer, the owner
    sums them and pushes the result to every rank.

    Holds, per rank, one zeroed device buffer with the receive region
    [tp, max_rows, hidden], two output buffers [max_rows, hidden] (calls
    alternate between them) and the tile flags; the ranks' buffers are mapped
    into each other with CUDA IPC once, at construction (a collective over
    ``group``). Every rank must call it in the same order. The returned tensor
    is a view of an output buffer: it stays valid until the call after next."""

    def __init__(self, max_rows: int, hidden: int, group=None, device=None):
        if hidden % 256:
            raise ValueError("hidden must be a multiple of 256")
        self.distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
        self._group = group
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.rank = dist.get_rank(group) if self.distributed else 0
        if self.world > _native.OPROJ_MAX_RANKS:
            raise ValueError(f"at most {_native.OPROJ_MAX_RANKS} ranks")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_rows, self.hidden = max_rows, hidden
        tiles = ((max_rows + 127) // 128) * (hidden // 256)

        def up(n):
            return (n + 255) // 256 * 256

        y_bytes = up(max_rows * hidden * 2)
        self._off_recv = 0
        self._off_y = (up(self.world * max_rows * hidden * 2), up(self.world * max_rows * hidden * 2) + y_bytes)
        self._off_flags = self._off_y[1] + y_bytes
        total = self._off_flags + up((self.world + 1) * tiles * 4)
        self.buf = torch.zeros(total, dtype=torch.uint8, device=self.device)
        lib = _native.lib()
        bases = [0] * self.world
        self._opened = []
        if self.distributed:
            handle = ctypes.create_string_buffer(_native.IPC_HANDLE_BYTES)
            off = ctypes.c_int64()
            with torch.cuda.device(self.device):
                _native.check(lib.dllm_ipc_export(self.buf.data_ptr(), handle, ctypes.byref(off)), "ipc_export")
            mine = (bytes(handle.raw), int(off.value))
            allh = [None] * self.world
            dist.all_gather_object(allh, mine, group=group)
            for p, (h, o) in enumerate(allh):
                if p == self.rank:
                    bases[p] = self.buf.data_ptr()
                    continue
                ptr = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    _native.check(lib.dllm_ipc_open(ctypes.create_string_buffer(h, _native.IPC_HANDLE_BYTES),
                                                    ctypes.byref(ptr)), "ipc_open")
                self._opened.append(ptr.value)
                bases[p] = ptr.value + o
        else:
            bases[0] = self.buf.data_ptr()
        arr = ctypes.c_void_p * self.world
        self._recv = arr(*[b + self._off_recv for b in bases])
        self._y = [arr(*[b + self._off_y[i] for b in bases]) for i in range(2)]
        self._flags = arr(*[b + self._off_flags for b in bases])
        self.epoch = 0

    def __call__(self, x: torch.Tensor, w_shard: torch.Tensor) -> torch.Tensor:
        """y = sum over ranks of x_r @ w_r^T for this rank's x [M, K] and
        W_o column slice w_shard [hidden, K] (bf16); returns [M, hidden]."""
        from . import ops

        M, K = x.shape
        if M > self.max_rows or w_shard.shape != (self.hidden, K):
            raise ValueError(f"x [{M}, {K}] / w {tuple(w_shard.shape)} do not fit [<= {self.max_rows}, K] / "
                             f"[{self.hidden}, K]")
        if x.dtype != torch.bfloat16 or w_shard.dtype != torch.bfloat16 or x.stride(1) != 1 or w_shard.stride(1) != 1:
            raise ValueError("x and w_shard must be bfloat16 with contiguous rows")
        if x.device != self.device or w_shard.device != self.device:
            raise ValueError(f"x and w_shard must be on {self.device}")
        if self.epoch >= 0x7FFFFFF0:
            self._reset_flags()
        self.epoch += 1
        parity = self.epoch & 1
        lib = _native.lib()
        with torch.cuda.device(self.device):
            rc = lib.dllm_oproj_allreduce(x.data_ptr(), x.stride(0), w_shard.data_ptr(), w_shard.stride(0), M,
                                          self.hidden, K, self._recv, self._y[parity], self._flags, self.rank,
                                          self.world, self.epoch, ops._status_ptr(self.device), ops._stream_ptr())
        _native.check(rc, "oproj_allreduce")
        ops.LAUNCHES[0] += 1
        start = self._off_y[parity]
        return self.buf[start:start + M * self.hidden * 2].view(torch.bfloat16).view(M, self.hidden)

    def _reset_flags(self) -> None:
        """Before the epoch counter wraps: every rank zeroes its own flags once
        all ranks' kernels have finished (a flag left from an old call would
        otherwise equal a new epoch), then the ranks meet again before any
        writes the new epoch's flags. A collective over the group."""
        torch.cuda.synchronize(self.device)
        if self.distributed:
            dist.barrier(group=self._group)
        self.buf[self._off_flags:].zero_()
        torch.cuda.synchronize(self.device)
        if self.distributed:
            dist.barrier(group=self._group)
        self.epoch = 0

    def close(self) -> None:
        """Unmaps the peers' buffers (collective use must have ended)."""
        lib = _native.lib()
        while self._opened:
            _native.check(lib.dllm_ipc_close(self._opened.pop()), "ipc_close")
