"""Per-denoising-step metadata for the diffusion attention path.

The reference rebuilds its packed Q/K/V lists inside every layer with a host
loop over sequences (dllmserve/layers/attention.py:168-304), issuing device
syncs (``torch.arange`` from 0-d CUDA tensors) and ~5 copy passes over Q/K/V.
Here the same per-sequence decisions are made ONCE per step, on the host, from
the sequences' sparse states, and turned into a handful of small device arrays
that every layer reuses:

  * ``cu``      int32 [B+1]: rows of each sequence in q/k/v/o (the layout the
                 model runner produces, model_runner.py:240-304)
  * ``cu_c``    int32 [B+1]: cached K/V rows of each "reuse" sequence (state 2)
  * ``slots_c`` int32: their cache slots, concatenated (context.slot_mapping)
  * ``desc_*``  int32 [n, 8]: selection descriptors of "compute cache"
                 sequences (state 1), split by ``head_select``
  * ``slots_*`` int32: their destination slots, concatenated

Per-sequence rules (same as the reference):
  state 0 / no sparse state: Q = K = V = all the sequence's rows
  state 1: as state 0 for attention; additionally score the candidates (all
           tokens outside the current block) and store the top n_keep rows
           (attention.py:179-233)
  state 2: the model runner fed only the block's rows; K/V = the n_keep cached
           rows followed by the block's rows (attention.py:235-265)
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field

import torch

from .. import _native, ops

from ..sparse.state import num_keep

STATE_DENSE = 0
STATE_COMPUTE = 1
STATE_REUSE = 2


def seq_state(seq) -> int:
    ss = getattr(seq, "sparse_state", None)
    if ss is None or ss.is_full_attention:
        return STATE_DENSE
    if ss.should_compute_cache:
        return STATE_COMPUTE
    if ss.should_reuse_cache:
        return STATE_REUSE
    raise ValueError(f"unrecognized cache state {ss.cache_state!r}")


@dataclass
class SeqInfo:
    state: int
    rows: int            # rows of this sequence in q/k/v
    row_start: int
    n_cached: int = 0    # state 2: cached rows attended before the fresh ones
    blk_start: int = 0   # state 1: current block, relative to the sequence
    blk_len: int = 0
    n_keep: int = 0      # state 1: rows selected and stored
    pool_kernel: int = 1
    head_select: bool = False


@dataclass
class StepPlan:
    infos: list
    cu: torch.Tensor
    max_rows: int
    total_rows: int
    cu_c: torch.Tensor | None
    slots_c: torch.Tensor | None
    total_c: int
    sel: dict = field(default_factory=dict)   # head_select(bool) -> (desc, slots, max_klen, idx_total)
    scratch: dict = field(default_factory=dict)

    @property
    def q_lens(self):
        return [i.rows for i in self.infos]

    @property
    def k_lens(self):
        return [i.rows + i.n_cached for i in self.infos]


def _h2d(values, device, dtype=torch.int32) -> torch.Tensor:
    t = torch.tensor(values, dtype=dtype)
    if device.type == "cuda":
        t = t.pin_memory().to(device, non_blocking=True)
    return t


def _seq_infos(ctx, total_rows: int):
    """Per-sequence rows, block, cached / selected row counts (the reference's
    per-sequence rules, attention.py:168-304) and the validated slot lists."""
    seqs = ctx.seqs
    if not seqs:
        raise ValueError("diffusion context without sequences")
    slot_mapping = ctx.slot_mapping
    infos, slot_lists = [], []
    row = 0
    for i, seq in enumerate(seqs):
        st = seq_state(seq)
        L = int(seq.num_tokens)
        if st == STATE_REUSE:
            ss = seq.sparse_state
            start, blen = ss.compute_block_boundaries(seq.num_prompt_tokens, L)
            n_c = num_keep(ss.num_unused_tokens(seq.num_prompt_tokens, L)
                           if hasattr(ss, "num_unused_tokens")
                           else L - blen, ss.retention_ratio)
            info = SeqInfo(STATE_REUSE, blen, row, n_cached=n_c)
        elif st == STATE_COMPUTE:
            ss = seq.sparse_state
            start, blen = ss.compute_block_boundaries(seq.num_prompt_tokens, L)
            if blen <= 0:
                raise ValueError(f"sequence {i} has an empty diffusion block; nothing to score")
            klen = L - blen
            pool = ss.pool_kernel if ss.pool_kernel is not None else 1
            info = SeqInfo(STATE_COMPUTE, L, row, blk_start=start, blk_len=blen,
                           n_keep=num_keep(klen, ss.retention_ratio), pool_kernel=int(pool),
                           head_select=bool(ss.config.head_select))
        else:
            info = SeqInfo(STATE_DENSE, L, row)
        sm = None
        if st != STATE_DENSE:
            n_expect = info.n_cached if st == STATE_REUSE else info.n_keep
            sm = slot_mapping[i] if slot_mapping is not None else None
            if sm is None or not isinstance(sm, torch.Tensor) or sm.numel() != n_expect:
                got = None if not isinstance(sm, torch.Tensor) else sm.numel()
                raise ValueError(
                    f"slot_mapping[{i}] has {got} slots, sequence needs {n_expect}")
        infos.append(info)
        slot_lists.append(sm)
        row += info.rows
    if row != total_rows:
        raise ValueError(f"sequences cover {row} rows but q has {total_rows}")
    return infos, slot_lists


class _Staging:
    """A ring of pinned host buffers for the per-sequence rows of the device
    plan builder; a buffer is reused only after the copy that read it ran."""

    def __init__(self, n=4):
        self.bufs = [None] * n
        self.events = [None] * n
        self.next = 0

    def take(self, rows: int, device):
        i = self.next
        self.next = (i + 1) % len(self.bufs)
        ev = self.events[i]
        if ev is not None:
            ev.synchronize()
        if self.bufs[i] is None:
            self.bufs[i] = torch.empty((_native.PLAN_MAX_BATCH, _native.PLAN_SEQ_FIELDS),
                                       dtype=torch.int64, pin_memory=True)
        return i, self.bufs[i]

    def done(self, i):
        ev = self.events[i]
        if ev is None:  # one event per buffer, re-recorded at each use
            ev = self.events[i] = torch.cuda.Event()
        ev.record()


_STAGING: dict = {}


def _device_plan(ctx, device, total_rows, num_kv_heads, infos, slot_lists) -> "StepPlan":
    """Materialise the plan with one dllm_build_step_plan launch: the device
    re-derives every per-sequence quantity from the sequences' raw state and
    writes cu, cu_c, the selection descriptors and the concatenated slot
    lists into one int32 buffer whose sections become the plan's tensors."""
    B = len(infos)
    n_hs = sum(1 for f in infos if f.state == STATE_COMPUTE and f.head_select)
    n_sh = sum(1 for f in infos if f.state == STATE_COMPUTE and not f.head_select)
    total_c = sum(f.n_cached for f in infos if f.state == STATE_REUSE)
    slots_hs = sum(f.n_keep for f in infos if f.state == STATE_COMPUTE and f.head_select)
    slots_sh = sum(f.n_keep for f in infos if f.state == STATE_COMPUTE and not f.head_select)
    D8 = _native.SEQ_DESC_INTS
    off_cu_c = B + 1
    off_dhs = off_cu_c + B + 1
    off_dsh = off_dhs + n_hs * D8
    off_sc = off_dsh + n_sh * D8
    off_shs = off_sc + total_c
    off_ssh = off_shs + slots_hs
    total = off_ssh + slots_sh
    layout = (ctypes.c_int64 * _native.PLAN_LAYOUT_INTS)(
        total, off_cu_c, off_dhs, n_hs, off_dsh, n_sh, off_sc, total_c, off_shs, slots_hs, off_ssh, slots_sh)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    staging = _STAGING.get(idx)
    if staging is None:
        staging = _STAGING[idx] = _Staging()
    keep = []
    si, buf = staging.take(B, device)
    rows = []
    for f, seq, sm in zip(infos, ctx.seqs, slot_lists):
        ss = getattr(seq, "sparse_state", None)
        if f.state == STATE_DENSE:
            rows.append([0, int(seq.num_tokens), int(seq.num_prompt_tokens), 0, 0, 0, 0, 0, 0, 0])
            continue
        if sm.dtype != torch.int32 or not sm.is_contiguous() or sm.device != device:
            sm = sm.to(device=device, dtype=torch.int32).contiguous()
            keep.append(sm)
        pool = ss.pool_kernel if ss.pool_kernel is not None else 1
        ratio_bits = struct.unpack("<q", struct.pack("<d", float(ss.retention_ratio)))[0]
        rows.append([f.state, int(seq.num_tokens), int(seq.num_prompt_tokens), int(ss.current_block_idx),
                     int(ss.block_len), ratio_bits, int(pool) | (int(bool(ss.config.head_select)) << 32),
                     sm.data_ptr(), sm.numel(), 0])
    buf[:B] = torch.tensor(rows, dtype=torch.int64)
    with ops._on_device(device):
        dev_rows = torch.empty((B, _native.PLAN_SEQ_FIELDS), dtype=torch.int64, device=device)
        dev_rows.copy_(buf[:B], non_blocking=True)
        staging.done(si)
        out = torch.empty(total, dtype=torch.int32, device=device)
        rc = _native.lib().dllm_build_step_plan(dev_rows.data_ptr(), B, int(num_kv_heads), out.data_ptr(),
                                                layout, ops._status_ptr(device), ops._stream_ptr())
    _native.check(rc, "build_step_plan")
    ops.LAUNCHES[0] += 1
    keep += [dev_rows, out] + [sm for sm in slot_lists if sm is not None]
    plan = StepPlan(infos=infos, cu=out[:B + 1], max_rows=max(f.rows for f in infos), total_rows=total_rows,
                    cu_c=out[off_cu_c:off_cu_c + B + 1] if total_c else None,
                    slots_c=out[off_sc:off_sc + total_c] if total_c else None, total_c=total_c)
    for hs, n, off_d, off_s, n_slots in ((True, n_hs, off_dhs, off_shs, slots_hs),
                                         (False, n_sh, off_dsh, off_ssh, slots_sh)):
        if not n:
            continue
        sel_idx = [i for i, f in enumerate(infos) if f.state == STATE_COMPUTE and f.head_select == hs]
        max_klen = max(infos[i].rows - infos[i].blk_len for i in sel_idx)
        mult = num_kv_heads if hs else 1
        plan.sel[hs] = (sel_idx, None, out[off_s:off_s + n_slots], max_klen)
        plan.scratch[("sel", hs, num_kv_heads)] = (out[off_d:off_d + n * D8].view(n, D8),
                                                    out[off_s:off_s + n_slots], max_klen, n_slots * mult)
    plan.scratch["keepalive"] = keep
    return plan


def build_step_plan(ctx, device: torch.device, total_rows: int, num_kv_heads: int | None = None) -> StepPlan:
    """Turn the context of one diffusion step into device metadata.

    ``total_rows`` is q.shape[0]; the per-sequence row counts derived from the
    sparse states must add up to it (the model runner's layout). On a CUDA
    device with ``num_kv_heads`` given, the arrays are built by one device
    launch (dllm_build_step_plan); otherwise (CPU, used by host-logic tests)
    they are assembled here."""
    infos, slot_lists = _seq_infos(ctx, total_rows)
    if (device.type == "cuda" and num_kv_heads is not None and len(infos) <= _native.PLAN_MAX_BATCH):
        return _device_plan(ctx, device, total_rows, num_kv_heads, infos, slot_lists)
    slot_mapping = ctx.slot_mapping

    cu_host = [0]
    for inf in infos:
        cu_host.append(cu_host[-1] + inf.rows)
    cu = _h2d(cu_host, device)

    reuse = [i for i, inf in enumerate(infos) if inf.state == STATE_REUSE]
    cu_c = slots_c = None
    total_c = 0
    if reuse:
        cc = [0]
        for inf in infos:
            cc.append(cc[-1] + inf.n_cached)
        total_c = cc[-1]
        cu_c = _h2d(cc, device)
        parts = [slot_mapping[i].to(device=device, dtype=torch.int32).reshape(-1) for i in reuse]
        slots_c = torch.cat(parts) if parts else None

    sel = {}
    for hs in (True, False):
        idx = [i for i, inf in enumerate(infos) if inf.state == STATE_COMPUTE and inf.head_select == hs]
        if not idx:
            continue
        desc, parts = [], []
        slot_off = 0
        max_klen = 0
        for i in idx:
            inf = infos[i]
            klen = inf.rows - inf.blk_len
            max_klen = max(max_klen, klen)
            # [6] (top_idx offset) depends on num_kv_heads; selection_arrays fills it
            desc.append([inf.row_start, inf.rows, inf.blk_start, inf.blk_len, inf.n_keep,
                         slot_off, 0, inf.pool_kernel])
            parts.append(slot_mapping[i].to(device=device, dtype=torch.int32).reshape(-1))
            slot_off += inf.n_keep
        sel[hs] = (idx, desc, parts, max_klen)

    plan = StepPlan(infos=infos, cu=cu, max_rows=max(inf.rows for inf in infos),
                    total_rows=total_rows, cu_c=cu_c, slots_c=slots_c, total_c=total_c)
    for hs, (idx, desc, parts, max_klen) in sel.items():
        plan.sel[hs] = (idx, desc, torch.cat(parts) if parts else None, max_klen)
    return plan


def selection_arrays(plan: StepPlan, head_select: bool, num_kv_heads: int, device):
    """Device descriptor array for one selection launch, with index offsets
    for a top_idx buffer laid out per sequence as [Hkv, n_keep] (head_select)
    or [n_keep]. Returns (desc, slots, max_klen, idx_total) or None."""
    entry = plan.sel.get(head_select)
    if entry is None:
        return None
    key = ("sel", head_select, num_kv_heads)
    cached = plan.scratch.get(key)
    if cached is not None:
        return cached
    idx, desc, slots, max_klen = entry
    if desc is None:
        raise ValueError("this step plan was built on the device for another num_kv_heads; "
                         "build one per num_kv_heads")
    rows = []
    idx_off = 0
    for d in desc:
        d = list(d)
        d[6] = idx_off
        idx_off += d[4] * (num_kv_heads if head_select else 1)
        rows.append(d)
    out = (_h2d(rows, device), slots, max_klen, idx_off)
    plan.scratch[key] = out
    return out
