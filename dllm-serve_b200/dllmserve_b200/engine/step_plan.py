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

from dataclasses import dataclass, field

import torch

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


def build_step_plan(ctx, device: torch.device, total_rows: int) -> StepPlan:
    """Turn the context of one diffusion step into device metadata.

    ``total_rows`` is q.shape[0]; the per-sequence row counts derived from the
    sparse states must add up to it (the model runner's layout)."""
    seqs = ctx.seqs
    if not seqs:
        raise ValueError("diffusion context without sequences")
    slot_mapping = ctx.slot_mapping
    infos = []
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
        if st != STATE_DENSE:
            n_expect = info.n_cached if st == STATE_REUSE else info.n_keep
            sm = slot_mapping[i] if slot_mapping is not None else None
            if sm is None or sm.numel() != n_expect:
                got = None if sm is None else sm.numel()
                raise ValueError(
                    f"slot_mapping[{i}] has {got} slots, sequence needs {n_expect}")
        infos.append(info)
        row += info.rows
    if row != total_rows:
        raise ValueError(f"sequences cover {row} rows but q has {total_rows}")

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
