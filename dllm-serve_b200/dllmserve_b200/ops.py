"""Torch-facing wrappers of the native attention-path ops.

Every op validates shapes/dtypes on the host (no device reads), then calls
the C ABI on the tensors' device with ``torch.cuda.current_stream()``.
The tensors must live on a CUDA device; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _native

_STATUS: dict[int, torch.Tensor] = {}

# Number of native kernel launches issued through this module (benchmarks
# report the count inside their timed region).
LAUNCHES = [0]


def device_status_word(device: torch.device) -> torch.Tensor:
    """The int32 device word the kernels report DLLM_DEV_* codes into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def _status_ptr(device: torch.device) -> int:
    """Pointer of the status word, or 0 (no device status) when none exists yet
    and the current stream is being captured (memory allocated during a
    capture belongs to that graph and must not be cached)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STATUS and torch.cuda.is_current_stream_capturing():
        return 0
    return device_status_word(device).data_ptr()


def read_device_status(device: torch.device, reset: bool = True) -> int:
    """Synchronising read of the device status word (tests / debug only)."""
    t = device_status_word(device)
    v = int(t.item())
    if reset and v:
        t.zero_()
    return v


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError("dllmserve_b200 ops need CUDA tensors (there is no CPU path)")
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_raw_device = getattr(torch._C, "_cuda_getDevice", None)


def _current_device() -> int:
    """torch.cuda.current_device() without its lazy-initialisation checks
    (about a microsecond per call); only called once the inputs are CUDA
    tensors, i.e. after CUDA was initialised."""
    if _raw_device is not None:
        return _raw_device()
    return torch.cuda.current_device()


def _stream_ptr() -> int:
    """cudaStream_t of the current stream on the current device (the raw query
    is several microseconds cheaper per call than building a Stream object)."""
    if _raw_stream is not None:
        return _raw_stream(_current_device())
    return torch.cuda.current_stream().cuda_stream


class _Current:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


_CURRENT = _Current()


def _on_device(dev: torch.device):
    """torch.cuda.device(dev), or a no-op context when dev is already current."""
    if dev.index is None or dev.index == _current_device():
        return _CURRENT
    return torch.cuda.device(dev)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# KV cache (attention.py:33-50, 77-92)
# ---------------------------------------------------------------------------
def store_kvcache(key, value, k_cache, v_cache, slot_mapping):
    """cache[slot_mapping[i]] <- key[i], value[i]. Same argument order and
    assertions as the reference's ``store_kvcache`` (attention.py:33-50)."""
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    _kv_copy(True, key, value, k_cache, v_cache, slot_mapping, D)


def load_kvcache(key, value, k_cache, v_cache, slot_mapping):
    """key[i], value[i] <- cache[slot_mapping[i]] (attention.py:77-92)."""
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    _kv_copy(False, key, value, k_cache, v_cache, slot_mapping, D)


def _kv_copy(store, key, value, k_cache, v_cache, slot_mapping, D):
    N = key.shape[0]
    if N == 0:
        return
    dev = _require_cuda(key, value, k_cache, v_cache, slot_mapping)
    if key.dtype != k_cache.dtype or value.dtype != v_cache.dtype or key.dtype != value.dtype:
        raise ValueError("key/value and cache dtypes must match")
    if slot_mapping.dtype != torch.int32:
        raise ValueError("slot_mapping must be int32")
    if not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be contiguous")
    # a cache slot is D contiguous elements, slots D apart (asserted above)
    num_slots = k_cache.numel() // D
    if v_cache.numel() // D != num_slots:
        raise ValueError("k_cache and v_cache hold different numbers of slots")
    lib = _native.lib()
    fn = lib.dllm_store_kvcache if store else lib.dllm_load_kvcache
    with _on_device(dev):
        rc = fn(
            key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
            k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(),
            N, D, key.element_size(), num_slots,
            _status_ptr(dev), _stream_ptr(),
        )
    _native.check(rc, "store_kvcache" if store else "load_kvcache")
    LAUNCHES[0] += 1


# ---------------------------------------------------------------------------
# Attention (attention.py:289-299, 235-265)
# ---------------------------------------------------------------------------
def _check_rows(name, t, heads, head_dim):
    if t.dim() != 3 or t.shape[1] != heads or t.shape[2] != head_dim:
        raise ValueError(f"{name} must be [tokens, {heads}, {head_dim}], got {tuple(t.shape)}")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16")
    if t.stride(2) != 1 or t.stride(1) != head_dim:
        raise ValueError(f"{name} must have contiguous heads (strides [*, {head_dim}, 1])")


_SCHED_WS: dict = {}


def sched_workspace(dev: torch.device, stream: int) -> int:
    """Device pointer of the attention scheduler workspace of (``dev``,
    ``stream``): zeroed int32 words that every launch leaves zero. Launches on
    one stream are ordered, so they can share one; launches on different
    streams may overlap and get their own. Returns 0 (round-robin order, same
    results) when the stream has none yet and is being captured: memory
    allocated during a capture belongs to that graph and must not be cached."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _SCHED_WS.get((idx, stream))
    if ws is None:
        if torch.cuda.is_current_stream_capturing():
            return 0
        ws = torch.zeros(_native.SCHED_WORKSPACE_INTS, dtype=torch.int32, device=torch.device("cuda", idx))
        _SCHED_WS[(idx, stream)] = ws
    return ws.data_ptr()


def varlen_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    max_seqlen_q: int,
    softmax_scale: float | None = None,
    *,
    k_cached: torch.Tensor | None = None,
    v_cached: torch.Tensor | None = None,
    cu_seqlens_c: torch.Tensor | None = None,
    k_cache: torch.Tensor | None = None,
    v_cache: torch.Tensor | None = None,
    slots: torch.Tensor | None = None,
    cu_seqlens_slots: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    heads: torch.Tensor | None = None,
) -> torch.Tensor:
    """Non-causal varlen attention (bf16). With ``k_cached``/``v_cached``/
    ``cu_seqlens_c`` each sequence attends to [cached rows ; fresh rows]; with
    ``k_cache``/``v_cache``/``slots``/``cu_seqlens_slots`` the cached rows are
    read straight from the paged cache (slots[cu[b]:cu[b+1]] for sequence b).

    ``rope=(positions, cos_sin_cache)``: ``q`` and the fresh ``k`` are not yet
    rotated; the result equals ``rope_neox(positions, q, k, cos_sin_cache)``
    followed by this attention, bit for bit. Launches whose query segments fit
    one 128-row tile rotate on chip (``dllm_attn_varlen_rope_fwd``: q and k are
    left untouched); longer ones rotate into new tensors first.

    ``heads`` (int32 device tensor of query-head indices): only those heads are
    computed (``dllm_attn_varlen_heads_fwd``); the output rows of the other
    heads are left as they are (pass ``out`` to keep them meaningful)."""
    if rope is not None:
        positions, cos_sin = rope
        if k_cached is not None:
            raise ValueError("rope is supported with the paged cache (k_cache/slots), not k_cached")
        if int(max_seqlen_q) > 128:
            qr, kr = rope_neox(positions, q, k, cos_sin)
            return varlen_attention(qr, kr, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale,
                                    k_cache=k_cache, v_cache=v_cache, slots=slots,
                                    cu_seqlens_slots=cu_seqlens_slots, out=out)
        return _varlen_attention_rope(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale,
                                      positions, cos_sin, k_cache, v_cache, slots, cu_seqlens_slots, out)
    Hq, D = q.shape[1], q.shape[2]
    Hkv = k.shape[1]
    _check_rows("q", q, Hq, D)
    _check_rows("k", k, Hkv, D)
    _check_rows("v", v, Hkv, D)
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    dev = _require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k)
    for name, c in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        if c.dtype != torch.int32 or not c.is_contiguous():
            raise ValueError(f"{name} must be contiguous int32")
    B = cu_seqlens_q.numel() - 1
    if cu_seqlens_k.numel() != B + 1:
        raise ValueError("cu_seqlens_q and cu_seqlens_k sizes differ")
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    else:
        _check_rows("out", out, Hq, D)
        if out.shape[0] != q.shape[0]:
            raise ValueError("out must have as many rows as q")
    lib = _native.lib()
    status = _status_ptr(dev)
    if heads is not None:
        if heads.dtype != torch.int32 or heads.dim() != 1 or not heads.is_contiguous() or heads.device != dev:
            raise ValueError("heads must be a contiguous 1-D int32 tensor on the inputs' device")
        if k_cached is not None or rope is not None:
            raise ValueError("heads works with the fresh rows or the paged cache (k_cache/slots) only")
        if k_cache is not None:
            row = _check_paged(q, k_cache, v_cache, slots, cu_seqlens_slots, B, Hkv, D)
            cache_args = (k_cache.data_ptr(), v_cache.data_ptr(), row, k_cache.numel() // row,
                          slots.data_ptr(), cu_seqlens_slots.data_ptr())
        else:
            cache_args = (None, None, 0, 0, None, None)
        with _on_device(dev):
            stream = _stream_ptr()
            rc = lib.dllm_attn_varlen_heads_fwd(
                q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), *cache_args,
                out.data_ptr(), out.stride(0), cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), B,
                int(max_seqlen_q), q.shape[0], k.shape[0], Hq, Hkv, D, float(softmax_scale),
                heads.data_ptr(), heads.numel(), sched_workspace(dev, stream), status, stream)
        _native.check(rc, "varlen_attention(heads)")
        if B > 0 and q.shape[0] > 0 and heads.numel() > 0:
            LAUNCHES[0] += 1
        return out
    with _on_device(dev):
        stream = _stream_ptr()
        sched = sched_workspace(dev, stream)
        if k_cache is not None:
            row = _check_paged(q, k_cache, v_cache, slots, cu_seqlens_slots, B, Hkv, D)
            rc = lib.dllm_attn_varlen_paged_fwd(
                q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                k_cache.data_ptr(), v_cache.data_ptr(), row, k_cache.numel() // row,
                slots.data_ptr(), cu_seqlens_slots.data_ptr(), out.data_ptr(), out.stride(0),
                cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), B, int(max_seqlen_q), q.shape[0],
                k.shape[0], Hq, Hkv, D, float(softmax_scale), sched, status, stream,
            )
        elif k_cached is None:
            rc = lib.dllm_attn_varlen_fwd(
                q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                out.data_ptr(), out.stride(0), cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(),
                B, int(max_seqlen_q), q.shape[0], k.shape[0], Hq, Hkv, D, float(softmax_scale),
                sched, status, stream,
            )
        else:
            _check_rows("k_cached", k_cached, Hkv, D)
            _check_rows("v_cached", v_cached, Hkv, D)
            _require_cuda(q, k_cached, v_cached, cu_seqlens_c)
            if cu_seqlens_c.dtype != torch.int32 or cu_seqlens_c.numel() != B + 1:
                raise ValueError("cu_seqlens_c must be int32 [batch+1]")
            if v_cached.shape[0] != k_cached.shape[0]:
                raise ValueError("k_cached and v_cached rows differ")
            rc = lib.dllm_attn_varlen_cached_fwd(
                q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                k_cached.data_ptr(), k_cached.stride(0), v_cached.data_ptr(), v_cached.stride(0),
                out.data_ptr(), out.stride(0), cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(),
                cu_seqlens_c.data_ptr(), B, int(max_seqlen_q), q.shape[0], k.shape[0],
                k_cached.shape[0], Hq, Hkv, D, float(softmax_scale), sched, status, stream,
            )
    _native.check(rc, "varlen_attention")
    if B > 0 and q.shape[0] > 0:
        LAUNCHES[0] += 1
    return out


class AttentionLaunch:
    """A varlen attention launch whose step-level arguments (sequence offsets,
    maximum query length, head counts, scale and, for reuse steps, the slot
    list) were validated once; each call checks only what can differ per call
    (q/k/v/out layout and row counts) and passes a prepared argument tuple to
    the C ABI, whose own checks (alignment, strides, sizes) still run on every
    call. One object serves every layer of a step that shares these arguments
    (layers differ only in their q/k/v and, for reuse steps, their paged
    cache, given per call as ``paged_cache_args``). Built by
    ``prepare_attention``."""

    __slots__ = ("_fn", "_slots", "_tail", "_dev", "_dev_index", "_heads", "_rows", "_status", "_ws")

    def __init__(self, fn, slots, tail, dev, heads, rows):
        self._fn = fn
        self._slots = slots          # (slots ptr, cu_seqlens_slots ptr) of a paged launch, else None
        self._tail = tail
        self._dev = dev
        self._dev_index = dev.index if dev.index is not None else torch.cuda.current_device()
        self._heads = heads          # (Hq, Hkv, D)
        self._rows = rows            # rows of q (and of the fresh k/v)
        self._status = _status_ptr(dev)
        self._ws: dict = {}

    def _check(self, name, t, h) -> int:
        """Raises unless t is a bf16 [rows, h*D] / [rows, h, D] tensor with
        contiguous heads on the launch's device; returns its token stride."""
        D = self._heads[2]
        sh, st = t.shape, t.stride()
        if (t.dtype is not torch.bfloat16 or t.get_device() != self._dev_index or sh[0] != self._rows
                or not ((len(sh) == 2 and sh[1] == h * D and st[1] == 1)
                        or (len(sh) == 3 and sh[1] == h and sh[2] == D and st[2] == 1 and st[1] == D))):
            raise ValueError(f"{name}: expected bfloat16 [{self._rows}, {h}*{D}] or [{self._rows}, {h}, {D}] "
                             f"with contiguous heads on {self._dev}, got {t.dtype} {tuple(sh)} strides {st}")
        return st[0]

    def __call__(self, q, k, v, out, cache_args=None, out_checked=False):
        """q/out: [rows, Hq*D] or [rows, Hq, D]; k/v likewise with Hkv (any
        token stride, heads contiguous). Returns out. ``out_checked``: the
        caller made ``out`` itself with this launch's layout (the layer's own
        output buffer), so its check is skipped."""
        Hq, Hkv, D = self._heads
        idx = self._dev_index
        check = self._check
        qs0 = check("q", q, Hq)
        ks0 = check("k", k, Hkv)
        vs0 = check("v", v, Hkv)
        os0 = out.stride(0) if out_checked else check("out", out, Hq)
        if self._slots is not None:
            if cache_args is None or cache_args[2] != Hkv * D:
                raise ValueError("a paged launch needs paged_cache_args of num_kv_heads * head_dim rows")
            mid = tuple(cache_args) + self._slots
        else:
            mid = ()
        with _on_device(self._dev):
            stream = _raw_stream(idx) if _raw_stream is not None else _stream_ptr()
            ws = self._ws.get(stream)
            if ws is None:
                ws = sched_workspace(self._dev, stream)
                if ws:
                    self._ws[stream] = ws
            rc = self._fn(q.data_ptr(), qs0, k.data_ptr(), ks0, v.data_ptr(), vs0,
                          *mid, out.data_ptr(), os0, *self._tail, ws, self._status, stream)
        if rc:
            _native.check(rc, "varlen_attention")
        LAUNCHES[0] += 1
        return out


def paged_cache_args(k_cache, v_cache, num_kv_heads, head_dim) -> tuple:
    """(k_cache ptr, v_cache ptr, slot row length, number of slots) of a paged
    KV cache [blocks, block_size, num_kv_heads, head_dim] (bf16, contiguous)."""
    if k_cache.device.type != "cuda" or v_cache.device != k_cache.device:
        raise ValueError("caches must be CUDA tensors on one device")
    if k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError("caches must be bfloat16")
    row = num_kv_heads * head_dim
    if (k_cache.numel() % row or v_cache.numel() != k_cache.numel()
            or not k_cache.is_contiguous() or not v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous [blocks, block_size, num_kv_heads, head_dim]")
    return (k_cache.data_ptr(), v_cache.data_ptr(), row, k_cache.numel() // row)


def prepare_attention(cu_seqlens_q, cu_seqlens_k, max_seqlen_q, total_rows, num_heads, num_kv_heads,
                      head_dim, softmax_scale, device, *, slots=None,
                      cu_seqlens_slots=None) -> AttentionLaunch:
    """Validates the step-level arguments of a varlen attention launch once and
    returns an AttentionLaunch for q/k/v/out of ``total_rows`` rows. With
    ``slots`` and ``cu_seqlens_slots`` the keys of sequence b are [its cached
    rows read by slot from the paged cache given per call ; its fresh rows]
    (dllm_attn_varlen_paged_fwd)."""
    if head_dim != 128:
        raise NotImplementedError("head_dim must be 128")
    for name, c in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        if c.dtype != torch.int32 or not c.is_contiguous() or c.device != device:
            raise ValueError(f"{name} must be contiguous int32 on {device}")
    B = cu_seqlens_q.numel() - 1
    if cu_seqlens_k.numel() != B + 1:
        raise ValueError("cu_seqlens_q and cu_seqlens_k sizes differ")
    lib = _native.lib()
    tail = (cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), B, int(max_seqlen_q), int(total_rows),
            int(total_rows), num_heads, num_kv_heads, head_dim, float(softmax_scale))
    if slots is not None:
        for name, c in (("slots", slots), ("cu_seqlens_slots", cu_seqlens_slots)):
            if c is None or c.dtype != torch.int32 or not c.is_contiguous() or c.device != device:
                raise ValueError(f"{name} must be contiguous int32 on {device}")
        if cu_seqlens_slots.numel() != B + 1:
            raise ValueError("cu_seqlens_slots must have batch+1 entries")
        return AttentionLaunch(lib.dllm_attn_varlen_paged_fwd, (slots.data_ptr(), cu_seqlens_slots.data_ptr()),
                               tail, device, (num_heads, num_kv_heads, head_dim), total_rows)
    return AttentionLaunch(lib.dllm_attn_varlen_fwd, None, tail, device,
                           (num_heads, num_kv_heads, head_dim), total_rows)


def _check_paged(q, k_cache, v_cache, slots, cu_seqlens_slots, B, Hkv, D) -> int:
    """Validates the paged-cache arguments; returns the cache row length."""
    _require_cuda(q, k_cache, v_cache, slots, cu_seqlens_slots)
    if k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError("caches must be bfloat16")
    row = Hkv * D
    if (k_cache.stride(-1) != 1 or k_cache.numel() % row or v_cache.numel() != k_cache.numel()
            or not k_cache.is_contiguous() or not v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous [blocks, block_size, num_kv_heads, head_dim]")
    for name, c in (("slots", slots), ("cu_seqlens_slots", cu_seqlens_slots)):
        if c.dtype != torch.int32 or not c.is_contiguous():
            raise ValueError(f"{name} must be contiguous int32")
    if cu_seqlens_slots.numel() != B + 1:
        raise ValueError("cu_seqlens_slots must have batch+1 entries")
    return row


def _varlen_attention_rope(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale,
                           positions, cos_sin, k_cache, v_cache, slots, cu_seqlens_slots, out):
    """On-chip rotary + attention (dllm_attn_varlen_rope_fwd); max_seqlen_q <= 128."""
    Hq, D = q.shape[1], q.shape[2]
    Hkv = k.shape[1]
    _check_rows("q", q, Hq, D)
    _check_rows("k", k, Hkv, D)
    _check_rows("v", v, Hkv, D)
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    dev = _require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k, positions, cos_sin)
    for name, c in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        if c.dtype != torch.int32 or not c.is_contiguous():
            raise ValueError(f"{name} must be contiguous int32")
    if positions.dtype != torch.int64 or not positions.is_contiguous() or positions.numel() != q.shape[0]:
        raise ValueError("positions must be contiguous int64 [num_tokens]")
    if k.shape[0] != q.shape[0]:
        raise ValueError("rope needs as many fresh key rows as query rows")
    if cos_sin.dtype != torch.float32 or not cos_sin.is_contiguous() or cos_sin.dim() != 2 or cos_sin.shape[1] != D:
        raise ValueError(f"cos_sin_cache must be contiguous float32 [max_position, {D}]")
    B = cu_seqlens_q.numel() - 1
    if cu_seqlens_k.numel() != B + 1:
        raise ValueError("cu_seqlens_q and cu_seqlens_k sizes differ")
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    else:
        _check_rows("out", out, Hq, D)
        if out.shape[0] != q.shape[0]:
            raise ValueError("out must have as many rows as q")
    lib = _native.lib()
    status = _status_ptr(dev)
    with _on_device(dev):
        stream = _stream_ptr()
        if k_cache is not None:
            row = _check_paged(q, k_cache, v_cache, slots, cu_seqlens_slots, B, Hkv, D)
            cache_args = (k_cache.data_ptr(), v_cache.data_ptr(), row, k_cache.numel() // row,
                          slots.data_ptr(), cu_seqlens_slots.data_ptr())
        else:
            cache_args = (None, None, 0, 0, None, None)
        rc = lib.dllm_attn_varlen_rope_fwd(
            positions.data_ptr(), cos_sin.data_ptr(), cos_sin.shape[0],
            q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
            *cache_args, out.data_ptr(), out.stride(0), cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(),
            B, int(max_seqlen_q), q.shape[0], k.shape[0], Hq, Hkv, D, float(softmax_scale), status, stream,
        )
    _native.check(rc, "varlen_attention(rope)")
    if B > 0 and q.shape[0] > 0:
        LAUNCHES[0] += 1
    return out


# ---------------------------------------------------------------------------
# Scoring + top-k + gather + store (attention.py:308-342, 344-413, 204-233)
# ---------------------------------------------------------------------------
def rope_neox(
    positions: torch.Tensor,
    query: torch.Tensor,
    key: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    *,
    query_out: torch.Tensor | None = None,
    key_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """NeoX rotary embedding of ``query`` [N, Hq, 128] and ``key`` [N, Hkv, 128]
    (bf16) at ``positions`` (int64 [N]) from the fp32 ``cos_sin_cache``
    [max_position, 128] (cos | sin), as RotaryEmbedding.forward
    (rotary_embedding.py:41-57). Writes ``query_out``/``key_out`` (new tensors
    by default; pass the inputs for in place) and returns them."""
    Hq, D = query.shape[1], query.shape[2]
    Hkv = key.shape[1]
    _check_rows("query", query, Hq, D)
    _check_rows("key", key, Hkv, D)
    dev = _require_cuda(positions, query, key, cos_sin_cache)
    if positions.dtype != torch.int64 or not positions.is_contiguous() or positions.numel() != query.shape[0]:
        raise ValueError("positions must be contiguous int64 [num_tokens]")
    if key.shape[0] != query.shape[0]:
        raise ValueError("query and key have different token counts")
    if (cos_sin_cache.dtype != torch.float32 or cos_sin_cache.dim() != 2 or cos_sin_cache.shape[1] != D
            or not cos_sin_cache.is_contiguous()):
        raise ValueError("cos_sin_cache must be contiguous float32 [max_position, head_dim]")
    if query_out is None:
        query_out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    if key_out is None:
        key_out = torch.empty(key.shape, dtype=key.dtype, device=key.device)
    _check_rows("query_out", query_out, Hq, D)
    _check_rows("key_out", key_out, Hkv, D)
    lib = _native.lib()
    with _on_device(dev):
        rc = lib.dllm_rope_neox(
            positions.data_ptr(), query.data_ptr(), query.stride(0), query_out.data_ptr(),
            query_out.stride(0), key.data_ptr(), key.stride(0), key_out.data_ptr(), key_out.stride(0),
            cos_sin_cache.data_ptr(), cos_sin_cache.shape[0], query.shape[0], Hq, Hkv, D,
            _status_ptr(dev), _stream_ptr(),
        )
    _native.check(rc, "rope_neox")
    if query.shape[0] > 0:
        LAUNCHES[0] += 1
    return query_out, key_out


def select_kv_store(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    seq_desc: torch.Tensor,
    max_klen: int,
    head_select: bool,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    slots: torch.Tensor,
    top_idx: torch.Tensor | None = None,
) -> None:
    """Score candidates, pick the top n_keep per sequence (per KV head with
    ``head_select``), write their K/V rows into ``slots`` of the cache and,
    if given, the chosen candidate indices into ``top_idx`` (int64)."""
    Hq, D = q.shape[1], q.shape[2]
    Hkv = k.shape[1]
    _check_rows("q", q, Hq, D)
    _check_rows("k", k, Hkv, D)
    _check_rows("v", v, Hkv, D)
    dev = _require_cuda(q, k, v, seq_desc, k_cache, v_cache, slots)
    if seq_desc.dtype != torch.int32 or seq_desc.dim() != 2 or seq_desc.shape[1] != _native.SEQ_DESC_INTS:
        raise ValueError("seq_desc must be int32 [n_seqs, 8]")
    if not seq_desc.is_contiguous() or slots.dtype != torch.int32 or not slots.is_contiguous():
        raise ValueError("seq_desc and slots must be contiguous int32")
    if k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError("caches must be bfloat16")
    row = Hkv * D
    if k_cache.stride(-1) != 1 or k_cache.numel() % row != 0 or v_cache.numel() != k_cache.numel():
        raise ValueError("caches must be contiguous rows of num_kv_heads*head_dim")
    if top_idx is not None:
        _require_cuda(q, top_idx)
        if top_idx.dtype != torch.int64 or not top_idx.is_contiguous():
            raise ValueError("top_idx must be contiguous int64")
    lib = _native.lib()
    with _on_device(dev):
        rc = lib.dllm_select_kv_store(
            q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
            seq_desc.data_ptr(), seq_desc.shape[0], int(max_klen), Hq, Hkv, D, int(bool(head_select)),
            k_cache.data_ptr(), v_cache.data_ptr(), row, k_cache.numel() // row, slots.data_ptr(),
            _ptr(top_idx), _status_ptr(dev), _stream_ptr(),
        )
    _native.check(rc, "select_kv_store")
    if seq_desc.shape[0] > 0 and max_klen > 0:
        LAUNCHES[0] += 1

