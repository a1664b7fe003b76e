"""ctypes binding of libdllm_attn.so (the C ABI declared in include/dllm_attn.h).

There is no fallback: if the library is missing, every op raises
``NativeLibraryMissing`` (build it with ``python dllm-serve_b200/build_lib.py``).
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdllm_attn.so")

DLLM_OK = 0
DLLM_ERR_INVALID_ARG = 1
DLLM_ERR_UNSUPPORTED = 2
DLLM_ERR_ALIGNMENT = 3
DLLM_ERR_TOO_LARGE = 4
DLLM_ERR_CUDA = 5

DLLM_DEV_SLOT_OUT_OF_RANGE = 1
DLLM_DEV_WAIT_TIMEOUT = 2
DLLM_DEV_BAD_SEQUENCE = 3

SEQ_DESC_INTS = 8
PLAN_SEQ_FIELDS = 10   # DLLM_PLAN_SEQ_FIELDS
PLAN_LAYOUT_INTS = 12  # DLLM_PLAN_LAYOUT_INTS
PLAN_MAX_BATCH = 1024  # DLLM_PLAN_MAX_BATCH
OPROJ_MAX_RANKS = 8    # DLLM_OPROJ_MAX_RANKS
IPC_HANDLE_BYTES = 64  # DLLM_IPC_HANDLE_BYTES
SCHED_WORKSPACE_INTS = 2  # DLLM_SCHED_WORKSPACE_INTS

# Every exported entry point with its (argtypes, restype).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "dllm_version": ([], _I),
    "dllm_last_error": ([], ctypes.c_char_p),
    "dllm_store_kvcache": ([_P, _I64, _P, _I64, _P, _P, _P, _I64, _I64, _I, _I64, _P, _P], _I),
    "dllm_load_kvcache": ([_P, _I64, _P, _I64, _P, _P, _P, _I64, _I64, _I, _I64, _P, _P], _I),
    "dllm_attn_varlen_fwd": (
        [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I, _I, _I64, _I64, _I, _I, _I, _F, _P, _P, _P],
        _I,
    ),
    "dllm_attn_varlen_fwd_static_ws": (
        [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I, _I, _I64, _I64, _I, _I, _I, _F, _P, _P],
        _I,
    ),
    "dllm_attn_varlen_cached_fwd": (
        [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I, _I, _I64, _I64,
         _I64, _I, _I, _I, _F, _P, _P, _P],
        _I,
    ),
    "dllm_attn_varlen_paged_fwd": (
        [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _I64, _P, _P, _I, _I, _I64,
         _I64, _I, _I, _I, _F, _P, _P, _P],
        _I,
    ),
    "dllm_attn_varlen_rope_fwd": (
        [_P, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _I64, _P, _P,
         _I, _I, _I64, _I64, _I, _I, _I, _F, _P, _P],
        _I,
    ),
    "dllm_attn_varlen_heads_fwd": (
        [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _I64, _P, _P, _I, _I, _I64, _I64,
         _I, _I, _I, _F, _P, _I, _P, _P, _P],
        _I,
    ),
    "dllm_rope_neox": (
        [_P, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I, _I, _I, _P, _P],
        _I,
    ),
    "dllm_build_step_plan": ([_P, _I, _I, _P, _P, _P, _P], _I),
    "dllm_oproj_allreduce": ([_P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _I, _I, _I, _P, _P], _I),
    "dllm_ipc_export": ([_P, _P, _P], _I),
    "dllm_ipc_open": ([_P, _P], _I),
    "dllm_ipc_close": ([_P], _I),
    "dllm_select_kv_store": (
        [_P, _I64, _P, _I64, _P, _I64, _P, _I, _I, _I, _I, _I, _I, _P, _P, _I64, _I64, _P, _P, _P, _P],
        _I,
    ),
}


class NativeLibraryMissing(RuntimeError):
    pass


class DllmError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[dllm error {code}] {message}")
        self.code = code


_lib = None
_lock = threading.Lock()


def lib():
    """Load the shared library once and bind every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_PATH} not found; build it with `python dllm-serve_b200/build_lib.py`"
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc == DLLM_OK:
        return
    msg = lib().dllm_last_error().decode(errors="replace")
    if rc in (DLLM_ERR_INVALID_ARG, DLLM_ERR_ALIGNMENT):
        raise ValueError(f"{what}: {msg}")
    if rc == DLLM_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise DllmError(rc, f"{what}: {msg}")
