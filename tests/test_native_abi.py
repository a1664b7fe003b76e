"""CPU checks of the C ABI: the library loads, exports every symbol that
include/dllm_attn.h declares, and rejects bad arguments before any CUDA call."""
import ctypes
import os
import re

import pytest

from dllmserve_b200 import _native

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "dllm_attn.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DLLM_API\s+[\w\s\*]+?\b(dllm_\w+)\s*\(", text)))


def test_header_declares_the_bound_entry_points():
    assert declared_symbols() == sorted(_native.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.dllm_version() >= 100


def test_nm_exports_match_header():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted({l.split()[-1] for l in out.splitlines() if " T dllm_" in l})
    assert exported == declared_symbols()


def test_validation_errors_without_gpu():
    lib = _native.lib()
    # head_dim 64 is rejected before any device work
    rc = lib.dllm_attn_varlen_fwd(None, 0, None, 0, None, 0, None, 0, None, None, 1, 1, 1, 1,
                                  4, 4, 64, ctypes.c_float(0.1), None, None, None)
    assert rc == _native.DLLM_ERR_UNSUPPORTED
    assert "head_dim" in lib.dllm_last_error().decode()
    # GQA ratio must divide
    rc = lib.dllm_attn_varlen_fwd(None, 0, None, 0, None, 0, None, 0, None, None, 1, 1, 1, 1,
                                  6, 4, 128, ctypes.c_float(0.1), None, None, None)
    assert rc == _native.DLLM_ERR_UNSUPPORTED
    # non-positive scale
    rc = lib.dllm_attn_varlen_fwd(None, 0, None, 0, None, 0, None, 0, None, None, 1, 1, 1, 1,
                                  4, 4, 128, ctypes.c_float(0.0), None, None, None)
    assert rc == _native.DLLM_ERR_INVALID_ARG
    # a misaligned scheduler workspace is refused before any device work
    rc = lib.dllm_attn_varlen_fwd(None, 0, None, 0, None, 0, None, 0, None, None, 1, 1, 1, 1,
                                  4, 4, 128, ctypes.c_float(0.1), 2, None, None)
    assert rc == _native.DLLM_ERR_ALIGNMENT
    # empty batch is a no-op
    rc = lib.dllm_attn_varlen_fwd(None, 0, None, 0, None, 0, None, 0, None, None, 0, 0, 0, 0,
                                  4, 4, 128, ctypes.c_float(0.1), None, None, None)
    assert rc == _native.DLLM_OK
    # cached variant needs cu_seqlens_c
    rc = lib.dllm_attn_varlen_cached_fwd(None, 0, None, 0, None, 0, None, 0, None, 0, None, 0,
                                         None, None, None, 1, 1, 1, 1, 1, 4, 4, 128,
                                         ctypes.c_float(0.1), None, None, None)
    assert rc == _native.DLLM_ERR_INVALID_ARG
    # kv copies
    rc = lib.dllm_store_kvcache(None, 0, None, 0, None, None, None, 0, 8, 2, 1, None, None)
    assert rc == _native.DLLM_OK  # zero tokens
    rc = lib.dllm_store_kvcache(None, 0, None, 0, None, None, None, 4, 8, 3, 1, None, None)
    assert rc == _native.DLLM_ERR_INVALID_ARG  # elem_bytes
    rc = lib.dllm_load_kvcache(None, 0, None, 0, None, None, None, 4, 8, 2, 1, None, None)
    assert rc == _native.DLLM_ERR_INVALID_ARG  # null pointers
    # selection limits
    rc = lib.dllm_select_kv_store(None, 0, None, 0, None, 0, None, 1, 20000, 4, 4, 128, 1,
                                  None, None, 512, 1, None, None, None, None)
    assert rc == _native.DLLM_ERR_TOO_LARGE
    rc = lib.dllm_select_kv_store(None, 0, None, 0, None, 0, None, 0, 0, 4, 4, 128, 1,
                                  None, None, 512, 1, None, None, None, None)
    assert rc == _native.DLLM_OK


def test_check_maps_codes_to_python_errors():
    with pytest.raises(ValueError):
        _native.check(_native.DLLM_ERR_ALIGNMENT, "x")
    with pytest.raises(NotImplementedError):
        _native.check(_native.DLLM_ERR_UNSUPPORTED, "x")
    with pytest.raises(_native.DllmError):
        _native.check(_native.DLLM_ERR_CUDA, "x")


def test_ops_refuse_cpu_tensors():
    import torch
    from dllmserve_b200 import ops

    q = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    cu = torch.tensor([0, 4], dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        ops.varlen_attention(q, q, q, cu, cu, 4)


def test_rope_attention_validation_without_gpu():
    """dllm_attn_varlen_rope_fwd refuses bad arguments before any device work."""
    lib = _native.lib()
    f = ctypes.c_float(0.1)

    def call(positions=1, cos_sin=16, max_pos=16, slots=None, cu_slots=None, num_slots=0,
             batch=1, max_q=32, total_q=32, total_k=32, hd=128):
        return lib.dllm_attn_varlen_rope_fwd(
            positions, cos_sin, max_pos, None, 0, None, 0, None, 0, None, None, 0, num_slots,
            slots, cu_slots, None, 0, None, None, batch, max_q, total_q, total_k, 4, 4, hd, f, None, None)

    assert call(positions=None) == _native.DLLM_ERR_INVALID_ARG
    assert "positions" in lib.dllm_last_error().decode()
    assert call(slots=64, cu_slots=None) == _native.DLLM_ERR_INVALID_ARG  # slots without their offsets
    assert call(slots=64, cu_slots=64, num_slots=0) == _native.DLLM_ERR_INVALID_ARG
    assert call(cos_sin=None) == _native.DLLM_ERR_INVALID_ARG
    assert call(cos_sin=8) == _native.DLLM_ERR_ALIGNMENT  # cos/sin rows are read 16 bytes at a time
    assert call(max_q=129, total_q=129, total_k=129) == _native.DLLM_ERR_UNSUPPORTED
    assert "rotate first" in lib.dllm_last_error().decode()
    assert call(total_k=31) == _native.DLLM_ERR_INVALID_ARG  # one position per query and key row
    assert call(hd=64) == _native.DLLM_ERR_UNSUPPORTED
    assert call(batch=0, max_q=0, total_q=0, total_k=0) == _native.DLLM_OK  # empty: no-op
