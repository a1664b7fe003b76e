"""Build libdllm_attn.so (the sm_100a kernels + C ABI) in-tree with nvcc.

Usage: python dllm-serve_b200/build_lib.py [--force] [--ptxas-verbose]

The library lands next to the Python package (dllmserve_b200/libdllm_attn.so)
so that it travels with the repository snapshot and is the file the package
loads. nvcc cross-compiles for sm_100a without a GPU.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
OUT = os.path.join(HERE, "dllmserve_b200", "libdllm_attn.so")
SOURCES = ["attn_fwd.cu", "attn_fwd_split.cu", "kvcache.cu", "select_kv.cu", "rope.cu", "step_plan.cu",
           "oproj_ar.cu", "capi.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xlinker", "--no-undefined",
    "--expt-relaxed-constexpr",
    "-shared",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, "dllm_attn.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, ptxas_verbose: bool = False) -> str:
    if not force and not _stale():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    tmp = OUT + ".tmp"
    cmd += ["-o", tmp]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libdllm_attn.so")
    if ptxas_verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, ptxas_verbose=args.ptxas_verbose))
