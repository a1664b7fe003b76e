"""Golden-vector case definitions (shared by make_golden.py and the tests).

A sparse case runs two consecutive diffusion steps of one attention layer:
  step 1: every sparse sequence in state 1 (full attention + select + store),
  step 2: the same sequences in state 2 (block rows only, cached K/V reused).
Dense sequences (state 0) ride along in both steps.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class SeqSpec:
    prompt_len: int
    gen_len: int
    block_idx: int = 0
    sparse: bool = True          # False: no SparseConfig (dense every step)


@dataclass
class SparseCase:
    name: str
    seed: int
    kind: str                    # "grid" or "normal" (see inputs.py)
    num_heads: int
    num_kv_heads: int
    head_dim: int
    seqs: list
    retention_ratio: float = 0.5
    pool_kernel: int = 3
    head_select: bool = True
    block_len: int = 32
    num_pages: int = 8


SPARSE_CASES = [
    SparseCase("mha_head_select", 11, "grid", 4, 4, 128,
               [SeqSpec(40, 32), SeqSpec(70, 64, block_idx=0), SeqSpec(20, 32, sparse=False),
                SeqSpec(60, 64, block_idx=1)]),
    SparseCase("gqa7_head_select", 12, "grid", 7, 1, 128,
               [SeqSpec(50, 32), SeqSpec(33, 64, block_idx=1), SeqSpec(1, 32)]),
    SparseCase("gqa_shared", 13, "grid", 8, 2, 128,
               [SeqSpec(45, 32), SeqSpec(90, 64, block_idx=0)], head_select=False),
    SparseCase("mha_shared", 14, "grid", 4, 4, 128,
               [SeqSpec(64, 32), SeqSpec(20, 64, block_idx=1)], head_select=False),
    SparseCase("ratio_zero", 15, "grid", 4, 2, 128,
               [SeqSpec(40, 32), SeqSpec(96, 32)], retention_ratio=0.0),
    SparseCase("ratio_one", 16, "grid", 4, 2, 128,
               [SeqSpec(40, 32), SeqSpec(96, 32)], retention_ratio=1.0),
    SparseCase("pool1", 17, "grid", 4, 4, 128, [SeqSpec(80, 32), SeqSpec(30, 64)], pool_kernel=1),
    SparseCase("pool4_even", 18, "grid", 4, 4, 128, [SeqSpec(80, 32), SeqSpec(30, 64)],
               pool_kernel=4),
    SparseCase("pool5_shared", 19, "grid", 4, 2, 128, [SeqSpec(77, 32)], pool_kernel=5,
               head_select=False),
    SparseCase("normal_mha", 20, "normal", 4, 4, 128, [SeqSpec(100, 32), SeqSpec(50, 64)]),
    SparseCase("block16", 21, "grid", 4, 4, 128, [SeqSpec(60, 48, block_idx=2)], block_len=16),
]

# Config 1 of the benchmark spec: one bidirectional layer, fp32, LLaDA-8B head
# shape, 64 prompt + 32 block tokens, RoPE theta 5e5, dense.
C1 = dict(seed=0, prompt_len=64, gen_len=32, num_heads=32, num_kv_heads=32, head_dim=128,
          rope_theta=500000.0)

# Sparse-state traces: (delay_step, block_len, prompt_len, gen_len, n_steps)
STATE_TRACES = [
    (1, 32, 64, 128, 140),
    (0, 32, 10, 64, 70),
    (2, 16, 5, 48, 60),
    (3, 8, 0, 20, 30),
    (1, 32, 7, 0, 5),
]


# Selection at benchmark scale (BASELINE configs 3 and 4), one compute-cache
# step per sequence at its first generation block. Inputs: N(0,1) q/k/v with
# margin-separated keys (inputs.margin_selection_batch), so every fp32
# summation order ranks the candidates alike and the reference's top_idx can
# be matched index for index. Only top_idx is recorded (the outputs at this
# size are checked against the oracle on the GPU instead).
@dataclass
class SelectionCase:
    name: str
    seed: int
    num_heads: int
    num_kv_heads: int
    batch: int
    prompt_range: tuple
    gen_len: int
    head_select: bool
    retention_ratio: float = 0.5
    pool_kernel: int = 3
    block_len: int = 32
    scaled_heads: int = 0        # KV heads whose keys are scaled 3x (config 3's recipe)


SELECTION_CASES = [
    SelectionCase("c3_sel", 3, 32, 32, 8, (512, 512), 128, True, scaled_heads=4),
    SelectionCase("c4_sel_head", 4, 28, 4, 32, (128, 768), 256, True),
    SelectionCase("c4_sel_shared", 5, 28, 4, 32, (128, 768), 256, False),
]
