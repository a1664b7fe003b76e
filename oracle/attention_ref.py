"""CPU restatement (torch fp32 / numpy) of the reference's diffusion attention
path. TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Every function cites the reference lines it restates (paths relative to the
chosen-ox/dLLM-Serve project root).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F


# ---------------------------------------------------------------------------
# Sizing rules
# ---------------------------------------------------------------------------
def num_keep(klen: int, ratio: float) -> int:
    """dllmserve/layers/attention.py:396-399 and engine/sequence.py:119-123."""
    if klen <= 0:
        return 0
    return min(max(1, int(klen * ratio)), klen)


def block_boundaries(prompt_len: int, total_len: int, block_idx: int, block_len: int):
    """dllmserve/sparse/state.py:44-62."""
    if total_len - prompt_len <= 0:
        return prompt_len, 0
    start = prompt_len + block_idx * block_len
    return start, min(block_len, total_len - start)


# ---------------------------------------------------------------------------
# Non-causal varlen attention (stand-in for flash_attn_varlen_func,
# attention.py:289-299, causal=False)
# ---------------------------------------------------------------------------
def sdpa_seq(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """softmax(q k^T * scale) v for one sequence, fp32. q [Lq,Hq,D], k/v [Lk,Hkv,D];
    GQA shares KV head h//(Hq/Hkv) (flash-attn's grouping)."""
    qf, kf, vf = q.float(), k.float(), v.float()
    Hq, Hkv = qf.shape[1], kf.shape[1]
    if Hq != Hkv:
        kf = kf.repeat_interleave(Hq // Hkv, dim=1)
        vf = vf.repeat_interleave(Hq // Hkv, dim=1)
    if kf.shape[0] == 0:
        return torch.zeros_like(qf)
    o = F.scaled_dot_product_attention(
        qf.transpose(0, 1), kf.transpose(0, 1), vf.transpose(0, 1), scale=scale
    )
    return o.transpose(0, 1)


def varlen_attention(q, k, v, cu_q, cu_k, scale, kc=None, vc=None, cu_c=None) -> torch.Tensor:
    """Per-sequence non-causal attention over packed rows; with kc/vc/cu_c the
    keys of sequence b are [kc[cu_c[b]:cu_c[b+1]] ; k[cu_k[b]:cu_k[b+1]]]
    (the reuse-state concatenation of attention.py:261-263)."""
    cu_q = [int(x) for x in cu_q]
    cu_k = [int(x) for x in cu_k]
    out = torch.zeros(q.shape, dtype=torch.float32)
    for b in range(len(cu_q) - 1):
        qs = q[cu_q[b]:cu_q[b + 1]]
        ks = k[cu_k[b]:cu_k[b + 1]]
        vs = v[cu_k[b]:cu_k[b + 1]]
        if kc is not None:
            c0, c1 = int(cu_c[b]), int(cu_c[b + 1])
            ks = torch.cat([kc[c0:c1], ks], 0)
            vs = torch.cat([vc[c0:c1], vs], 0)
        if qs.shape[0]:
            out[cu_q[b]:cu_q[b + 1]] = sdpa_seq(qs, ks, vs, scale)
    return out


# ---------------------------------------------------------------------------
# KV cache (attention.py:11-92)
# ---------------------------------------------------------------------------
def store_kvcache(key, value, k_cache, v_cache, slots) -> None:
    """cache.view(-1, row)[slot[i]] = key[i] (store_kvcache_kernel, attention.py:11-30).
    Slots < 0 are skipped (the native kernel's documented convention)."""
    row = key.shape[1] * key.shape[2]
    kc = k_cache.view(-1, row)
    vc = v_cache.view(-1, row)
    s = torch.as_tensor(slots).long()
    keep = s >= 0
    kc[s[keep]] = key.reshape(-1, row)[keep]
    vc[s[keep]] = value.reshape(-1, row)[keep]


def load_kvcache(k_cache, v_cache, slots, num_kv_heads, head_dim):
    """out[i] = cache.view(-1, row)[slot[i]] (load_kvcache_kernel, attention.py:53-74)."""
    row = num_kv_heads * head_dim
    s = torch.as_tensor(slots).long()
    k = k_cache.view(-1, row)[s].view(-1, num_kv_heads, head_dim)
    v = v_cache.view(-1, row)[s].view(-1, num_kv_heads, head_dim)
    return k.clone(), v.clone()


# ---------------------------------------------------------------------------
# Importance scoring and top-k (attention.py:308-413)
# ---------------------------------------------------------------------------
def _div_sqrt_d(x: np.ndarray, head_dim: int) -> np.ndarray:
    """x / D**0.5 with the divisor rounded to fp32 and an IEEE fp32 division
    (the reference divides an fp32 tensor by the Python float D**0.5)."""
    return (x.astype(np.float32) / np.float32(math.sqrt(head_dim))).astype(np.float32)


def q_block_mean(q_block: torch.Tensor) -> np.ndarray:
    """q_block.mean(dim=0) in fp32 (attention.py:315, :367)."""
    qb = q_block.float().numpy()
    return (qb.sum(axis=0, dtype=np.float32) / np.float32(qb.shape[0])).astype(np.float32)


def head_scores(q_block, k_cand, num_heads, num_kv_heads) -> np.ndarray:
    """[Hkv, Klen] per-KV-head scores, max over the GQA group (attention.py:366-384)."""
    D = q_block.shape[2]
    q_avg = q_block_mean(q_block)                            # [Hq, D]
    kp = k_cand.float().numpy().transpose(1, 0, 2)           # [Hkv, Klen, D]
    G = num_heads // num_kv_heads
    qg = q_avg.reshape(num_kv_heads, G, D)
    s = np.einsum("hgd,hkd->hgk", qg.astype(np.float64), kp.astype(np.float64))
    s = _div_sqrt_d(s.astype(np.float32), D)
    return s.max(axis=1)


def shared_scores(q_block, k_cand, num_heads, num_kv_heads) -> np.ndarray:
    """[Klen] token scores summed over all heads (attention.py:314-326)."""
    D = q_block.shape[2]
    q_avg = q_block_mean(q_block)                            # [Hq, D]
    G = num_heads // num_kv_heads
    k_exp = np.repeat(k_cand.float().numpy(), G, axis=1)     # [Klen, Hq, D]
    s = np.einsum("hd,khd->k", q_avg.astype(np.float64), k_exp.astype(np.float64))
    return _div_sqrt_d(s.astype(np.float32), D)


# ---------------------------------------------------------------------------
# The same scores in the fp32 accumulation order of the GPU selection kernel
# (dllm-serve_b200/csrc/select_kv.cu). The reference fixes no summation order
# (it scores in bf16 on the GPU, fp32 on the CPU); restating the kernel's order
# makes scores -- and with them the top-k indices -- bit-identical on ANY
# input, so selection can be checked bit for bit on plain N(0,1) data at full
# size. Parity with the reference's own ordering is pinned separately, on
# margin-separated inputs where every summation order ranks alike.
# ---------------------------------------------------------------------------
def fma32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """fp32 fused multiply-add with one rounding (round to nearest even).
    The product of two fp32 values is exact in float64; the float64 sum's
    rounding error is recovered exactly (TwoSum), and the one case where
    rounding float64 -> fp32 can then differ from a single rounding (the
    float64 sum sits exactly halfway between two fp32 values) is corrected by
    the error's sign."""
    a64, b64, c64 = (np.asarray(x, dtype=np.float32).astype(np.float64) for x in (a, b, c))
    p = a64 * b64
    s = p + c64
    bv = s - p
    e = (p - (s - bv)) + (c64 - bv)
    r = s.astype(np.float32)
    r64 = r.astype(np.float64)
    toward = np.where(s > r64, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
    other = np.nextafter(r, toward)
    mid = (r64 + other.astype(np.float64)) * 0.5
    tie = (s != r64) & (s == mid) & (e != 0) & (np.sign(e) == np.sign(s - r64))
    return np.where(tie, other, r).astype(np.float32)


def q_block_mean_kernel_order(q_block: torch.Tensor) -> np.ndarray:
    """q_block.mean(dim=0) as the kernel sums it: eight interleaved fp32
    partial sums (row t into partial t mod 8, rows in increasing order; rows
    past the last multiple of 8 into partial 0), combined as
    ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)), then an fp32 division by the row count."""
    qb = q_block.float().numpy().astype(np.float32)
    n = qb.shape[0]
    s8 = np.zeros((8,) + qb.shape[1:], dtype=np.float32)
    t = 0
    while t + 8 <= n:
        for u in range(8):
            s8[u] = s8[u] + qb[t + u]
        t += 8
    while t < n:
        s8[0] = s8[0] + qb[t]
        t += 1
    tot = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]))
    return (tot / np.float32(n)).astype(np.float32)


def _xor_tree_sum(v: np.ndarray) -> np.ndarray:
    """Butterfly sum over the last axis (lanes): v_l += v_(l xor o) for
    o = n/2, ..., 1; every lane ends with the same value, returned."""
    n = v.shape[-1]
    lanes = np.arange(n)
    o = n // 2
    while o >= 1:
        v = (v + v[..., lanes ^ o]).astype(np.float32)
        o //= 2
    return v[..., 0]


def head_scores_kernel_order(q_block, k_cand, num_heads, num_kv_heads) -> np.ndarray:
    """head_scores() in the kernel's order: 16 lanes x 8 dims per candidate row;
    per lane the product of dims 8l and then an FMA chain over the next 7,
    a 16-lane butterfly sum, max over the GQA group, fp32 division by
    fp32(sqrt(D))."""
    D = q_block.shape[2]
    G = num_heads // num_kv_heads
    q_avg = q_block_mean_kernel_order(q_block).reshape(num_kv_heads, G, 16, 8)   # [Hkv,G,lane,i]
    kp = k_cand.float().numpy().astype(np.float32).transpose(1, 0, 2)           # [Hkv,Klen,D]
    kl = kp.reshape(num_kv_heads, 1, kp.shape[1], 16, 8)                        # [Hkv,1,Klen,lane,i]
    qa = q_avg[:, :, None, :, :]                                                # [Hkv,G,1,lane,i]
    p = (qa[..., 0] * kl[..., 0]).astype(np.float32)
    for i in range(1, 8):
        p = fma32(qa[..., i], kl[..., i], p)
    s = _xor_tree_sum(p)                                                        # [Hkv,G,Klen]
    s = s.max(axis=1)
    return (s / np.float32(math.sqrt(D))).astype(np.float32)


def shared_scores_kernel_order(q_block, k_cand, num_heads, num_kv_heads) -> np.ndarray:
    """shared_scores() in the kernel's order: a warp per candidate row, lane l
    taking the 8-element vectors e = l, l + 32, ... of the row (vector e is
    dims 8(e mod 16).. of KV head e div 16) and, for each, one FMA chain over
    the group's query heads then the 8 dims; a 32-lane butterfly sum; fp32
    division by fp32(sqrt(D))."""
    D = q_block.shape[2]
    G = num_heads // num_kv_heads
    q_avg = q_block_mean_kernel_order(q_block)                                  # [Hq, D]
    kc = k_cand.float().numpy().astype(np.float32).reshape(k_cand.shape[0], -1)  # [Klen, Hkv*D]
    row_vec = num_kv_heads * D // 8
    klen = kc.shape[0]
    p = np.zeros((klen, 32), dtype=np.float32)
    for e0 in range(0, row_vec, 32):
        lanes = np.arange(32)
        e = e0 + lanes
        valid = e < row_vec
        hk, dd = (e * 8) // D, (e * 8) % D
        for g in range(G):
            for i in range(8):
                qv = np.where(valid, q_avg[np.minimum(hk * G + g, num_heads - 1), np.minimum(dd + i, D - 1)],
                              np.float32(0))
                xv = kc[:, np.minimum(e * 8 + i, kc.shape[1] - 1)]                # [Klen, 32]
                nxt = fma32(qv[None, :], xv, p)
                p = np.where(valid[None, :], nxt, p)
    s = _xor_tree_sum(p)
    return (s / np.float32(math.sqrt(D))).astype(np.float32)


def select_kernel_order(q_block, k_cand, num_heads, num_kv_heads, pool_kernel, ratio, head_select):
    """top-k indices of the kernel-order scores: [Hkv, n_keep] with
    head_select, else [n_keep]."""
    if head_select:
        s = head_scores_kernel_order(q_block, k_cand, num_heads, num_kv_heads)
    else:
        s = shared_scores_kernel_order(q_block, k_cand, num_heads, num_kv_heads)
    return topk_desc(max_pool(s, pool_kernel), num_keep(k_cand.shape[0], ratio))


def max_pool(scores: np.ndarray, pool_kernel: int) -> np.ndarray:
    """F.max_pool1d(kernel=pool_kernel, stride=1, padding=pool_kernel//2)[..., :Klen]
    along the last axis, padding acting as -inf (attention.py:386-393, :328-335)."""
    if pool_kernel <= 1 or scores.shape[-1] == 0:
        return scores
    klen = scores.shape[-1]
    pad = pool_kernel // 2
    out = np.empty_like(scores)
    for c in range(klen):
        lo, hi = max(0, c - pad), min(klen - 1, c - pad + pool_kernel - 1)
        out[..., c] = scores[..., lo:hi + 1].max(axis=-1)
    return out


def topk_desc(scores: np.ndarray, n_keep: int) -> np.ndarray:
    """Indices of the n_keep largest scores along the last axis, ordered by
    descending score; equal scores by ascending index. (torch.topk at
    attention.py:341/:402-404 leaves the order of exact ties unspecified;
    this fixes it.)"""
    order = np.argsort(-scores.astype(np.float64), axis=-1, kind="stable")
    return order[..., :n_keep].astype(np.int64)


def select_important_head_kv(q_block, k_cand, v_cand, num_heads, num_kv_heads, pool_kernel, ratio):
    """attention.py:344-413: returns (top_idx [Hkv, n_keep], k_sel, v_sel [n_keep, Hkv, D])."""
    klen = k_cand.shape[0]
    if klen == 0:
        return np.zeros((num_kv_heads, 0), np.int64), k_cand, v_cand
    s = max_pool(head_scores(q_block, k_cand, num_heads, num_kv_heads), pool_kernel)
    idx = topk_desc(s, num_keep(klen, ratio))
    ti = torch.from_numpy(idx)
    kp, vp = k_cand.permute(1, 0, 2), v_cand.permute(1, 0, 2)
    e = ti.unsqueeze(-1).expand(-1, -1, k_cand.shape[2])
    k_sel = torch.gather(kp, 1, e).transpose(0, 1).contiguous()
    v_sel = torch.gather(vp, 1, e).transpose(0, 1).contiguous()
    return idx, k_sel, v_sel


def select_important_kv(q_block, k_cand, num_heads, num_kv_heads, pool_kernel, ratio) -> np.ndarray:
    """attention.py:308-342: one shared ranking -> indices [n_keep]."""
    s = max_pool(shared_scores(q_block, k_cand, num_heads, num_kv_heads), pool_kernel)
    return topk_desc(s, num_keep(k_cand.shape[0], ratio))


# ---------------------------------------------------------------------------
# RoPE (dllmserve/layers/rotary_embedding.py:6-57), used by config 1
# ---------------------------------------------------------------------------
def rope_cache(head_dim: int, max_pos: int, theta: float) -> torch.Tensor:
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor) -> torch.Tensor:
    """NeoX half-split rotation in fp32, cast back to x.dtype."""
    cos, sin = cache[positions].chunk(2, dim=-1)
    cos, sin = cos.unsqueeze(-2), sin.unsqueeze(-2)
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


# ---------------------------------------------------------------------------
# One layer of the diffusion step (attention.py:150-306)
# ---------------------------------------------------------------------------
@dataclass
class SeqMeta:
    """Host view of one sequence in a diffusion step.
    state: 0 dense, 1 compute+store cache, 2 reuse cache (sparse/state.py:150-163)."""
    state: int
    num_tokens: int          # L of the sequence
    prompt_len: int
    block_idx: int = 0
    block_len: int = 32      # SparseConfig.default_block_len
    ratio: float = 0.5
    pool_kernel: int = 3
    head_select: bool = False

    def block(self):
        return block_boundaries(self.prompt_len, self.num_tokens, self.block_idx, self.block_len)

    def rows(self) -> int:
        """Rows this sequence contributes to q/k/v (model_runner.py:240-283)."""
        return self.block()[1] if self.state == 2 else self.num_tokens

    def n_keep(self) -> int:
        return num_keep(self.num_tokens - self.block()[1], self.ratio)


def diffusion_layer(q, k, v, seqs, k_cache, v_cache, slot_lists, scale, num_heads, num_kv_heads,
                    record=None):
    """Reference semantics of Attention._mixed_sparse_dense_attention for one
    layer: returns the fp32 output [N, Hq, D]; mutates k_cache/v_cache for
    state-1 sequences; ``record`` (dict) receives per-sequence top_idx."""
    D = q.shape[2]
    Qs, Ks, Vs, pos = [], [], [], []
    row = 0
    for i, s in enumerate(seqs):
        n = s.rows()
        r0, r1 = row, row + n
        row = r1
        if s.state in (0, 1):
            Qs.append(q[r0:r1]); Ks.append(k[r0:r1]); Vs.append(v[r0:r1]); pos.append((r0, r1))
            if s.state == 1:
                b0, bl = s.block()
                blk = torch.arange(r0 + b0, r0 + b0 + bl)
                allr = torch.arange(r0, r1)
                ps = allr[~torch.isin(allr, blk)]
                if s.head_select:
                    idx, ksel, vsel = select_important_head_kv(
                        q[blk], k[ps], v[ps], num_heads, num_kv_heads, s.pool_kernel, s.ratio)
                else:
                    idx = select_important_kv(q[blk], k[ps], num_heads, num_kv_heads,
                                              s.pool_kernel, s.ratio)
                    ksel, vsel = k[ps][torch.from_numpy(idx)], v[ps][torch.from_numpy(idx)]
                if record is not None:
                    record[i] = idx
                store_kvcache(ksel, vsel, k_cache, v_cache, slot_lists[i])
        else:
            kc, vc = load_kvcache(k_cache, v_cache, slot_lists[i], num_kv_heads, D)
            Qs.append(q[r0:r1])
            Ks.append(torch.cat([kc, k[r0:r1]], 0))
            Vs.append(torch.cat([vc, v[r0:r1]], 0))
            pos.append((r0, r1))
    out = torch.zeros(q.shape, dtype=torch.float32)
    for (r0, r1), qs, ks, vs in zip(pos, Qs, Ks, Vs):
        out[r0:r1] = sdpa_seq(qs, ks, vs, scale)
    return out
