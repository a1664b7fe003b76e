// Importance scoring + top-k selection + gather + KV-cache store, sm_100a.
//
// Restates, for the "compute cache" state of a diffusion block:
//   _select_important_head_kv  (dllmserve/layers/attention.py:344-413, head_select=True)
//   _select_important_kv       (attention.py:308-342, head_select=False)
// followed by the gather of the selected candidate rows and store_kvcache
// into the sequence's slots (attention.py:204-233).
//
// One CTA per (sequence, KV head) with head_select, one CTA per sequence
// otherwise. The pass over the candidate keys is HBM-bound (one read of each
// candidate row); ranking runs in shared memory as a bitonic sort of 64-bit
// keys  (order-preserving score bits << 32) | (0xffffffff - candidate)  so the
// result is "descending score, ties by ascending candidate index".
#include "common.cuh"
#include "select_kv.h"

namespace dllm {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kD = 128;

DLLM_DEVICE uint32_t order_bits(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

DLLM_DEVICE void bf16x4_to_f32(uint2 w, float (&x)[4]) {
  x[0] = __uint_as_float(w.x << 16);
  x[1] = __uint_as_float(w.x & 0xffff0000u);
  x[2] = __uint_as_float(w.y << 16);
  x[3] = __uint_as_float(w.y & 0xffff0000u);
}

DLLM_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Candidate c of a sequence -> token row offset inside the sequence.
DLLM_DEVICE int cand_token(int c, int blk_start, int blk_len) {
  return c < blk_start ? c : c + blk_len;
}

template <bool kHeadSelect>
__global__ void __launch_bounds__(kThreads, 1) select_kv_kernel(SelectArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int seq = blockIdx.y;
  const int h = blockIdx.x;  // KV head (head_select) or 0
  const int* d = a.seq_desc + seq * 8;
  const int tok_start = d[0], L = d[1], blk_start = d[2], blk_len = d[3];
  const int n_keep = d[4], slot_off = d[5], idx_off = d[6], pool_k = d[7];
  const int Klen = L - blk_len;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (Klen <= 0 || n_keep <= 0) return;
  if (Klen > a.max_klen || n_keep > Klen || blk_start < 0 || blk_start + blk_len > L ||
      blk_len <= 0) {
    if (threadIdx.x == 0) set_error(a.err, kDevBadSequence);
    return;
  }

  // shared memory: q_avg [nq][128] f32 | scores [max_klen] f32 | keys [p2] u64
  const int nq = kHeadSelect ? a.group : a.Hq;  // query heads that score this CTA's rows
  float* q_avg = reinterpret_cast<float*>(smem);
  float* scores = q_avg + nq * kD;
  uint64_t* keys = reinterpret_cast<uint64_t*>(
      smem + (((size_t)nq * kD * 4 + (size_t)a.max_klen * 4 + 15) & ~(size_t)15));
  int p2 = 1;
  while (p2 < Klen) p2 <<= 1;

  // 1) q_avg = mean over the block's query rows (fp32), attention.py:367 / :315.
  const int qh0 = kHeadSelect ? h * a.group : 0;
  for (int e = threadIdx.x; e < nq * kD; e += kThreads) {
    const int g = e / kD, dd = e % kD;
    const __nv_bfloat16* qp =
        a.q + (int64_t)(tok_start + blk_start) * a.q_tok_stride + (int64_t)(qh0 + g) * kD + dd;
    float s = 0.f;
    for (int t = 0; t < blk_len; ++t) s += __bfloat162float(qp[(int64_t)t * a.q_tok_stride]);
    q_avg[e] = s / (float)blk_len;
  }
  __syncthreads();

  // 2) scores (one warp per candidate row), attention.py:374-384 / :317-326.
  if (kHeadSelect) {
    const int G = a.group;
    for (int c = warp; c < Klen; c += kWarps) {
      const int tok = tok_start + cand_token(c, blk_start, blk_len);
      const uint2 w = __ldg(reinterpret_cast<const uint2*>(a.k + (int64_t)tok * a.k_tok_stride +
                                                           (int64_t)h * kD) + lane);
      float x[4];
      bf16x4_to_f32(w, x);
      float best = -INFINITY;
      for (int g = 0; g < G; ++g) {
        const float4 qa = reinterpret_cast<const float4*>(q_avg + g * kD)[lane];
        float p = qa.x * x[0];
        p = fmaf(qa.y, x[1], p);
        p = fmaf(qa.z, x[2], p);
        p = fmaf(qa.w, x[3], p);
        p = warp_sum(p);
        best = fmaxf(best, p);
      }
      if (lane == 0) scores[c] = __fdiv_rn(best, a.sqrt_d);
    }
  } else {
    // Shared ranking: sum over every query head h of q_avg[h] . k[c, h / group].
    const int Hkv = a.Hkv, G = a.group;
    const int row_vec = Hkv * kD / 4;  // uint2 (4 bf16) per lane step
    for (int c = warp; c < Klen; c += kWarps) {
      const int tok = tok_start + cand_token(c, blk_start, blk_len);
      const uint2* kr = reinterpret_cast<const uint2*>(a.k + (int64_t)tok * a.k_tok_stride);
      float p = 0.f;
      for (int e = lane; e < row_vec; e += 32) {
        float x[4];
        bf16x4_to_f32(__ldg(kr + e), x);
        const int hk = (e * 4) / kD, dd = (e * 4) % kD;
        for (int g = 0; g < G; ++g) {
          const float* qa = q_avg + (hk * G + g) * kD + dd;
          p = fmaf(qa[0], x[0], p);
          p = fmaf(qa[1], x[1], p);
          p = fmaf(qa[2], x[2], p);
          p = fmaf(qa[3], x[3], p);
        }
      }
      p = warp_sum(p);
      if (lane == 0) scores[c] = __fdiv_rn(p, a.sqrt_d);
    }
  }
  __syncthreads();

  // 3) max_pool1d(kernel=pool_k, stride 1, padding pool_k/2)[:Klen] + sort keys,
  //    attention.py:386-393 / :328-335.
  const int pad = pool_k / 2;
  for (int c = threadIdx.x; c < p2; c += kThreads) {
    uint64_t key = 0;  // padding sorts last
    if (c < Klen) {
      float m = scores[c];
      if (pool_k > 1) {
        const int lo = max(0, c - pad), hi = min(Klen - 1, c - pad + pool_k - 1);
        m = -INFINITY;
        for (int j = lo; j <= hi; ++j) m = fmaxf(m, scores[j]);
      }
      key = ((uint64_t)order_bits(m) << 32) | (uint64_t)(0xffffffffu - (uint32_t)c);
    }
    keys[c] = key;
  }
  __syncthreads();

  // 4) descending bitonic sort of p2 keys, attention.py:402-404 / :341.
  for (int k = 2; k <= p2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < p2; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = keys[i], y = keys[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            keys[i] = y;
            keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }

  // 5) indices out + gather/store of the selected rows (attention.py:405-411, :222-233).
  for (int j = threadIdx.x; j < n_keep && a.top_idx != nullptr; j += kThreads) {
    const int c = (int)(0xffffffffu - (uint32_t)(keys[j] & 0xffffffffu));
    const int64_t o = kHeadSelect ? (int64_t)idx_off + (int64_t)h * n_keep + j : (int64_t)idx_off + j;
    a.top_idx[o] = c;
  }
  if (kHeadSelect) {
    // 16 lanes x 16 B = one 256-byte head row per half warp.
    const int half = threadIdx.x >> 4, hl = threadIdx.x & 15;
    for (int j = half; j < n_keep; j += kThreads / 16) {
      const int c = (int)(0xffffffffu - (uint32_t)(keys[j] & 0xffffffffu));
      const int64_t slot = a.slots[slot_off + j];
      if (slot < 0) continue;
      if (slot >= a.num_slots) {
        if (hl == 0) set_error(a.err, kDevSlotOutOfRange);
        continue;
      }
      const int64_t tok = tok_start + cand_token(c, blk_start, blk_len);
      const uint4* ks = reinterpret_cast<const uint4*>(a.k + tok * a.k_tok_stride + (int64_t)h * kD);
      const uint4* vs = reinterpret_cast<const uint4*>(a.v + tok * a.v_tok_stride + (int64_t)h * kD);
      uint4* kd = reinterpret_cast<uint4*>(a.k_cache + slot * a.cache_tok_stride + (int64_t)h * kD);
      uint4* vd = reinterpret_cast<uint4*>(a.v_cache + slot * a.cache_tok_stride + (int64_t)h * kD);
      kd[hl] = __ldg(ks + hl);
      vd[hl] = __ldg(vs + hl);
    }
  } else {
    const int row_vec = a.Hkv * kD / 8;  // uint4 per row
    for (int j = warp; j < n_keep; j += kWarps) {
      const int c = (int)(0xffffffffu - (uint32_t)(keys[j] & 0xffffffffu));
      const int64_t slot = a.slots[slot_off + j];
      if (slot < 0) continue;
      if (slot >= a.num_slots) {
        if (lane == 0) set_error(a.err, kDevSlotOutOfRange);
        continue;
      }
      const int64_t tok = tok_start + cand_token(c, blk_start, blk_len);
      const uint4* ks = reinterpret_cast<const uint4*>(a.k + tok * a.k_tok_stride);
      const uint4* vs = reinterpret_cast<const uint4*>(a.v + tok * a.v_tok_stride);
      uint4* kd = reinterpret_cast<uint4*>(a.k_cache + slot * a.cache_tok_stride);
      uint4* vd = reinterpret_cast<uint4*>(a.v_cache + slot * a.cache_tok_stride);
      for (int e = lane; e < row_vec; e += 32) {
        kd[e] = __ldg(ks + e);
        vd[e] = __ldg(vs + e);
      }
    }
  }
}

}  // namespace

size_t select_kv_smem_bytes(int nq, int max_klen) {
  int p2 = 1;
  while (p2 < max_klen) p2 <<= 1;
  const size_t head = (((size_t)nq * kD * 4 + (size_t)max_klen * 4 + 15) & ~(size_t)15);
  return head + (size_t)p2 * 8;
}

cudaError_t launch_select_kv(const SelectArgs& a, bool head_select, int n_seqs, cudaStream_t stream) {
  if (n_seqs == 0) return cudaSuccess;
  const int nq = head_select ? a.group : a.Hq;
  const size_t smem = select_kv_smem_bytes(nq, a.max_klen);
  dim3 grid(head_select ? a.Hkv : 1, n_seqs);
  // The dynamic-smem opt-in is per device and kernel; raise it only when a
  // launch needs more than before (so steady-state launches, including ones
  // recorded into a CUDA graph, make no attribute calls).
  static size_t smem_set[2][64] = {{0}};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  size_t* have = (dev >= 0 && dev < 64) ? &smem_set[head_select ? 1 : 0][dev] : nullptr;
  if (have == nullptr || *have < smem) {
    e = head_select ? cudaFuncSetAttribute(select_kv_kernel<true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                    : cudaFuncSetAttribute(select_kv_kernel<false>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (have != nullptr) *have = smem;
  }
  if (head_select)
    select_kv_kernel<true><<<grid, kThreads, smem, stream>>>(a);
  else
    select_kv_kernel<false><<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace dllm
