// Importance scoring + top-k selection + gather + KV-cache store, sm_100a.
//
// Restates, for the "compute cache" state of a diffusion block:
//   _select_important_head_kv  (dllmserve/layers/attention.py:344-413, head_select=True)
//   _select_important_kv       (attention.py:308-342, head_select=False)
// followed by the gather of the selected candidate rows and store_kvcache
// into the sequence's slots (attention.py:204-233).
//
// One CTA per (sequence, KV head) with head_select; without it a cluster of
// kClusterCtas CTAs per sequence that exchange scores and the selection
// through distributed shared memory (no multicast copies). The pass over the candidate keys is HBM-bound (one read of each
// candidate row, several rows in flight per half warp). Ranking runs in shared
// memory: a radix select (4 passes of 8 bits) finds the n_keep-th largest
// pooled score T, the keys above T plus the lowest-index keys equal to T are
// compacted, and only those n_keep keys are bitonic-sorted as 64-bit
// (order-preserving score bits << 32) | (0xffffffff - candidate), so the result
// is "descending score, ties by ascending candidate index".
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "select_kv.h"

namespace cg = cooperative_groups;

namespace dllm {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kD = 128;
constexpr int kRowsInFlight = 4;                     // candidate rows per half warp per pass
constexpr int kFullSortMax = 512;  // up to this many (padded) candidates the whole set is sorted, no select
// Shared ranking (head_select off) runs as a cluster of kClusterCtas CTAs per
// sequence: all score a slice of the candidates into the leader's shared
// memory, the leader selects, all gather a slice of the selected rows.
constexpr int kClusterCtas = 8;  // up to this many (padded) keys a full sort beats radix select

DLLM_DEVICE uint32_t order_bits(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

DLLM_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

DLLM_DEVICE uint64_t shfl_xor_u64(uint64_t v, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), m);
  return ((uint64_t)hi << 32) | lo;
}

// Descending bitonic sort of sel[0, p2) (p2 a power of two, 32 <= p2 and
// p2 / E <= kThreads), called by every thread of the CTA. Element i lives in thread t = i / (32E) * 32 + i % 32, register
// e = (i / 32) % E, so compare-exchange partners at distance j < 32 are lanes
// of one warp (shuffles), at 32 <= j < 32E registers of one thread, and only
// j >= 32E goes through shared memory (one synchronised pass each): the
// network is the same as the plain shared-memory one, with far fewer passes.
template <int E>
DLLM_DEVICE void sort_desc_regs(uint64_t* sel, int p2) {
  const int t = threadIdx.x, lane = t & 31;
  const bool act = t < p2 / E;  // whole warps (p2 / E is a multiple of 32)
  const int base = (t >> 5) * 32 * E + lane;
  uint64_t x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = act ? sel[base + e * 32] : 0ull;
  for (int k = 2; k <= p2; k <<= 1) {
    if (k > 32 * E) {
      if (act) {
#pragma unroll
        for (int e = 0; e < E; ++e) sel[base + e * 32] = x[e];
      }
      __syncthreads();
      for (int j = k >> 1; j >= 32 * E; j >>= 1) {
        for (int i = t; i < p2; i += kThreads) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const uint64_t a = sel[i], b = sel[ixj];
            const bool desc = (i & k) == 0;
            if (desc ? (a < b) : (a > b)) {
              sel[i] = b;
              sel[ixj] = a;
            }
          }
        }
        __syncthreads();
      }
      if (act) {
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = sel[base + e * 32];
      }
    }
    if (act) {
      // partners in this thread's registers (j = 32d), d fixed at compile time
#pragma unroll
      for (int d = E / 2; d >= 1; d >>= 1) {
        if (32 * d <= (k >> 1)) {
#pragma unroll
          for (int e = 0; e < E; ++e) {
            if ((e & d) == 0) {
              const bool desc = ((base + e * 32) & k) == 0;
              const uint64_t a = x[e], b = x[e | d];
              const bool swap = desc ? (a < b) : (a > b);
              x[e] = swap ? b : a;
              x[e | d] = swap ? a : b;
            }
          }
        }
      }
      // partners in other lanes of the warp
      for (int j = min(k >> 1, 16); j > 0; j >>= 1) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const uint64_t y = shfl_xor_u64(x[e], j);
          const int i = base + e * 32;
          const bool lower = (i & j) == 0, desc = (i & k) == 0;
          x[e] = (lower == desc) ? (x[e] > y ? x[e] : y) : (x[e] < y ? x[e] : y);
        }
      }
    }
  }
  if (act) {
#pragma unroll
    for (int e = 0; e < E; ++e) sel[base + e * 32] = x[e];
  }
  __syncthreads();
}

// Candidate c of a sequence -> token row offset inside the sequence.
DLLM_DEVICE int cand_token(int c, int blk_start, int blk_len) {
  return c < blk_start ? c : c + blk_len;
}

// kGroup (head_select only): more than one query head per KV head. The two
// cases are separate instantiations so that the grouped scoring's registers
// do not cost the single-head scoring loop.
template <bool kHeadSelect, bool kGroup>
__global__ void __launch_bounds__(kThreads, 2) select_kv_kernel(SelectArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int seq = blockIdx.y;
  const int h = kHeadSelect ? blockIdx.x : 0;  // KV head (head_select)
  // shared ranking: rank in the sequence's cluster (0 = leader)
  const int crank = kHeadSelect ? 0 : (int)cg::this_cluster().block_rank();
  griddep_wait();  // inputs are read only after the previous grid in the stream finished
  griddep_launch_dependents();
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

  // shared memory: q_avg [nq][128] f32 | scores [max_klen] f32 | sel [p2(max_klen)] u64 |
  // hist [256] u32 | wsum [kWarps] u32 | misc [4] u32
  const int nq = kHeadSelect ? a.group : a.Hq;  // query heads that score this CTA's rows
  float* q_avg = reinterpret_cast<float*>(smem);
  float* scores = q_avg + nq * kD;
  int p2max = 32;
  while (p2max < a.max_klen) p2max <<= 1;
  uint64_t* sel = reinterpret_cast<uint64_t*>(
      smem + (((size_t)nq * kD * 4 + (size_t)a.max_klen * 4 + 15) & ~(size_t)15));
  uint32_t* hist = reinterpret_cast<uint32_t*>(sel + p2max);
  uint32_t* wsum = hist + 256;
  uint32_t* misc = wsum + kWarps;
  // the leader's scores / selection (distributed shared memory) for the shared path
  float* lead_scores = scores;
  const uint64_t* lead_sel = sel;
  if (!kHeadSelect) {
    lead_scores = cg::this_cluster().map_shared_rank(scores, 0);
    lead_sel = cg::this_cluster().map_shared_rank(sel, 0);
  }

  // 1) q_avg = mean over the block's query rows (fp32), attention.py:367 / :315.
  //    Eight interleaved partial sums (row t into partial t mod 8; rows past
  //    the last multiple of 8 into partial 0) combined as
  //    ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)), then an fp32 division. With one
  //    query head per CTA (MHA head_select: 128 elements) four consecutive
  //    threads share an element, thread j holding partials 2j and 2j+1, and
  //    the tree is two shuffles; otherwise a thread keeps all eight.
  const int qh0 = kHeadSelect ? h * a.group : 0;
  if (nq * kD * 4 == kThreads) {
    const int e = threadIdx.x >> 2, j = threadIdx.x & 3;
    const __nv_bfloat16* qp =
        a.q + (int64_t)(tok_start + blk_start) * a.q_tok_stride + (int64_t)qh0 * kD + e;
    float sa = 0.f, sb = 0.f;
    int t = 0;
    for (; t + 8 <= blk_len; t += 8) {
      sa += __bfloat162float(qp[(int64_t)(t + 2 * j) * a.q_tok_stride]);
      sb += __bfloat162float(qp[(int64_t)(t + 2 * j + 1) * a.q_tok_stride]);
    }
    if (j == 0)
      for (; t < blk_len; ++t) sa += __bfloat162float(qp[(int64_t)t * a.q_tok_stride]);
    float p = sa + sb;
    p += __shfl_xor_sync(0xffffffffu, p, 1);
    p += __shfl_xor_sync(0xffffffffu, p, 2);
    if (j == 0) q_avg[e] = p / (float)blk_len;
  } else {
    for (int e = threadIdx.x; e < nq * kD; e += kThreads) {
      const int g = e / kD, dd = e % kD;
      const __nv_bfloat16* qp =
          a.q + (int64_t)(tok_start + blk_start) * a.q_tok_stride + (int64_t)(qh0 + g) * kD + dd;
      // 8 independent partial sums keep 8 loads in flight per thread
      float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      int t = 0;
      for (; t + 8 <= blk_len; t += 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) s8[u] += __bfloat162float(qp[(int64_t)(t + u) * a.q_tok_stride]);
      }
      for (; t < blk_len; ++t) s8[0] += __bfloat162float(qp[(int64_t)t * a.q_tok_stride]);
      const float s = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
      q_avg[e] = s / (float)blk_len;
    }
  }
  if (threadIdx.x == 0) misc[2] = 0;  // selection counter
  if (kHeadSelect) {
    __syncthreads();
  } else {
    cg::this_cluster().sync();  // every CTA of the cluster runs before any remote access
  }

  // 2) scores, attention.py:374-384 / :317-326.
  if (kHeadSelect) {
    // Half warp per candidate row (16 lanes x 8 bf16 = the 128-dim head row),
    // kRowsInFlight rows per half warp per pass.
    const int G = a.group;
    const int hw = threadIdx.x >> 4, hl = threadIdx.x & 15;
    constexpr int kHalves = kThreads / 16;
    // The trip count is uniform over the warp (both halves step together), so
    // the 16-lane shuffle reductions always run with all 32 lanes.
    // Software-pipelined: the next batch's rows are requested before the
    // current batch is scored, so every half warp keeps 2 x kRowsInFlight
    // row loads outstanding instead of waiting a full memory latency per batch.
    constexpr int kStride = kHalves * kRowsInFlight;
    auto load_batch = [&](int cw, uint4 (&w)[kRowsInFlight]) {
      const int c0 = cw + (hw & 1);
#pragma unroll
      for (int r = 0; r < kRowsInFlight; ++r) {
        const int c = c0 + r * kHalves;
        w[r] = make_uint4(0, 0, 0, 0);
        if (c < Klen) {
          const int tok = tok_start + cand_token(c, blk_start, blk_len);
          w[r] = __ldg(reinterpret_cast<const uint4*>(a.k + (int64_t)tok * a.k_tok_stride +
                                                      (int64_t)h * kD) + hl);
        }
      }
    };
    // the lane's 8 query-mean values of the group's first head stay in registers
    const float4 qa0 = reinterpret_cast<const float4*>(q_avg)[2 * hl];
    const float4 qb0 = reinterpret_cast<const float4*>(q_avg)[2 * hl + 1];
    uint4 w[kRowsInFlight], wn[kRowsInFlight];
    if (2 * warp < Klen) load_batch(2 * warp, w);
    for (int cw = 2 * warp; cw < Klen; cw += kStride) {
      if (cw + kStride < Klen) load_batch(cw + kStride, wn);
      const int c0 = cw + (hw & 1);
#pragma unroll
      for (int r = 0; r < kRowsInFlight; ++r) {
        float x[8];
        bf16x8_to_f32(w[r], x);
        // lane partial of q_avg[g] . k over this lane's 8 dimensions
        auto dot8 = [&](int g) -> float {
          const float4 qa = g == 0 ? qa0 : reinterpret_cast<const float4*>(q_avg + g * kD)[2 * hl];
          const float4 qb = g == 0 ? qb0 : reinterpret_cast<const float4*>(q_avg + g * kD)[2 * hl + 1];
          float p = qa.x * x[0];
          p = fmaf(qa.y, x[1], p);
          p = fmaf(qa.z, x[2], p);
          p = fmaf(qa.w, x[3], p);
          p = fmaf(qb.x, x[4], p);
          p = fmaf(qb.y, x[5], p);
          p = fmaf(qb.z, x[6], p);
          p = fmaf(qb.w, x[7], p);
          return p;
        };
        float best = -INFINITY;
        if constexpr (!kGroup) {
          best = dot8(0);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) best += __shfl_xor_sync(0xffffffffu, best, o);
        } else if (G <= 8) {
          // GQA: the 16-lane xor-tree sums of all (up to 8) group heads at once,
          // as a reduce-scatter: at distance 8, 4, 2 each lane keeps half of its
          // heads and adds its partner's partials of them, then distance 1; every
          // head's sum is the same tree (the same bits) as one reduction per
          // head, in 8 shuffles instead of 4 per head. Lanes 2h, 2h+1 end with
          // head h; the maximum is then taken over the heads in order (one
          // shuffle per head).
          float hs[8];
#pragma unroll
          for (int g = 0; g < 8; ++g) hs[g] = g < G ? dot8(g) : 0.f;
          const bool u8 = (hl & 8) != 0, u4 = (hl & 4) != 0, u2 = (hl & 2) != 0;
          float h4[4], h2[2];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            h4[i] = (u8 ? hs[4 + i] : hs[i]) + __shfl_xor_sync(0xffffffffu, u8 ? hs[i] : hs[4 + i], 8);
#pragma unroll
          for (int i = 0; i < 2; ++i)
            h2[i] = (u4 ? h4[2 + i] : h4[i]) + __shfl_xor_sync(0xffffffffu, u4 ? h4[i] : h4[2 + i], 4);
          float d = (u2 ? h2[1] : h2[0]) + __shfl_xor_sync(0xffffffffu, u2 ? h2[0] : h2[1], 2);
          d += __shfl_xor_sync(0xffffffffu, d, 1);
          for (int g = 0; g < G; ++g) best = fmaxf(best, __shfl_sync(0xffffffffu, d, (lane & 16) + 2 * g));
        } else {
          for (int g = 0; g < G; ++g) {
            float p = dot8(g);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
            best = fmaxf(best, p);
          }
        }
        const int c = c0 + r * kHalves;
        if (hl == 0 && c < Klen) scores[c] = best;  // divided by sqrt(D) in the pooling pass
      }
#pragma unroll
      for (int r = 0; r < kRowsInFlight; ++r) w[r] = wn[r];
    }
  } else {
    // Shared ranking: sum over every query head h of q_avg[h] . k[c, h / group].
    // Warp per candidate row, 16 bytes per lane, kVecBatch loads in flight per lane.
    const int Hkv = a.Hkv, G = a.group;
    const int row_vec = Hkv * kD / 8;  // uint4 (8 bf16) per lane step
    constexpr int kVecBatch = 8;
    for (int c = crank * kWarps + warp; c < Klen; c += kClusterCtas * kWarps) {
      const int tok = tok_start + cand_token(c, blk_start, blk_len);
      const uint4* kr = reinterpret_cast<const uint4*>(a.k + (int64_t)tok * a.k_tok_stride);
      float p = 0.f;
      for (int e0 = 0; e0 < row_vec; e0 += 32 * kVecBatch) {
        uint4 w[kVecBatch];
#pragma unroll
        for (int u = 0; u < kVecBatch; ++u) {
          const int e = e0 + u * 32 + lane;
          w[u] = e < row_vec ? __ldg(kr + e) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kVecBatch; ++u) {
          const int e = e0 + u * 32 + lane;
          if (e >= row_vec) continue;
          float x[8];
          bf16x8_to_f32(w[u], x);
          const int hk = (e * 8) / kD, dd = (e * 8) % kD;
          for (int g = 0; g < G; ++g) {
            const float* qa = q_avg + (hk * G + g) * kD + dd;
#pragma unroll
            for (int i = 0; i < 8; ++i) p = fmaf(qa[i], x[i], p);
          }
        }
      }
      p = warp_sum(p);
      if (lane == 0) lead_scores[c] = p;  // divided by sqrt(D) in the pooling pass
    }
  }
  if (kHeadSelect) {
    __syncthreads();
  } else {
    cg::this_cluster().sync();  // every score is in the leader's shared memory
  }
  if (kHeadSelect || crank == 0) {

  // 3) scores / sqrt(D) (an IEEE fp32 division, attention.py:376-383 / :324-325) and
  //    max_pool1d(kernel=pool_k, stride 1, padding pool_k/2)[:Klen]
  //    (attention.py:386-393 / :328-335), as order-preserving bits, computed
  //    once: into the (still unused) selection buffer, then copied over the
  //    raw scores, which nothing reads afterwards; every later pass reads one
  //    word per key. The division of the window's maximum equals the maximum
  //    of the divided scores bit for bit (division by a positive constant is
  //    monotonic in round-to-nearest), so each key is divided once.
  const int pad = pool_k / 2;
  uint32_t* pbits = reinterpret_cast<uint32_t*>(scores);
  {
    uint32_t* tmp = reinterpret_cast<uint32_t*>(sel);  // 2 * p2max >= Klen words
    for (int c = threadIdx.x; c < Klen; c += kThreads) {
      float m = scores[c];
      if (pool_k > 1) {
        const int lo = max(0, c - pad), hi = min(Klen - 1, c - pad + pool_k - 1);
        m = -INFINITY;
        for (int j = lo; j <= hi; ++j) m = fmaxf(m, scores[j]);
      }
      tmp[c] = order_bits(__fdiv_rn(m, a.sqrt_d));
    }
    __syncthreads();
    for (int c = threadIdx.x; c < Klen; c += kThreads) pbits[c] = tmp[c];
    __syncthreads();
  }

  int p2k = 1;
  while (p2k < Klen) p2k <<= 1;
  const bool full_sort = p2k <= kFullSortMax;
  // 4) radix select (MSB first, 8 bits a pass) of the n_keep-th largest pooled
  //    score T; `krem` = how many keys equal to T belong to the top n_keep.
  //    Small candidate sets skip it (T = 0, every key selected, full sort).
  uint32_t prefix = 0, mask = 0;
  int krem = full_sort ? Klen : n_keep;
  for (int shift = 24; shift >= 0 && !full_sort; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    for (int cb = warp * 32; cb < Klen; cb += kThreads) {  // warp-uniform trip count
      const int c = cb + lane;
      const uint32_t v = c < Klen ? pbits[c] : 0u;
      const bool match = c < Klen && (v & mask) == prefix;
      const uint32_t active = __ballot_sync(0xffffffffu, match);
      if (match) {
        const uint32_t dig = (v >> shift) & 255u;
        const uint32_t peers = __match_any_sync(active, dig);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[dig], (uint32_t)__popc(peers));
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l holds bins 255-8l .. 248-8l (descending digit order)
      uint32_t cnt[8], sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cnt[i] = hist[255 - 8 * lane - i];
        sum += cnt[i];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const uint32_t excl = incl - sum;
      if (excl < (uint32_t)krem && (uint32_t)krem <= incl) {
        uint32_t acc = excl;
        for (int i = 0; i < 8; ++i) {
          if (acc + cnt[i] >= (uint32_t)krem) {
            misc[0] = 255u - 8u * lane - i;
            misc[1] = (uint32_t)krem - acc;
            break;
          }
          acc += cnt[i];
        }
      }
    }
    __syncthreads();
    prefix |= misc[0] << shift;
    mask |= 255u << shift;
    krem = (int)misc[1];
  }
  const uint32_t T = prefix;  // order bits are never 0 (NaN-free scores), so T = 0 keeps every key

  // 5) compaction: every key above T, and the krem keys equal to T with the
  //    lowest candidate indices (ties by ascending index), in any order. With
  //    the whole set sorted every key goes in: a plain copy.
  if (full_sort) {
    for (int c = threadIdx.x; c < Klen; c += kThreads)
      sel[c] = ((uint64_t)pbits[c] << 32) | (uint64_t)(0xffffffffu - (uint32_t)c);
  } else {
    uint32_t eq_base = 0;
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (int c0 = 0; c0 < Klen; c0 += kThreads) {
      const int c = c0 + threadIdx.x;
      const uint32_t v = c < Klen ? pbits[c] : 0u;
      const bool gt = c < Klen && v > T;
      const bool eq = c < Klen && v == T;
      const uint32_t be = __ballot_sync(0xffffffffu, eq);
      if (lane == 0) wsum[warp] = (uint32_t)__popc(be);
      __syncthreads();
      uint32_t before = 0, total = 0;
      for (int w = 0; w < kWarps; ++w) {
        const uint32_t x = wsum[w];
        before += w < warp ? x : 0u;
        total += x;
      }
      const uint32_t rank = eq_base + before + (uint32_t)__popc(be & lt_mask);
      if (gt || (eq && rank < (uint32_t)krem)) {
        const uint32_t pos = atomicAdd(&misc[2], 1u);
        sel[pos] = ((uint64_t)v << 32) | (uint64_t)(0xffffffffu - (uint32_t)c);
      }
      eq_base += total;
      __syncthreads();
    }
  }
  const int n_sel = full_sort ? Klen : n_keep;
  int p2 = 32;
  while (p2 < n_sel) p2 <<= 1;
  for (int i = n_sel + threadIdx.x; i < p2; i += kThreads) sel[i] = 0;  // padding sorts last
  __syncthreads();

  // 6) descending sort of the n_sel selected keys, attention.py:402-404 / :341.
  if (p2 <= kThreads) {
    sort_desc_regs<1>(sel, p2);
  } else if (p2 <= 2 * kThreads) {
    sort_desc_regs<2>(sel, p2);
  } else if (p2 <= 4 * kThreads) {
    sort_desc_regs<4>(sel, p2);
  } else if (p2 <= 8 * kThreads) {
    sort_desc_regs<8>(sel, p2);
  } else {
    for (int k = 2; k <= p2; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < p2; i += kThreads) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const uint64_t x = sel[i], y = sel[ixj];
            const bool desc = (i & k) == 0;
            if (desc ? (x < y) : (x > y)) {
              sel[i] = y;
              sel[ixj] = x;
            }
          }
        }
        __syncthreads();
      }
    }
  }

  }  // selection (every CTA with head_select, the leader otherwise)
  if (!kHeadSelect) cg::this_cluster().sync();  // the leader's selection is final

  // 7) indices out + gather/store of the selected rows (attention.py:405-411, :222-233).
  for (int j = threadIdx.x; j < n_keep && a.top_idx != nullptr && crank == 0; j += kThreads) {
    const int c = (int)(0xffffffffu - (uint32_t)(sel[j] & 0xffffffffu));
    const int64_t o = kHeadSelect ? (int64_t)idx_off + (int64_t)h * n_keep + j : (int64_t)idx_off + j;
    a.top_idx[o] = c;
  }
  if (kHeadSelect) {
    // 16 lanes x 16 B = one 256-byte head row per half warp, kRowsInFlight rows at a time.
    const int half = threadIdx.x >> 4, hl = threadIdx.x & 15;
    constexpr int kHalves = kThreads / 16;
    for (int j0 = half; j0 < n_keep; j0 += kHalves * kRowsInFlight) {
      uint4 kv[kRowsInFlight][2];
      int64_t dst[kRowsInFlight];
#pragma unroll
      for (int r = 0; r < kRowsInFlight; ++r) {
        const int j = j0 + r * kHalves;
        dst[r] = -1;
        if (j < n_keep) {
          // the row loads do not wait for the slot (only the store needs it):
          // both memory latencies overlap
          const int c = (int)(0xffffffffu - (uint32_t)(sel[j] & 0xffffffffu));
          const int64_t tok = tok_start + cand_token(c, blk_start, blk_len);
          kv[r][0] = __ldg(reinterpret_cast<const uint4*>(a.k + tok * a.k_tok_stride + (int64_t)h * kD) + hl);
          kv[r][1] = __ldg(reinterpret_cast<const uint4*>(a.v + tok * a.v_tok_stride + (int64_t)h * kD) + hl);
          dst[r] = a.slots[slot_off + j];
        }
      }
#pragma unroll
      for (int r = 0; r < kRowsInFlight; ++r) {
        if (dst[r] < 0) continue;  // negative slot: skipped (padding convention)
        if (dst[r] >= a.num_slots) {
          if (hl == 0) set_error(a.err, kDevSlotOutOfRange);
          continue;
        }
        reinterpret_cast<uint4*>(a.k_cache + dst[r] * a.cache_tok_stride + (int64_t)h * kD)[hl] = kv[r][0];
        reinterpret_cast<uint4*>(a.v_cache + dst[r] * a.cache_tok_stride + (int64_t)h * kD)[hl] = kv[r][1];
      }
    }
  } else {
    const int row_vec = a.Hkv * kD / 8;  // uint4 per row
    for (int j = crank * kWarps + warp; j < n_keep; j += kClusterCtas * kWarps) {
      const int c = (int)(0xffffffffu - (uint32_t)(lead_sel[j] & 0xffffffffu));
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
#pragma unroll 8
      for (int e = lane; e < row_vec; e += 32) {
        kd[e] = __ldg(ks + e);
        vd[e] = __ldg(vs + e);
      }
    }
  }
  // the leader's shared memory must outlive the other CTAs' reads of it
  if (!kHeadSelect) cg::this_cluster().sync();
}

}  // namespace

size_t select_kv_smem_bytes(int nq, int max_klen) {
  int p2 = 32;
  while (p2 < max_klen) p2 <<= 1;
  const size_t head = (((size_t)nq * kD * 4 + (size_t)max_klen * 4 + 15) & ~(size_t)15);
  return head + (size_t)p2 * 8 + (256 + kWarps + 4) * 4;
}

cudaError_t launch_select_kv(const SelectArgs& a, bool head_select, int n_seqs, cudaStream_t stream) {
  if (n_seqs == 0) return cudaSuccess;
  const int nq = head_select ? a.group : a.Hq;
  const size_t smem = select_kv_smem_bytes(nq, a.max_klen);
  dim3 grid(head_select ? a.Hkv : kClusterCtas, n_seqs);
  // The dynamic-smem opt-in is per device and kernel; raise it only when a
  // launch needs more than before (so steady-state launches, including ones
  // recorded into a CUDA graph, make no attribute calls).
  // Host threads share these caches; raising the attribute is serialised so
  // that a concurrent smaller request never lowers it under a larger one.
  static std::atomic<size_t> smem_set[3][64];
  static std::mutex raise_mu;
  const int kind = head_select ? (a.group > 1 ? 2 : 1) : 0;
  void (*kernel)(SelectArgs) = kind == 0   ? select_kv_kernel<false, false>
                               : kind == 1 ? select_kv_kernel<true, false>
                                           : select_kv_kernel<true, true>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::atomic<size_t>* have = (dev >= 0 && dev < 64) ? &smem_set[kind][dev] : nullptr;
  if (have == nullptr || have->load(std::memory_order_acquire) < smem) {
    std::lock_guard<std::mutex> lock(raise_mu);
    const size_t target = have != nullptr ? std::max(have->load(), smem) : smem;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)target);
    if (e != cudaSuccess) return e;
    if (have != nullptr) have->store(target, std::memory_order_release);
  }
  if (head_select)
    return launch_pdl(kernel, grid, dim3(kThreads), smem, stream, a);
  return launch_pdl_cluster(kernel, grid, dim3(kThreads), smem, stream, kClusterCtas, a);
}

}  // namespace dllm
