// Non-causal varlen flash-attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the `flash_attn_varlen_func(..., causal=False)` call of the
// reference's diffusion attention (dllmserve/layers/attention.py:289-299),
// including the cached-K/V ("reuse") sequences whose keys are the selected
// cached rows followed by the block's fresh rows (attention.py:235-265).
//
// Persistent kernel: one CTA per SM loops over work units = (sequence b,
// query head h, pair of 128-row query tiles). Roles inside the CTA (11 warps):
//   warps 0-3  softmax warpgroup 0  (query tile 0, TMEM lanes 0-127)
//   warps 4-7  softmax warpgroup 1  (query tile 1)
//   warp  8    TMA producer: Q tiles and the K ring (kStagesK deep)
//   warp  9    MMA issuer (also allocates / frees TMEM)
//   warp  10   TMA producer: the V ring (kStagesV deep)
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// P_i (bf16) is written over the first 64 columns of S_i. The MMA issue
// order per KV tile j is  PV_i(j) then QK_i(j+1) for each tile i, so the next
// S_i overwrites P_i only after the PV that read it (tcgen05 MMAs of one
// thread execute in order).
//
// Each KV sequence is the concatenation of up to two segments:
//   segment 0: cached rows (k_cache/v_cache gathered rows, `cu_c`), optional
//   segment 1: fresh rows of the step's k/v (`cu_k`)
// KV tiles never straddle segments; a partial tile uses a smaller MMA N.
#include <atomic>

#include "common.cuh"
#include "attn_fwd.h"

namespace dllm {

namespace {

constexpr int kD = 128;          // head dim (only 128 is instantiated)
constexpr int kTileM = 128;      // query rows per tile
constexpr int kTileN = 128;      // kv rows per tile
constexpr int kStagesK = 3;      // K ring depth (K runs one tile ahead of V)
constexpr int kStagesV = 2;      // V ring depth
constexpr int kThreads = 352;

constexpr uint32_t kTileBytes = kTileM * kD * 2;  // 32 KB (bf16)
constexpr uint32_t kChunkBytes = 128 * 128;       // 128 rows x 128 B (64 bf16)

// Shared-memory map (offsets from a 1024-aligned base).
constexpr uint32_t kOffQ = 0;                                   // 2 tiles
constexpr uint32_t kOffK = kOffQ + 2 * kTileBytes;              // kStagesK tiles
constexpr uint32_t kOffV = kOffK + kStagesK * kTileBytes;       // kStagesV tiles
constexpr uint32_t kOffBar = kOffV + kStagesV * kTileBytes;     // barriers
constexpr uint32_t kNumBars = 2 + 2 * kStagesK + 2 * kStagesV + 2 + 2 + 2 + 1 + 2 * 4;  // + unit ring
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
constexpr uint32_t kOffRing = kOffMisc + 64;                   // kRing unit ids
constexpr int kOrderMaxSeqs = 128;                             // sequences a long-first launch may rank
constexpr uint32_t kOffOrder = kOffRing + 16;                  // long-first order + its keys
constexpr uint32_t kSmemBytes = kOffOrder + 8 * kOrderMaxSeqs + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "pair kernel shared memory over the 227 KB opt-in limit");
// A launch with at most this many units (counted as B * heads * qunits) per SM
// hands out long sequences first. Config-2 lengths (16 sequences of 419-1,087
// tokens): 4 heads 40.5 -> 38.8 us, 8 heads 63.4 -> 58.1 us, 16 heads (8.6
// units per SM) 108.6 -> 106.5 us; at 32 heads (17.3 per SM) long-first is
// 6 % slower than the sequence order, which then balances as well.
constexpr int kLongFirstUnitsPerSm = 10;

// barrier indices
constexpr int BAR_Q = 0;
constexpr int BAR_QEMPTY = 1;
constexpr int BAR_KFULL = 2;
constexpr int BAR_KEMPTY = BAR_KFULL + kStagesK;
constexpr int BAR_VFULL = BAR_KEMPTY + kStagesK;
constexpr int BAR_VEMPTY = BAR_VFULL + kStagesV;
constexpr int BAR_SFULL = BAR_VEMPTY + kStagesV;  // 2
constexpr int BAR_PFULL = BAR_SFULL + 2;         // 2
constexpr int BAR_OFULL = BAR_PFULL + 2;         // 2
constexpr int BAR_DRAIN = BAR_OFULL + 2;         // 1
constexpr int kRing = 4;                         // unit ids published ahead of their use
constexpr int BAR_UFULL = BAR_DRAIN + 1;         // kRing: unit id published
constexpr int BAR_UEMPTY = BAR_UFULL + kRing;    // kRing: every role read it

struct KvTile {
  int seg;    // 0 = cached, 1 = fresh
  int row0;   // first row in the segment's source tensor
  int valid;  // valid rows in this tile (1..128)
};

// Tile t of a sequence whose cached segment has nc rows starting at c0 and
// fresh segment nk rows starting at k0.
DLLM_DEVICE KvTile kv_tile(int t, int nc, int c0, int nk, int k0) {
  int tc = (nc + kTileN - 1) / kTileN;
  KvTile r;
  if (t < tc) {
    r.seg = 0;
    r.row0 = c0 + t * kTileN;
    r.valid = min(kTileN, nc - t * kTileN);
  } else {
    int u = t - tc;
    r.seg = 1;
    r.row0 = k0 + u * kTileN;
    r.valid = min(kTileN, nk - u * kTileN);
  }
  return r;
}

// P = 2^(S*scale_log2 - m) for one row of a 128-column tile (MUFU ex2),
// packed to bf16 pairs and stored to TMEM over the first 64 columns of the S
// tile; returns the row sum of P (fp32).
DLLM_DEVICE float exp_store_tile(const uint32_t (&s)[4][32], float sl2, float m, uint32_t tS) {
  const float neg_m = -m;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float p0 = ex2_approx(fmaf(__uint_as_float(s[c][2 * e]), sl2, neg_m));
      const float p1 = ex2_approx(fmaf(__uint_as_float(s[c][2 * e + 1]), sl2, neg_m));
      acc[(2 * e) & 3] += p0;
      acc[(2 * e + 1) & 3] += p1;
      pk[e] = pack_bf16x2(p0, p1);
    }
    tmem_st16(tS + c * 16, pk);
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

}  // namespace

// One work unit: (sequence b, query head hq, pair p of 128-row query tiles).
struct Unit {
  bool valid;
  int hq, hkv;
  int q_begin, Lq, q0, ntiles;
  int k_begin, nk, c_begin, nc, nkv;
};

// Units are numbered ((b * Hq) + hq) * qunits + p, so consecutive units share
// a sequence and head (their K/V stay hot in L2 while several CTAs read them).
DLLM_DEVICE Unit decode_unit(int u, const AttnKernelArgs& a) {
  Unit r;
  const int per_b = a.n_heads * a.qunits;
  const int b = u / per_b;
  const int rem = u - b * per_b;
  const int hsel = rem / a.qunits;
  const int p = rem - hsel * a.qunits;
  r.hq = a.head_idx != nullptr ? a.head_idx[hsel] : hsel;
  const bool head_ok = r.hq >= 0 && r.hq < a.Hq;
  if (!head_ok) r.hq = 0;
  r.hkv = r.hq / a.group;
  r.q_begin = a.cu_q[b];
  r.Lq = a.cu_q[b + 1] - r.q_begin;
  r.q0 = p * 2 * kTileM;
  r.valid = head_ok && r.q0 < r.Lq;
  r.ntiles = (r.Lq - r.q0 > kTileM) ? 2 : 1;
  r.k_begin = a.cu_k[b];
  r.nk = a.cu_k[b + 1] - r.k_begin;
  r.c_begin = 0;
  r.nc = 0;
  if (a.cu_c != nullptr) {
    r.c_begin = a.cu_c[b];
    r.nc = a.cu_c[b + 1] - r.c_begin;
  }
  r.nkv = (r.nc + kTileN - 1) / kTileN + (r.nk + kTileN - 1) / kTileN;
  return r;
}

// Persistent kernel. Warp 8 (lane 0) chooses the CTA's units and publishes
// them through a ring of kRing ids in shared memory that every role reads:
// with a scheduler workspace (args.sched, two int32 words that are zero on
// entry) CTA c starts at unit c and then claims gridDim.x + atomicAdd(counter)
// — the CTAs that finish early take the remaining units, which evens out
// batches of unequal sequence lengths — and the last CTA to exit zeroes the
// workspace again; without one, CTA c takes c, c + gridDim.x, ... Barrier
// phases run on across units (ring counters below), so the producer loads the
// next unit's Q/K/V and the MMA warp starts its QK while the softmax warps
// still write the previous unit's output.
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKc,
                    const __grid_constant__ CUtensorMap tmVc, AttnKernelArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_units = args.total_units;

  const uint32_t bar0 = base + kOffBar;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc + 16);

  if (threadIdx.x == 0) {
    mbar_init(bar(BAR_Q), 1);
    mbar_init(bar(BAR_QEMPTY), 1);
    for (int s = 0; s < kStagesK; ++s) {
      mbar_init(bar(BAR_KFULL + s), 1);
      mbar_init(bar(BAR_KEMPTY + s), 1);
    }
    for (int s = 0; s < kStagesV; ++s) {
      mbar_init(bar(BAR_VFULL + s), 1);
      mbar_init(bar(BAR_VEMPTY + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(BAR_SFULL + i), 1);
      mbar_init(bar(BAR_PFULL + i), 4);  // one arrival per softmax warp
      mbar_init(bar(BAR_OFULL + i), 1);
    }
    mbar_init(bar(BAR_DRAIN), 1);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(bar(BAR_UFULL + i), 1);
      mbar_init(bar(BAR_UEMPTY + i), 10);  // V producer, MMA thread, 8 softmax warps
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if (args.cu_c != nullptr) {
      tma_prefetch_desc(&tmKc);
      tma_prefetch_desc(&tmVc);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Everything above (barriers, TMEM, descriptor prefetch) may overlap the
  // previous kernel in the stream; every global access below comes after it.
  griddep_wait();
  griddep_launch_dependents();
  volatile int* uring = reinterpret_cast<volatile int*>(smem + kOffRing);
  // consumer side: next unit id from the ring (bounded wait); -1 on abort
  // warp_wide: every lane of the warp calls it (one arrival from lane 0);
  // otherwise a single thread calls it and arrives itself.
  auto take_unit = [&](uint32_t n, bool warp_wide) -> int {
    const bool got = warp_wide ? mbar_wait_warp(bar(BAR_UFULL + n % kRing), (n / kRing) & 1, abort_flag)
                               : mbar_wait(bar(BAR_UFULL + n % kRing), (n / kRing) & 1, abort_flag);
    if (!got) return -1;
    const int u = uring[n % kRing];
    if (warp_wide) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_UEMPTY + n % kRing));
    } else {
      mbar_arrive(bar(BAR_UEMPTY + n % kRing));
    }
    return u;
  };

  if (warp == 8 || warp == 10) {
    // ------------------------------------------------------------------ TMA
    // warp 8: Q and K tiles; warp 10: V tiles (independent rings, so a wait
    // for a free V stage never holds back a K load and vice versa). The whole
    // warp walks the loop (uniformly); lane 0 issues the TMA copies and the
    // barrier operations, all lanes help with paged cached tiles.
    const bool kq = warp == 8;
    const uint64_t pol_q = policy_evict_first();
    const uint64_t pol_kv = policy_evict_last();
    const int nst = kq ? kStagesK : kStagesV;
    const int bfull = kq ? BAR_KFULL : BAR_VFULL;
    const int bempty = kq ? BAR_KEMPTY : BAR_VEMPTY;
    const uint32_t ring = base + (kq ? kOffK : kOffV);
    const __nv_bfloat16* cache = kq ? args.kc : args.vc;
    uint32_t q_it = 0;     // units whose Q was loaded (warp 8)
    uint32_t done = 0;     // tiles issued into this ring
    int next_static = (int)blockIdx.x + (int)gridDim.x;  // static order (warp 8, lane 0)
    int* order = reinterpret_cast<int*>(smem + kOffOrder);
    if (kq && args.long_first) {
      // order[r] = the sequence handed out r-th: most key tiles first, ties by
      // index. key = min(tiles, 2^22) * kOrderMaxSeqs + (kOrderMaxSeqs - 1 - b)
      // is distinct per sequence (B <= kOrderMaxSeqs) and fits an int; a
      // sequence's rank is the number of larger keys.
      int* keys = order + kOrderMaxSeqs;
      const int B = args.B;
      for (int b = lane; b < B; b += 32) {
        const int nk = args.cu_k[b + 1] - args.cu_k[b];
        const int nc = args.cu_c != nullptr ? args.cu_c[b + 1] - args.cu_c[b] : 0;
        const int tiles = min((nc + kTileN - 1) / kTileN + (nk + kTileN - 1) / kTileN, 1 << 22);
        keys[b] = tiles * kOrderMaxSeqs + (kOrderMaxSeqs - 1 - b);
      }
      __syncwarp();
      for (int b = lane; b < B; b += 32) {
        const int mine = keys[b];
        int r = 0;
#pragma unroll 4
        for (int c = 0; c < B; ++c) r += keys[c] > mine ? 1 : 0;
        order[r] = b;
      }
      __syncwarp();
    }
    // position v of the hand-out order -> unit id (identity unless long_first)
    auto unit_at = [&](int v) -> int {
      if (!args.long_first) return v;
      const int per_b = args.n_heads * args.qunits;
      const int r = v / per_b;
      return order[r] * per_b + (v - r * per_b);
    };
    bool ok = true;
    for (uint32_t n = 0; ok; ++n) {
      int u;
      if (kq) {
        // claim the next valid unit: the first is blockIdx.x, later ones from the counter
        if (n >= (uint32_t)kRing) ok = mbar_wait_warp(bar(BAR_UEMPTY + n % kRing), (n / kRing - 1) & 1, abort_flag);
        if (!ok) break;
        if (lane == 0) {
          // Dynamic: every CTA starts at unit blockIdx.x and then claims units
          // gridDim.x, gridDim.x + 1, ... from the counter (fast CTAs take more).
          // Static: units blockIdx.x + i * gridDim.x.
          auto claim = [&]() -> int {
            if (args.sched != nullptr) return (int)gridDim.x + atomicAdd(&args.sched[0], 1);
            const int r = next_static;
            next_static += (int)gridDim.x;
            return r;
          };
          u = n == 0 ? (int)blockIdx.x : claim();
          while (u < total_units && !decode_unit(unit_at(u), args).valid) {
            if (args.head_idx != nullptr) {
              const int hs = (u % (args.n_heads * args.qunits)) / args.qunits;
              const int hq = args.head_idx[hs];
              if (hq < 0 || hq >= args.Hq) set_error(args.err, kDevBadSequence);
            }
            u = claim();
          }
          u = u < total_units ? unit_at(u) : -2;
          uring[n % kRing] = u;
          mbar_arrive(bar(BAR_UFULL + n % kRing));
        }
        u = __shfl_sync(0xffffffffu, u, 0);
        if (u < 0) break;
      } else {
        u = take_unit(n, true);
        if (u == -1) { ok = false; break; }
        if (u < 0) break;
      }
      const Unit t = decode_unit(u, args);
      if (kq) {
        if (q_it > 0) ok = mbar_wait_warp(bar(BAR_QEMPTY), (q_it - 1) & 1, abort_flag);
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(bar(BAR_Q), t.ntiles * kTileBytes);
          for (int i = 0; i < t.ntiles; ++i) {
            const uint32_t dst = base + kOffQ + i * kTileBytes;
            const int row = t.q_begin + t.q0 + i * kTileM;
            tma_load_3d(dst, &tmQ, bar(BAR_Q), 0, t.hq, row, pol_q);
            tma_load_3d(dst + kChunkBytes, &tmQ, bar(BAR_Q), 64, t.hq, row, pol_q);
          }
        }
        ++q_it;
      }
      for (int j = 0; j < t.nkv; ++j) {
        const KvTile kt = kv_tile(j, t.nc, t.c_begin, t.nk, t.k_begin);
        const int st = done % nst;
        if (done >= (uint32_t)nst) ok = mbar_wait_warp(bar(bempty + st), (done / nst - 1) & 1, abort_flag);
        if (!ok) break;
        const uint32_t dk = ring + st * kTileBytes;
        if (kt.seg == 0 && args.slots != nullptr) {
          // Paged cached tile: rows slots[row0 .. row0+valid) of the cache.
          // Consecutive slots (the page layout the model runner produces)
          // become one TMA copy of the cache; anything else is gathered by
          // the warp with bounds-checked 16-byte loads.
          const int32_t* sp = args.slots + kt.row0;
          const int s0 = sp[0];
          int sl[4];
          bool contig = s0 >= 0 && (int64_t)s0 + kt.valid <= args.num_slots;
#pragma unroll
          for (int r4 = 0; r4 < 4; ++r4) {
            const int r = lane + 32 * r4;
            sl[r4] = r < kt.valid ? sp[r] : -1;
            if (r < kt.valid && sl[r4] != s0 + r) contig = false;
          }
          contig = __all_sync(0xffffffffu, contig);
          if (contig) {
            if (lane == 0) {
              const CUtensorMap* mp = kq ? &tmKc : &tmVc;
              mbar_arrive_expect_tx(bar(bfull + st), kTileBytes);
              tma_load_3d(dk, mp, bar(bfull + st), 0, t.hkv, s0, pol_kv);
              tma_load_3d(dk + kChunkBytes, mp, bar(bfull + st), 64, t.hkv, s0, pol_kv);
            }
          } else {
            uint8_t* tile = smem + (dk - base);
#pragma unroll 1
            for (int r4 = 0; r4 < 4; ++r4) {
              const int r = lane + 32 * r4;
              const int64_t slot = sl[r4];
              const bool in_range = slot >= 0 && slot < args.num_slots;
              if (r < kt.valid && !in_range) set_error(args.err, kDevSlotOutOfRange);
              const uint4* src = reinterpret_cast<const uint4*>(
                  cache + (in_range ? slot : 0) * args.c_tok_stride + (int64_t)t.hkv * kD);
#pragma unroll
              for (int c16 = 0; c16 < 16; ++c16) {
                uint4 val = make_uint4(0, 0, 0, 0);
                if (r < kt.valid && in_range) val = __ldg(src + c16);
                // SW128 layout: 16-byte unit index XOR (row mod 8) inside each 64-column half
                const uint32_t off = (c16 >> 3) * kChunkBytes + r * 128 + (((c16 & 7) ^ (r & 7)) << 4);
                *reinterpret_cast<uint4*>(tile + off) = val;
              }
            }
            fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(bfull + st));
          }
        } else if (lane == 0) {
          const CUtensorMap* mp = kq ? (kt.seg == 0 ? &tmKc : &tmK) : (kt.seg == 0 ? &tmVc : &tmV);
          mbar_arrive_expect_tx(bar(bfull + st), kTileBytes);
          tma_load_3d(dk, mp, bar(bfull + st), 0, t.hkv, kt.row0, pol_kv);
          tma_load_3d(dk + kChunkBytes, mp, bar(bfull + st), 64, t.hkv, kt.row0, pol_kv);
        }
        ++done;
      }
    }
    if (lane == 0 && *abort_flag) {
      // Drain: wait (bounded) for the loads that may still be in flight.
      if (kq && q_it > 0) mbar_wait_drain(bar(BAR_Q), (q_it - 1) & 1, 100000000ull);
      for (uint32_t n = (done > (uint32_t)nst ? done - nst : 0); n < done; ++n)
        mbar_wait_drain(bar(bfull + n % nst), (n / nst) & 1, 100000000ull);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      // Shared-memory descriptors are precomputed per buffer; a K-step adds a
      // constant to the 14-bit start-address field (all offsets stay inside
      // the 256 KB shared window, so the field never carries).
      const uint32_t idesc_pv = make_idesc_bf16(128, 128, true);
      const uint32_t idesc_qk_full = make_idesc_bf16(128, 128, false);
      // Buffers of one kind are kTileBytes apart: stage n adds n * (kTileBytes >> 4).
      const uint64_t dq0 = make_sw128_desc(base + kOffQ, 16, 1024);
      const uint64_t dk0 = make_sw128_desc(base + kOffK, 16, 1024);
      const uint64_t dv0 = make_sw128_desc(base + kOffV, kChunkBytes, 1024);
      constexpr uint64_t kStageStep = kTileBytes >> 4;
      auto qk = [&](int i, int st, int n_rows) {
        const uint32_t idesc =
            n_rows == kTileN ? idesc_qk_full : make_idesc_bf16(128, (n_rows + 15) & ~15, false);
        const uint64_t a = dq0 + (uint64_t)i * kStageStep, b = dk0 + (uint64_t)st * kStageStep;
        const uint32_t d = tmem + i * 128;
#pragma unroll
        for (int s = 0; s < kD / 16; ++s) {
          const uint64_t off = (uint64_t)(((s >> 2) * kChunkBytes + (s & 3) * 32) >> 4);
          umma_ss(d, a + off, b + off, idesc, s > 0 ? 1u : 0u);
        }
      };
      auto pv = [&](int i, int st, int n_rows, bool acc) {
        const uint64_t b = dv0 + (uint64_t)st * kStageStep;
        const uint32_t d = tmem + 256 + i * 128;
        const uint32_t a = tmem + i * 128;
        if (n_rows == kTileN) {
#pragma unroll
          for (int s = 0; s < 8; ++s)
            umma_ts(d, a + s * 8, b + (uint64_t)(s * (2048 >> 4)), idesc_pv, (acc || s > 0) ? 1u : 0u);
        } else {
          const int ksteps = (n_rows + 15) >> 4;
          for (int s = 0; s < ksteps; ++s)
            umma_ts(d, a + s * 8, b + (uint64_t)(s * (2048 >> 4)), idesc_pv, (acc || s > 0) ? 1u : 0u);
        }
      };
      uint32_t q_it = 0, kv_it = 0;
      uint32_t p_it[2] = {0, 0};
      bool ok = true;
      for (uint32_t n = 0; ok; ++n) {
        const int u = take_unit(n, false);
        if (u == -1) { ok = false; break; }
        if (u < 0) break;
        const Unit t = decode_unit(u, args);
        ok = mbar_wait(bar(BAR_Q), q_it & 1, abort_flag);
        if (!ok) break;
        ++q_it;
        if (t.nkv == 0) {
          umma_commit(bar(BAR_QEMPTY));
          continue;
        }
        {
          const int st0 = kv_it % kStagesK;
          ok = mbar_wait(bar(BAR_KFULL + st0), (kv_it / kStagesK) & 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const KvTile t0 = kv_tile(0, t.nc, t.c_begin, t.nk, t.k_begin);
          for (int i = 0; i < t.ntiles; ++i) {
            qk(i, st0, t0.valid);
            umma_commit(bar(BAR_SFULL + i));
          }
          umma_commit(bar(BAR_KEMPTY + st0));
          if (t.nkv == 1) umma_commit(bar(BAR_QEMPTY));
        }
        for (int j = 0; j < t.nkv && ok; ++j) {
          const uint32_t kvj = kv_it + j;
          const int vst = kvj % kStagesV;
          const KvTile kt = kv_tile(j, t.nc, t.c_begin, t.nk, t.k_begin);
          ok = mbar_wait(bar(BAR_VFULL + vst), (kvj / kStagesV) & 1, abort_flag);
          if (!ok) break;
          const bool more = j + 1 < t.nkv;
          const int kst = (kvj + 1) % kStagesK;
          const KvTile tn = more ? kv_tile(j + 1, t.nc, t.c_begin, t.nk, t.k_begin) : kt;
          bool k_ready = !more;
          for (int i = 0; i < t.ntiles; ++i) {
            ok = mbar_wait(bar(BAR_PFULL + i), p_it[i] & 1, abort_flag);
            if (!ok) break;
            ++p_it[i];
            tc_fence_after();
            pv(i, vst, kt.valid, j > 0);
            if (more) {
              if (!k_ready) {
                ok = mbar_wait(bar(BAR_KFULL + kst), ((kvj + 1) / kStagesK) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                k_ready = true;
              }
              qk(i, kst, tn.valid);
              umma_commit(bar(BAR_SFULL + i));
            } else {
              umma_commit(bar(BAR_OFULL + i));
            }
          }
          if (!ok) break;
          umma_commit(bar(BAR_VEMPTY + vst));
          if (more) umma_commit(bar(BAR_KEMPTY + kst));
          if (more && j + 2 == t.nkv) umma_commit(bar(BAR_QEMPTY));  // last QK issued
        }
        kv_it += t.nkv;
      }
      // Make sure every issued MMA has finished before TMEM is released.
      umma_commit(bar(BAR_DRAIN));
      mbar_wait_drain(bar(BAR_DRAIN), 0, 100000000ull);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax
    const int wg = warp >> 2;           // 0 or 1: query tile
    const int wq = warp & 3;            // warp within the warpgroup
    const int row_in_tile = threadIdx.x & 127;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + wg * 128;
    const uint32_t tO = tmem + lane_base + 256 + wg * 128;
    const float sl2 = args.scale_log2;
    uint32_t s_it = 0, o_it = 0;
    bool ok = true;
    for (uint32_t n = 0; ok; ++n) {
      const int u = take_unit(n, true);
      if (u == -1) { ok = false; break; }
      if (u < 0) break;
      const Unit t = decode_unit(u, args);
      if (wg >= t.ntiles) continue;
      float m = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < t.nkv; ++j) {
        const KvTile kt = kv_tile(j, t.nc, t.c_begin, t.nk, t.k_begin);
        ok = mbar_wait_warp(bar(BAR_SFULL + wg), s_it & 1, abort_flag);
        if (!ok) break;
        ++s_it;
        tc_fence_after();
        uint32_t s[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, s[c]);
        tmem_wait_ld();
        const bool partial = kt.valid < kTileN;
        if (partial) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e >= kt.valid) s[c][e] = __float_as_uint(-INFINITY);
        }
        // row max: four independent 3-input max chains
        float mq[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float a = __uint_as_float(s[c][0]);
#pragma unroll
          for (int e = 1; e < 31; e += 2)
            a = max3f(a, __uint_as_float(s[c][e]), __uint_as_float(s[c][e + 1]));
          mq[c] = fmaxf(a, __uint_as_float(s[c][31]));
        }
        const float mxs = max3f(mq[0], mq[1], fmaxf(mq[2], mq[3])) * sl2;
        bool rescale = false;
        float alpha = 1.f;
        if (j == 0) {
          m = mxs;
        } else {
          // Lazy rescaling: keep a stale maximum while the new one exceeds it
          // by at most 8 (log2 units), so P stays <= 256 and O/l stay exact
          // up to rounding; rescale O only when a warp needs it.
          const bool need = mxs > m + 8.f;
          if (__any_sync(0xffffffffu, need)) {
            const float mn = fmaxf(m, mxs);
            alpha = ex2_approx(m - mn);
            m = mn;
            l *= alpha;
            rescale = true;
          }
        }
        l += exp_store_tile(s, sl2, m, tS);  // masked columns give exact zeros
        if (rescale) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(BAR_PFULL + wg));
      }
      if (!ok) break;
      // Epilogue: O / l -> bf16 -> global.
      const int row = t.q0 + wg * kTileM + row_in_tile;
      const bool row_ok = row < t.Lq;
      __nv_bfloat16* orow = args.o + (int64_t)(t.q_begin + row) * args.o_tok_stride +
                            (int64_t)t.hq * args.o_head_stride;
      if (t.nkv > 0) {
        ok = mbar_wait_warp(bar(BAR_OFULL + wg), o_it & 1, abort_flag);
        if (!ok) break;
        ++o_it;
        tc_fence_after();
        const float inv_l = 1.f / l;
        // Rows are spread one per lane; a 4x4 transpose of 16-byte vectors
        // inside each lane quad lets every store instruction write 8 rows x 64
        // contiguous bytes (full sectors) instead of 32 rows x 16 bytes.
        const int qj = lane & 3;
        const int qrow0 = row - qj;  // first row of this lane's quad
        // TMEM loads run one chunk ahead of the conversion and stores.
        uint32_t onext[32];
        tmem_ld32(tO, onext);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = onext[e];
          if (c < 3) tmem_ld32(tO + (c + 1) * 32, onext);
          uint4 v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            v[e].x = pack_bf16x2(__uint_as_float(o[8 * e + 0]) * inv_l, __uint_as_float(o[8 * e + 1]) * inv_l);
            v[e].y = pack_bf16x2(__uint_as_float(o[8 * e + 2]) * inv_l, __uint_as_float(o[8 * e + 3]) * inv_l);
            v[e].z = pack_bf16x2(__uint_as_float(o[8 * e + 4]) * inv_l, __uint_as_float(o[8 * e + 5]) * inv_l);
            v[e].w = pack_bf16x2(__uint_as_float(o[8 * e + 6]) * inv_l, __uint_as_float(o[8 * e + 7]) * inv_l);
          }
          quad_transpose16(v, qj);  // v[r] = vector qj of the quad's row r
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            if (qrow0 + r < t.Lq) {
              uint4* dst = reinterpret_cast<uint4*>(orow + (int64_t)(r - qj) * args.o_tok_stride + c * 32);
              dst[qj] = v[r];
            }
          }
        }
        // O_i is read out; the next unit's first PV may overwrite it once this
        // warpgroup arrives on its first P barrier (program order + fence).
        tc_fence_before();
      } else if (row_ok) {
        // No keys at all: the output row is zero.
        uint4* dst = reinterpret_cast<uint4*>(orow);
        for (int v = 0; v < kD / 8; ++v) dst[v] = make_uint4(0, 0, 0, 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) set_error(args.err, kDevWaitTimeout);
  if (threadIdx.x == 0 && args.sched != nullptr) {
    // The last CTA to finish (every CTA has stopped claiming) returns the
    // workspace to zero for the next launch on the stream.
    __threadfence();
    if (atomicAdd(&args.sched[1], 1) == (int)gridDim.x - 1) {
      atomicExch(&args.sched[0], 0);
      atomicExch(&args.sched[1], 0);
    }
  }
}

uint32_t attn_fwd_smem_bytes() { return kSmemBytes; }
int attn_fwd_kv_rows_per_tile() { return kTileN; }

cudaError_t launch_attn_fwd(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                            const CUtensorMap& tmKc, const CUtensorMap& tmVc,
                            const AttnKernelArgs& args, int max_q, int num_sms,
                            cudaStream_t stream) {
  // The smem opt-in is per device; remember it for up to 64 devices.
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  AttnKernelArgs a = args;
  a.qunits = (max_q + 2 * kTileM - 1) / (2 * kTileM);
  if (a.head_idx == nullptr) a.n_heads = a.Hq;
  const long long units = (long long)a.B * a.n_heads * a.qunits;
  if (units == 0) return cudaSuccess;
  if (units > 0x7fffffffLL) return cudaErrorInvalidValue;
  a.total_units = (int)units;
  a.long_first = a.B <= kOrderMaxSeqs && units <= (long long)kLongFirstUnitsPerSm * num_sms ? 1 : 0;
  const int grid = (int)(units < num_sms ? units : num_sms);
  // Programmatic dependent launch: this grid may start while the previous
  // kernel in the stream finishes; it waits for it in griddep_wait().
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_fwd_kernel, tmQ, tmK, tmV, tmKc, tmVc, a);
}

}  // namespace dllm
