// Non-causal varlen flash-attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the `flash_attn_varlen_func(..., causal=False)` call of the
// reference's diffusion attention (dllmserve/layers/attention.py:289-299),
// including the cached-K/V ("reuse") sequences whose keys are the selected
// cached rows followed by the block's fresh rows (attention.py:235-265).
//
// Work unit: one CTA = (sequence b, query head h, pair of 128-row query tiles).
// Roles inside the CTA (10 warps):
//   warps 0-3  softmax warpgroup 0  (query tile 0, TMEM lanes 0-127)
//   warps 4-7  softmax warpgroup 1  (query tile 1)
//   warp  8    TMA producer          (Q once, K/V ring of kStages)
//   warp  9    MMA issuer            (also allocates / frees TMEM)
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
#include "common.cuh"
#include "attn_fwd.h"

namespace dllm {

namespace {

constexpr int kD = 128;          // head dim (only 128 is instantiated)
constexpr int kTileM = 128;      // query rows per tile
constexpr int kTileN = 128;      // kv rows per tile
constexpr int kStages = 2;       // K and V ring depth
constexpr int kThreads = 320;
constexpr uint32_t kTileBytes = kTileM * kD * 2;  // 32 KB (bf16)
constexpr uint32_t kChunkBytes = 128 * 128;       // 128 rows x 128 B (64 bf16)

// Shared-memory map (offsets from a 1024-aligned base).
constexpr uint32_t kOffQ = 0;                                   // 2 tiles
constexpr uint32_t kOffK = kOffQ + 2 * kTileBytes;              // kStages tiles
constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;        // kStages tiles
constexpr uint32_t kOffBar = kOffV + kStages * kTileBytes;      // barriers
constexpr uint32_t kNumBars = 1 + 4 * kStages + 2 + 2 + 2 + 1;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 64 + 1024;          // + alignment slack

// barrier indices
constexpr int BAR_Q = 0;
constexpr int BAR_KFULL = 1;
constexpr int BAR_KEMPTY = BAR_KFULL + kStages;
constexpr int BAR_VFULL = BAR_KEMPTY + kStages;
constexpr int BAR_VEMPTY = BAR_VFULL + kStages;
constexpr int BAR_SFULL = BAR_VEMPTY + kStages;  // 2
constexpr int BAR_PFULL = BAR_SFULL + 2;         // 2
constexpr int BAR_OFULL = BAR_PFULL + 2;         // 2
constexpr int BAR_DRAIN = BAR_OFULL + 2;         // 1

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

}  // namespace

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

  const int b = blockIdx.z;
  const int hq = blockIdx.y;
  const int hkv = hq / args.group;

  const int q_begin = args.cu_q[b];
  const int Lq = args.cu_q[b + 1] - q_begin;
  const int q0 = blockIdx.x * (2 * kTileM);
  if (q0 >= Lq) return;  // uniform for the CTA
  const int ntiles = (Lq - q0 > kTileM) ? 2 : 1;

  const int k_begin = args.cu_k[b];
  const int nk = args.cu_k[b + 1] - k_begin;
  int c_begin = 0, nc = 0;
  if (args.cu_c != nullptr) {
    c_begin = args.cu_c[b];
    nc = args.cu_c[b + 1] - c_begin;
  }
  const int nkv = (nc + kTileN - 1) / kTileN + (nk + kTileN - 1) / kTileN;

  const uint32_t bar0 = base + kOffBar;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc + 16);

  if (threadIdx.x == 0) {
    mbar_init(bar(BAR_Q), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(BAR_KFULL + s), 1);
      mbar_init(bar(BAR_KEMPTY + s), 1);
      mbar_init(bar(BAR_VFULL + s), 1);
      mbar_init(bar(BAR_VEMPTY + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(BAR_SFULL + i), 1);
      mbar_init(bar(BAR_PFULL + i), 128);
      mbar_init(bar(BAR_OFULL + i), 1);
    }
    mbar_init(bar(BAR_DRAIN), 1);
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
    if (nc > 0) {
      tma_prefetch_desc(&tmKc);
      tma_prefetch_desc(&tmVc);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();
      // Q: both tiles, two 64-column chunks each.
      mbar_arrive_expect_tx(bar(BAR_Q), ntiles * kTileBytes);
      for (int i = 0; i < ntiles; ++i) {
        const uint32_t dst = base + kOffQ + i * kTileBytes;
        const int row = q_begin + q0 + i * kTileM;
        tma_load_3d(dst, &tmQ, bar(BAR_Q), 0, hq, row, pol_q);
        tma_load_3d(dst + kChunkBytes, &tmQ, bar(BAR_Q), 64, hq, row, pol_q);
      }
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j % kStages;
        const uint32_t use = (uint32_t)(j / kStages);
        const KvTile t = kv_tile(j, nc, c_begin, nk, k_begin);
        const CUtensorMap* mk = t.seg == 0 ? &tmKc : &tmK;
        const CUtensorMap* mv = t.seg == 0 ? &tmVc : &tmV;
        if (j >= kStages) ok = mbar_wait(bar(BAR_KEMPTY + st), (use - 1) & 1, abort_flag);
        if (!ok) break;
        uint32_t dk = base + kOffK + st * kTileBytes;
        mbar_arrive_expect_tx(bar(BAR_KFULL + st), kTileBytes);
        tma_load_3d(dk, mk, bar(BAR_KFULL + st), 0, hkv, t.row0, pol_kv);
        tma_load_3d(dk + kChunkBytes, mk, bar(BAR_KFULL + st), 64, hkv, t.row0, pol_kv);
        if (j >= kStages) ok = mbar_wait(bar(BAR_VEMPTY + st), (use - 1) & 1, abort_flag);
        if (!ok) {
          issued = j + 1;  // K of tile j is in flight
          break;
        }
        uint32_t dv = base + kOffV + st * kTileBytes;
        mbar_arrive_expect_tx(bar(BAR_VFULL + st), kTileBytes);
        tma_load_3d(dv, mv, bar(BAR_VFULL + st), 0, hkv, t.row0, pol_kv);
        tma_load_3d(dv + kChunkBytes, mv, bar(BAR_VFULL + st), 64, hkv, t.row0, pol_kv);
        issued = j + 1;
      }
      if (*abort_flag) {
        // Drain: wait (bounded) for the loads that may still be in flight.
        mbar_wait_drain(bar(BAR_Q), 0, 100000000ull);
        for (int j = max(0, issued - kStages); j < issued; ++j) {
          const int st = j % kStages;
          const uint32_t use = (uint32_t)(j / kStages);
          mbar_wait_drain(bar(BAR_KFULL + st), use & 1, 100000000ull);
          mbar_wait_drain(bar(BAR_VFULL + st), use & 1, 100000000ull);
        }
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc_pv = make_idesc_bf16(128, 128, true);
      auto qk = [&](int i, int st, int n_rows) {
        const uint32_t qa = base + kOffQ + i * kTileBytes;
        const uint32_t ka = base + kOffK + st * kTileBytes;
        const int n = (n_rows + 15) & ~15;
        const uint32_t idesc = make_idesc_bf16(128, n, false);
#pragma unroll
        for (int s = 0; s < kD / 16; ++s) {
          const uint32_t off = (s >> 2) * kChunkBytes + (s & 3) * 32;
          umma_ss(tmem + i * 128, make_sw128_desc(qa + off, 16, 1024),
                  make_sw128_desc(ka + off, 16, 1024), idesc, s > 0 ? 1u : 0u);
        }
      };
      auto pv = [&](int i, int st, int n_rows, bool acc) {
        const uint32_t va = base + kOffV + st * kTileBytes;
        const int ksteps = (n_rows + 15) >> 4;
        for (int s = 0; s < ksteps; ++s) {
          umma_ts(tmem + 256 + i * 128, tmem + i * 128 + s * 8,
                  make_sw128_desc(va + s * 2048, kChunkBytes, 1024), idesc_pv,
                  (acc || s > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(bar(BAR_Q), 0, abort_flag);
      if (ok && nkv > 0) ok = mbar_wait(bar(BAR_KFULL + 0), 0, abort_flag);
      if (ok && nkv > 0) {
        tc_fence_after();
        const KvTile t0 = kv_tile(0, nc, c_begin, nk, k_begin);
        for (int i = 0; i < ntiles; ++i) {
          qk(i, 0, t0.valid);
          umma_commit(bar(BAR_SFULL + i));
        }
        umma_commit(bar(BAR_KEMPTY + 0));
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int vst = j % kStages;
        const KvTile t = kv_tile(j, nc, c_begin, nk, k_begin);
        ok = mbar_wait(bar(BAR_VFULL + vst), (uint32_t)(j / kStages) & 1, abort_flag);
        if (!ok) break;
        const bool more = j + 1 < nkv;
        const int kst = (j + 1) % kStages;
        KvTile tn = t;
        if (more) {
          tn = kv_tile(j + 1, nc, c_begin, nk, k_begin);
          ok = mbar_wait(bar(BAR_KFULL + kst), (uint32_t)((j + 1) / kStages) & 1, abort_flag);
          if (!ok) break;
        }
        for (int i = 0; i < ntiles; ++i) {
          ok = mbar_wait(bar(BAR_PFULL + i), (uint32_t)j & 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          pv(i, vst, t.valid, j > 0);
          if (more) {
            qk(i, kst, tn.valid);
            umma_commit(bar(BAR_SFULL + i));
          } else {
            umma_commit(bar(BAR_OFULL + i));
          }
        }
        if (!ok) break;
        umma_commit(bar(BAR_VEMPTY + vst));
        if (more) umma_commit(bar(BAR_KEMPTY + kst));
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
    if (wg < ntiles) {
      const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
      const uint32_t tS = tmem + lane_base + wg * 128;
      const uint32_t tO = tmem + lane_base + 256 + wg * 128;
      const float sl2 = args.scale_log2;
      float m = -INFINITY;
      float l = 0.f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        const KvTile t = kv_tile(j, nc, c_begin, nk, k_begin);
        ok = mbar_wait(bar(BAR_SFULL + wg), (uint32_t)j & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t s[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, s[c]);
        tmem_wait_ld();
        const bool partial = t.valid < kTileN;
        if (partial) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e >= t.valid) s[c][e] = __float_as_uint(-INFINITY);
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
        const float mx = max3f(mq[0], mq[1], fmaxf(mq[2], mq[3]));
        const float mxs = mx * sl2;
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
        const float neg_m = -m;
        float rsa[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1, p0, p1;
            fma2(x0, x1, __uint_as_float(s[c][2 * e]), __uint_as_float(s[c][2 * e + 1]), sl2, sl2,
                 neg_m, neg_m);
            // 3 of every 8 pairs on the FMA pipe, the rest on MUFU; masked
            // (partial) tiles stay on MUFU so masked columns are exactly 0.
            if (!partial && (e & 7) < 3) {
              exp2_poly2(x0, x1, p0, p1);
            } else {
              p0 = ex2_approx(x0);
              p1 = ex2_approx(x1);
            }
            add2(rsa[(e & 1) * 2], rsa[(e & 1) * 2 + 1], rsa[(e & 1) * 2], rsa[(e & 1) * 2 + 1], p0, p1);
            pk[e] = pack_bf16x2(p0, p1);
          }
          tmem_st16(tS + c * 16, pk);
        }
        const float rs = (rsa[0] + rsa[1]) + (rsa[2] + rsa[3]);
        l += rs;
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
        mbar_arrive(bar(BAR_PFULL + wg));
      }
      // Epilogue: O / l -> bf16 -> global.
      const int row = q0 + wg * kTileM + row_in_tile;
      const bool row_ok = row < Lq;
      __nv_bfloat16* orow = args.o + (int64_t)(q_begin + row) * args.o_tok_stride +
                            (int64_t)hq * args.o_head_stride;
      if (ok && nkv > 0) ok = mbar_wait(bar(BAR_OFULL + wg), 0, abort_flag);
      if (ok && nkv > 0) {
        tc_fence_after();
        const float inv_l = 1.f / l;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv_l, __uint_as_float(o[8 * v + 1]) * inv_l);
              w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv_l, __uint_as_float(o[8 * v + 3]) * inv_l);
              w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv_l, __uint_as_float(o[8 * v + 5]) * inv_l);
              w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv_l, __uint_as_float(o[8 * v + 7]) * inv_l);
              dst[v] = w;
            }
          }
        }
      } else if (ok && nkv == 0 && row_ok) {
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
}

uint32_t attn_fwd_smem_bytes() { return kSmemBytes; }

cudaError_t launch_attn_fwd(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                            const CUtensorMap& tmKc, const CUtensorMap& tmVc,
                            const AttnKernelArgs& args, int max_q, cudaStream_t stream) {
  // The smem opt-in is per device; remember it for up to 64 devices.
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  dim3 grid((max_q + 2 * kTileM - 1) / (2 * kTileM), args.Hq, args.B);
  if (grid.x == 0 || args.B == 0) return cudaSuccess;
  attn_fwd_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmKc, tmVc, args);
  return cudaGetLastError();
}

}  // namespace dllm
