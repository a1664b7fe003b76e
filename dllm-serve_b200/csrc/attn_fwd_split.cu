// Non-causal varlen flash-attention forward for sm_100a (tcgen05 + TMEM + TMA),
// "split" variant for launches whose query segments fit one 128-row tile
// (max_seqlen_q <= 128: the reuse steps' fresh blocks). The "pair" kernel in
// attn_fwd.cu gives each unit two query tiles; here a unit has one, and the
// two softmax warpgroups split every KV tile's columns instead, so neither
// sits idle on a lone tile.
//
// Replaces the `flash_attn_varlen_func(..., causal=False)` call of the
// reference's diffusion attention (dllmserve/layers/attention.py:289-299),
// including the cached-K/V ("reuse") sequences whose keys are the selected
// cached rows followed by the block's fresh rows (attention.py:235-265).
//
// Persistent kernel: one CTA per SM loops over work units = (sequence b,
// query head h, 128-row query tile), or, for GQA with short query segments,
// (sequence b, KV head, up to 128/Lq query heads of its group packed in one tile). Roles inside the CTA (11 warps):
//   warps 0-3  softmax warpgroup 0: kv rows 0-63 of every KV tile
//   warps 4-7  softmax warpgroup 1: kv rows 64-127 of every KV tile
//   warp  8    TMA producer: Q tiles (2-deep ring) and the K ring
//   warp  9    MMA issuer (also allocates / frees TMEM)
//   warp  10   TMA producer: the V ring
//   warp  11   (rotary launches only) rotates each Q tile and each fresh K
//              tile in shared memory between its TMA arrival and its MMA
// Both warpgroups own all 128 query rows (TMEM lanes) and split each KV
// tile's 128 columns; each keeps its own running max / sum and its own
// output accumulator, and the two partial results are merged once per unit.
// TMEM (512 columns): S buffers SB0 [0,128) and SB1 [128,256) (KV tile j
// uses SB(j mod 2)), O_a [256,384) (kv rows 0-63 of every tile), O_b
// [384,512) (kv rows 64-127). Warpgroup w writes its bf16 P half over the
// first 32 columns of its own S half (SB + 64w). MMA issue order per tile j:
//   PV_a(j), PV_b(j), QK(j+2) -> SB(j mod 2)
// so QK(j+1) has filled the other S buffer while the softmax works on tile
// j, and QK(j+2) overwrites P(j) only after the PVs that read it (tcgen05
// MMAs of one thread execute in order).
//
// Each KV sequence is the concatenation of up to two segments:
//   segment 0: cached rows (k_cache/v_cache gathered rows, `cu_c`), optional
//   segment 1: fresh rows of the step's k/v (`cu_k`)
// KV tiles never straddle segments; a partial tile uses a smaller MMA N.
#include <atomic>

#include "common.cuh"
#include "attn_fwd.h"

namespace dllm {
namespace split {

namespace {

constexpr int kD = 128;          // head dim (only 128 is instantiated)
constexpr int kTileM = 128;      // query rows per unit
constexpr int kTileN = 128;      // kv rows per tile
constexpr int kHalfN = 64;       // kv rows per softmax warpgroup
constexpr int kStagesQ = 2;      // Q ring depth (the next unit's Q loads early)
constexpr int kStagesK = 3;      // K ring depth (QK runs two tiles ahead of PV)
constexpr int kStagesV = 2;      // V ring depth
constexpr int kThreads = 352;
constexpr int kThreadsRope = 384;  // + the rotary warp

constexpr uint32_t kTileBytes = kTileM * kD * 2;  // 32 KB (bf16)
constexpr uint32_t kChunkBytes = 128 * 128;       // 128 rows x 128 B (64 bf16)

// Shared-memory map (offsets from a 1024-aligned base).
constexpr uint32_t kOffQ = 0;                                   // kStagesQ tiles
constexpr uint32_t kOffK = kOffQ + kStagesQ * kTileBytes;       // kStagesK tiles
constexpr uint32_t kOffV = kOffK + kStagesK * kTileBytes;       // kStagesV tiles
constexpr uint32_t kOffBar = kOffV + kStagesV * kTileBytes;     // barriers

// barrier indices
constexpr int BAR_QFULL = 0;
constexpr int BAR_QEMPTY = BAR_QFULL + kStagesQ;
constexpr int BAR_KFULL = BAR_QEMPTY + kStagesQ;
constexpr int BAR_KEMPTY = BAR_KFULL + kStagesK;
constexpr int BAR_VFULL = BAR_KEMPTY + kStagesK;
constexpr int BAR_VEMPTY = BAR_VFULL + kStagesV;
constexpr int BAR_SFULL = BAR_VEMPTY + kStagesV;  // 2: S buffer holds QK of a tile
constexpr int BAR_PFULL = BAR_SFULL + 2;          // 2: both P halves of a buffer written
constexpr int BAR_OREADY = BAR_PFULL + 2;         // 1: PVs of one more tile completed
constexpr int BAR_OFULL = BAR_OREADY + 1;         // 1: a unit's last PVs completed
constexpr int BAR_XML = BAR_OFULL + 1;            // 1: warpgroup 1's (max, sum) published
constexpr int BAR_XF = BAR_XML + 1;               // 1: the merge factors published
constexpr int BAR_DRAIN = BAR_XF + 1;             // 1
constexpr int BAR_QROPED = BAR_DRAIN + 1;         // kStagesQ: Q tile rotated (rotary launches)
constexpr int BAR_KROPED = BAR_QROPED + kStagesQ; // kStagesK: fresh K tile rotated
constexpr int BAR_KFRESH = BAR_KROPED + kStagesK; // kStagesK: fresh K tile landed (rotary launches)
constexpr uint32_t kNumBars = BAR_KFRESH + kStagesK;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;           // abort flag, TMEM address
constexpr uint32_t kOffXch = kOffMisc + 64;                     // float2 per query row
constexpr uint32_t kSmemBytes = kOffXch + kTileM * 8 + 1024;    // + alignment slack
static_assert(kSmemBytes <= 232448, "over the sm_100a per-CTA shared-memory limit");

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

// P = 2^(S*scale_log2 - m) for one row of a 64-column half tile (two chunks
// of 32 columns, MUFU ex2), packed to bf16 pairs and stored to TMEM at tP
// (chunk c -> columns 16c .. 16c+15); returns the row sum of P (fp32).
DLLM_DEVICE float exp_store_half(const uint32_t (&s)[2][32], float sl2, float m, uint32_t tP) {
  const float neg_m = -m;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float p0 = ex2_approx(fmaf(__uint_as_float(s[c][2 * e]), sl2, neg_m));
      const float p1 = ex2_approx(fmaf(__uint_as_float(s[c][2 * e + 1]), sl2, neg_m));
      acc[(2 * e) & 3] += p0;
      acc[(2 * e + 1) & 3] += p1;
      pk[e] = pack_bf16x2(p0, p1);
    }
    tmem_st16(tP + c * 16, pk);
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

}  // namespace

// One work unit: (sequence b, query head hq, 128-row query tile).
struct Unit {
  bool valid;
  int hq, hkv;     // first query head of the tile, its KV head
  int nheads;      // query heads packed in the tile (args.qpack mode), else 1
  int q_begin, Lq, q0;
  int k_begin, nk, c_begin, nc, nkv;
};

// Units are numbered ((b * Hq) + hq) * qunits + t, so consecutive units share
// a sequence and head (their K/V stay hot in L2 while several CTAs read them).
// With args.qpack = m > 1 (GQA, every query segment <= 128/m rows) a tile
// holds the rows of m query heads of one KV group: units ((b * Hkv) + hk) *
// qunits + c cover heads hk*group + c*m .. + m-1 (qunits = ceil(group / m)).
DLLM_DEVICE Unit decode_unit(int u, const AttnKernelArgs& a) {
  Unit r;
  int b, t;
  bool head_ok = true;
  if (a.qpack > 1) {
    const int per_b = a.Hkv * a.qunits;
    b = u / per_b;
    const int rem = u - b * per_b;
    r.hkv = rem / a.qunits;
    const int c = rem - r.hkv * a.qunits;
    r.hq = r.hkv * a.group + c * a.qpack;
    r.nheads = min(a.qpack, a.group - c * a.qpack);
    t = 0;
  } else {
    const int per_b = a.n_heads * a.qunits;
    b = u / per_b;
    const int rem = u - b * per_b;
    const int hsel = rem / a.qunits;
    t = rem - hsel * a.qunits;
    r.hq = a.head_idx != nullptr ? a.head_idx[hsel] : hsel;
    head_ok = r.hq >= 0 && r.hq < a.Hq;
    if (!head_ok) {
      set_error(a.err, kDevBadSequence);
      r.hq = 0;
    }
    r.hkv = r.hq / a.group;
    r.nheads = 1;
  }
  r.q_begin = a.cu_q[b];
  r.Lq = a.cu_q[b + 1] - r.q_begin;
  r.q0 = t * kTileM;
  r.valid = head_ok && r.q0 < r.Lq;
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

// Rotates, in place in shared memory, the rows of one SW128 tile (two 64-column
// halves kChunkBytes apart, 128-byte lines, 16-byte unit u of line r stored at
// unit u ^ (r mod 8)): line rr * qpack + hh holds head hh of token tok0 + rr
// (rr < rows, hh < nheads <= 4; other lines are left alone). Dimension pair
// (d, d + 64) sits at the same offset of the two halves. One warp: lane l
// covers unit (l mod 8) of rows l/8 + 4i; the positions, then the cos/sin rows
// of 16 rows are loaded at once (one round trip each) and applied to every
// head of the row.
DLLM_DEVICE void rope_tile_smem(uint8_t* tile, int lane, const AttnKernelArgs& a, int64_t tok0,
                                int rows, int qpack, int nheads) {
  const int c = lane & 7;
  for (int rb = lane >> 3; rb < rows; rb += 16) {
    int64_t pos[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = rb + 4 * i;
      pos[i] = r < rows ? __ldg(a.positions + tok0 + r) : 0;
    }
    float4 cv[4][2], sv[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = rb + 4 * i;
      const bool in_range = pos[i] >= 0 && pos[i] < a.max_position;
      if (r < rows && !in_range) set_error(a.err, kDevPositionOutOfRange);
      if (r < rows && in_range) {
        const float4* row = reinterpret_cast<const float4*>(a.cos_sin + pos[i] * kD);
        cv[i][0] = __ldg(row + 2 * c);
        cv[i][1] = __ldg(row + 2 * c + 1);
        sv[i][0] = __ldg(row + 16 + 2 * c);
        sv[i][1] = __ldg(row + 16 + 2 * c + 1);
      } else {  // out of range: the row becomes zero
        cv[i][0] = cv[i][1] = sv[i][0] = sv[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = rb + 4 * i;
      if (r >= rows) continue;
      // Scalar fp32 products and sums: the packed f32x2 forms of the same
      // operations were measured to differ from them in the last bf16 bit of
      // a few outputs, so they are not used here.
      const float cs[8] = {cv[i][0].x, cv[i][0].y, cv[i][0].z, cv[i][0].w,
                           cv[i][1].x, cv[i][1].y, cv[i][1].z, cv[i][1].w};
      const float sn[8] = {sv[i][0].x, sv[i][0].y, sv[i][0].z, sv[i][0].w,
                           sv[i][1].x, sv[i][1].y, sv[i][1].z, sv[i][1].w};
      uint4 w[4][2];
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        if (hh < nheads) {
          const int line = r * qpack + hh;
          const uint32_t off = line * 128 + ((c ^ (line & 7)) << 4);
          w[hh][0] = *reinterpret_cast<const uint4*>(tile + off);
          w[hh][1] = *reinterpret_cast<const uint4*>(tile + kChunkBytes + off);
        }
      }
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        if (hh < nheads) {
          const int line = r * qpack + hh;
          const uint32_t off = line * 128 + ((c ^ (line & 7)) << 4);
          rope_rotate8(w[hh][0], w[hh][1], cs, sn);
          *reinterpret_cast<uint4*>(tile + off) = w[hh][0];
          *reinterpret_cast<uint4*>(tile + kChunkBytes + off) = w[hh][1];
        }
      }
    }
  }
}

// Persistent kernel: CTA c processes units c, c + gridDim.x, ... Barrier
// phases run on across units (ring counters below), so the producers load the
// next unit's Q/K/V and the MMA warp starts its QKs while the softmax warps
// still write the previous unit's output.
template <bool kRope>
__global__ void __launch_bounds__(kRope ? kThreadsRope : kThreads, 1)
    attn_fwd_split_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
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
    for (int s = 0; s < kStagesQ; ++s) {
      mbar_init(bar(BAR_QFULL + s), 1);
      mbar_init(bar(BAR_QEMPTY + s), 1);
    }
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
      mbar_init(bar(BAR_PFULL + i), 8);  // one arrival per softmax warp
    }
    mbar_init(bar(BAR_OREADY), 1);
    mbar_init(bar(BAR_OFULL), 1);
    mbar_init(bar(BAR_XML), 128);  // every thread of warpgroup 1
    mbar_init(bar(BAR_XF), 128);   // every thread of warpgroup 0
    mbar_init(bar(BAR_DRAIN), 1);
    for (int s = 0; s < kStagesQ; ++s) mbar_init(bar(BAR_QROPED + s), 1);
    for (int s = 0; s < kStagesK; ++s) {
      mbar_init(bar(BAR_KROPED + s), 1);
      mbar_init(bar(BAR_KFRESH + s), 1);
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

  if (warp == 8 || warp == 10) {
    // ------------------------------------------------------------------ TMA
    // warp 8: Q tiles (2-deep ring) and the K ring; warp 10: the V ring (independent rings, so a wait
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
    // Rotary launches, K ring: a fresh tile completes on its stage's KFRESH
    // barrier instead of KFULL; per-stage phase parities of both barriers and
    // which of them each stage's latest load used (for the drain).
    uint32_t kfull_par = 0, kfresh_par = 0, last_fresh = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      const Unit t = decode_unit(u, args);
      if (!t.valid) continue;
      if (kq) {
        const int qs = q_it % kStagesQ;
        if (q_it >= (uint32_t)kStagesQ)
          ok = mbar_wait_warp(bar(BAR_QEMPTY + qs), (q_it / kStagesQ - 1) & 1, abort_flag);
        if (!ok) break;
        if (lane == 0) {
          const uint32_t dst = base + kOffQ + qs * kTileBytes;
          const int row = t.q_begin + t.q0;
          mbar_arrive_expect_tx(bar(BAR_QFULL + qs), kTileBytes);
          tma_load_3d(dst, &tmQ, bar(BAR_QFULL + qs), 0, t.hq, row, pol_q);
          tma_load_3d(dst + kChunkBytes, &tmQ, bar(BAR_QFULL + qs), 64, t.hq, row, pol_q);
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
          const uint32_t fb = bar(((kRope && kq && kt.seg == 1) ? BAR_KFRESH : bfull) + st);
          mbar_arrive_expect_tx(fb, kTileBytes);
          tma_load_3d(dk, mp, fb, 0, t.hkv, kt.row0, pol_kv);
          tma_load_3d(dk + kChunkBytes, mp, fb, 64, t.hkv, kt.row0, pol_kv);
        }
        if (kRope && kq) {
          const uint32_t bit = 1u << st;
          if (kt.seg == 1) {
            kfresh_par ^= bit;
            last_fresh |= bit;
          } else {
            kfull_par ^= bit;
            last_fresh &= ~bit;
          }
        }
        ++done;
      }
    }
    if (lane == 0 && *abort_flag) {
      // Drain: wait (bounded) for the loads that may still be in flight.
      if (kq)
        for (uint32_t n = (q_it > (uint32_t)kStagesQ ? q_it - kStagesQ : 0); n < q_it; ++n)
          mbar_wait_drain(bar(BAR_QFULL + n % kStagesQ), (n / kStagesQ) & 1, 100000000ull);
      if (kRope && kq) {
        // the latest load of each stage, on the barrier it completes on
        for (int st = 0; st < nst && st < (int)done; ++st) {
          const uint32_t bit = 1u << st;
          if (last_fresh & bit)
            mbar_wait_drain(bar(BAR_KFRESH + st), ((kfresh_par & bit) ? 1u : 0u) ^ 1u, 100000000ull);
          else
            mbar_wait_drain(bar(BAR_KFULL + st), ((kfull_par & bit) ? 1u : 0u) ^ 1u, 100000000ull);
        }
      } else {
        for (uint32_t n = (done > (uint32_t)nst ? done - nst : 0); n < done; ++n)
          mbar_wait_drain(bar(bfull + n % nst), (n / nst) & 1, 100000000ull);
      }
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
      // S(sb) = Q(qs) K(kst)^T over n_rows kv rows
      auto qk = [&](int qs, int kst, int n_rows, uint32_t sb) {
        const uint32_t idesc =
            n_rows == kTileN ? idesc_qk_full : make_idesc_bf16(128, (n_rows + 15) & ~15, false);
        const uint64_t a = dq0 + (uint64_t)qs * kStageStep, b = dk0 + (uint64_t)kst * kStageStep;
        const uint32_t d = tmem + sb * 128;
#pragma unroll
        for (int s = 0; s < kD / 16; ++s) {
          const uint64_t off = (uint64_t)(((s >> 2) * kChunkBytes + (s & 3) * 32) >> 4);
          umma_ss(d, a + off, b + off, idesc, s > 0 ? 1u : 0u);
        }
      };
      // O_h (+)= P_h V[64h .. 64h + 16 ksteps): P_h sits in TMEM at S buffer
      // column 64h, V rows 64h.. are K-steps 4h.. of the stage.
      auto pv_half = [&](int vst, uint32_t sb, int h, int ksteps, bool acc) {
        const uint64_t b = dv0 + (uint64_t)vst * kStageStep;
        const uint32_t d = tmem + 256 + h * 128;
        const uint32_t a = tmem + sb * 128 + h * kHalfN;
        if (ksteps == 4) {
#pragma unroll
          for (int s = 0; s < 4; ++s)
            umma_ts(d, a + s * 8, b + (uint64_t)((4 * h + s) * (2048 >> 4)), idesc_pv,
                    (acc || s > 0) ? 1u : 0u);
        } else {
          for (int s = 0; s < ksteps; ++s)
            umma_ts(d, a + s * 8, b + (uint64_t)((4 * h + s) * (2048 >> 4)), idesc_pv,
                    (acc || s > 0) ? 1u : 0u);
        }
      };
      uint32_t q_it = 0, k_it = 0, v_it = 0;
      uint32_t g = 0;  // KV tiles whose PVs were issued (all units), = S tile index
      // Rotary launches: per-stage phase parities of KFULL (cached tiles) and
      // KROPED (fresh tiles, released by the rotary warp).
      uint32_t kc_par = 0, kr_par = 0;
      // A K tile is ready for QK once it landed, or, for a fresh tile of a
      // rotary launch, once the rotary warp released it.
      auto wait_k = [&](int kst, int seg) -> bool {
        if (kRope) {
          uint32_t& pp = seg == 1 ? kr_par : kc_par;
          const uint32_t par = (pp >> kst) & 1u;
          pp ^= 1u << kst;
          return mbar_wait(bar((seg == 1 ? BAR_KROPED : BAR_KFULL) + kst), par, abort_flag);
        }
        return mbar_wait(bar(BAR_KFULL + kst), (k_it / kStagesK) & 1, abort_flag);
      };
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const Unit t = decode_unit(u, args);
        if (!t.valid) continue;
        const int qs = q_it % kStagesQ;
        ok = mbar_wait(bar((kRope ? BAR_QROPED : BAR_QFULL) + qs), (q_it / kStagesQ) & 1, abort_flag);
        if (!ok) break;
        ++q_it;
        if (t.nkv == 0) {
          umma_commit(bar(BAR_QEMPTY + qs));
          continue;
        }
        // Prologue: S of the unit's first two tiles.
        const int npro = t.nkv < 2 ? t.nkv : 2;
        for (int j = 0; j < npro && ok; ++j) {
          const KvTile kt = kv_tile(j, t.nc, t.c_begin, t.nk, t.k_begin);
          const int kst = k_it % kStagesK;
          ok = wait_k(kst, kt.seg);
          if (!ok) break;
          tc_fence_after();
          qk(qs, kst, kt.valid, (g + j) & 1);
          umma_commit(bar(BAR_SFULL + ((g + j) & 1)));
          umma_commit(bar(BAR_KEMPTY + kst));
          ++k_it;
        }
        if (!ok) break;
        if (t.nkv <= 2) umma_commit(bar(BAR_QEMPTY + qs));  // every QK of the unit issued
        bool b_started = false;  // O_b written in this unit
        for (int j = 0; j < t.nkv && ok; ++j, ++g) {
          const KvTile kt = kv_tile(j, t.nc, t.c_begin, t.nk, t.k_begin);
          const uint32_t sb = g & 1;
          const int vst = v_it % kStagesV;
          ok = mbar_wait(bar(BAR_VFULL + vst), (v_it / kStagesV) & 1, abort_flag);
          if (!ok) break;
          ok = mbar_wait(bar(BAR_PFULL + sb), (g >> 1) & 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const int ks = (kt.valid + 15) >> 4;  // 1..8 K-steps
          pv_half(vst, sb, 0, ks < 4 ? ks : 4, j > 0);
          if (ks > 4) {
            pv_half(vst, sb, 1, ks - 4, b_started);
            b_started = true;
          }
          umma_commit(bar(BAR_VEMPTY + vst));
          umma_commit(bar(BAR_OREADY));
          ++v_it;
          if (j + 2 < t.nkv) {
            const KvTile kn = kv_tile(j + 2, t.nc, t.c_begin, t.nk, t.k_begin);
            const int kst = k_it % kStagesK;
            ok = wait_k(kst, kn.seg);
            if (!ok) break;
            tc_fence_after();
            qk(qs, kst, kn.valid, sb);  // tile g + 2 uses the same S buffer
            umma_commit(bar(BAR_SFULL + sb));
            umma_commit(bar(BAR_KEMPTY + kst));
            ++k_it;
            if (j + 3 == t.nkv) umma_commit(bar(BAR_QEMPTY + qs));  // last QK issued
          }
        }
        if (!ok) break;
        umma_commit(bar(BAR_OFULL));
      }
      // Make sure every issued MMA has finished before TMEM is released.
      umma_commit(bar(BAR_DRAIN));
      mbar_wait_drain(bar(BAR_DRAIN), 0, 100000000ull);
    }
    __syncwarp();
  } else if (warp == 11) {
    // ------------------------------------------------------------- rotary
    // (rotary launches only) Follows the producer's order: the unit's Q tile
    // (rotated and released on its stage's QROPED barrier), then its fresh K
    // tiles (each completes on its stage's KFRESH barrier and is rotated and
    // released on KROPED); cached K tiles were rotated before they were
    // stored and bypass this warp (only counted, for the ring positions). A
    // stage holding a Q tile or a fresh K tile is refilled only after the MMA
    // warp consumed it, which needs this warp's release, so neither barrier
    // can run two phases ahead of this warp. The producer issues the next
    // unit's Q right after this unit's last K tile, about two KV tiles before
    // the unit ends, so the next Q is rotated off the critical path.
    uint32_t q_it = 0, k_it = 0, kf_par = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      const Unit t = decode_unit(u, args);
      if (!t.valid) continue;
      const int qs = q_it % kStagesQ;
      ok = mbar_wait_warp(bar(BAR_QFULL + qs), (q_it / kStagesQ) & 1, abort_flag);
      if (!ok) break;
      ++q_it;
      rope_tile_smem(smem + kOffQ + qs * kTileBytes, lane, args, (int64_t)t.q_begin + t.q0,
                     min(t.Lq - t.q0, kTileM / args.qpack), args.qpack, t.nheads);
      fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_QROPED + qs));
      for (int j = 0; j < t.nkv && ok; ++j, ++k_it) {
        const KvTile kt = kv_tile(j, t.nc, t.c_begin, t.nk, t.k_begin);
        if (kt.seg != 1) continue;
        const int kst = k_it % kStagesK;
        const uint32_t bit = 1u << kst;
        ok = mbar_wait_warp(bar(BAR_KFRESH + kst), (kf_par & bit) ? 1u : 0u, abort_flag);
        if (!ok) break;
        kf_par ^= bit;
        rope_tile_smem(smem + kOffK + kst * kTileBytes, lane, args, kt.row0, kt.valid, 1, 1);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(BAR_KROPED + kst));
      }
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax
    const int wg = warp >> 2;           // 0: kv rows 0-63 of a tile, 1: rows 64-127
    const int wq = warp & 3;            // warp within the warpgroup
    const int row_in_tile = threadIdx.x & 127;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tOwn = tmem + lane_base + 256 + wg * 128;  // this warpgroup's accumulator
    const uint32_t tOa = tmem + lane_base + 256;
    const uint32_t tOb = tmem + lane_base + 384;
    float2* xch = reinterpret_cast<float2*>(smem + kOffXch);
    const float sl2 = args.scale_log2;
    uint32_t g = 0, o_it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      const Unit t = decode_unit(u, args);
      if (!t.valid) continue;
      float m = -INFINITY;  // running max (log2 units), -inf until a valid column
      float l = 0.f;
      for (int j = 0; j < t.nkv; ++j, ++g) {
        const KvTile kt = kv_tile(j, t.nc, t.c_begin, t.nk, t.k_begin);
        const uint32_t sb = g & 1;
        ok = mbar_wait_warp(bar(BAR_SFULL + sb), (g >> 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t tS = tmem + lane_base + sb * 128 + wg * kHalfN;
        int nv = kt.valid - wg * kHalfN;  // valid columns of this half (warp-uniform)
        nv = nv < 0 ? 0 : (nv > kHalfN ? kHalfN : nv);
        if (nv > 0) {
          uint32_t s[2][32];
          tmem_ld32(tS, s[0]);
          tmem_ld32(tS + 32, s[1]);
          tmem_wait_ld();
          if (nv < kHalfN) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (c * 32 + e >= nv) s[c][e] = __float_as_uint(-INFINITY);
          }
          // row max: two independent 3-input max chains
          float mq[2];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float a = __uint_as_float(s[c][0]);
#pragma unroll
            for (int e = 1; e < 31; e += 2)
              a = max3f(a, __uint_as_float(s[c][e]), __uint_as_float(s[c][e + 1]));
            mq[c] = fmaxf(a, __uint_as_float(s[c][31]));
          }
          const float mxs = fmaxf(mq[0], mq[1]) * sl2;
          if (m == -INFINITY) {
            m = mxs;  // first valid columns: the accumulator starts fresh
          } else {
            // Lazy rescaling: keep a stale maximum while the new one exceeds
            // it by at most 8 (log2 units), so P stays <= 256 and O/l stay
            // exact up to rounding; rescale O only when a warp needs it.
            const bool need = mxs > m + 8.f;
            if (__any_sync(0xffffffffu, need)) {
              const float mn = fmaxf(m, mxs);
              const float alpha = ex2_approx(m - mn);
              m = mn;
              l *= alpha;
              // The accumulator must hold every PV up to tile g-1: PV(g-2)
              // completed before S(g) did, so one more completion of OREADY
              // (parity of tile g-1) is all there is to wait for.
              ok = mbar_wait_warp(bar(BAR_OREADY), (g - 1) & 1, abort_flag);
              if (!ok) break;
              tc_fence_after();
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                uint32_t o[32];
                tmem_ld32(tOwn + c * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                tmem_st32(tOwn + c * 32, o);
              }
            }
          }
          l += exp_store_half(s, sl2, m, tS);  // masked columns give exact zeros
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(BAR_PFULL + sb));
      }
      if (!ok) break;
      // Epilogue: merge the two halves, O / l -> bf16 -> global. Warpgroup w
      // writes output columns [64w, 64w + 64).
      // tile row -> (query row, packed head): the TMA box stores row r of head
      // hq + hh at tile row r * qpack + hh
      const int rr = row_in_tile / args.qpack;
      const int hh = row_in_tile - rr * args.qpack;
      const int row = t.q0 + rr;
      const bool row_ok = row < t.Lq && hh < t.nheads;
      __nv_bfloat16* orow = args.o + (int64_t)(t.q_begin + row) * args.o_tok_stride +
                            (int64_t)(t.hq + hh) * args.o_head_stride + wg * kHalfN;
      if (t.nkv > 0) {
        ok = mbar_wait_warp(bar(BAR_OFULL), o_it & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        // Merge factors: O = ca * O_a + cb * O_b with ca = 2^(m0-m)/L,
        // cb = 2^(m1-m)/L, m = max(m0, m1), L = l0 2^(m0-m) + l1 2^(m1-m).
        // Warpgroup 0 always has a valid column (every tile has >= 1 row);
        // warpgroup 1 may have none (m1 = -inf), then O_b was never written.
        float ca, cb;
        if (wg == 1) {
          xch[row_in_tile] = make_float2(m, l);
          mbar_arrive(bar(BAR_XML));
          ok = mbar_wait_warp(bar(BAR_XF), o_it & 1, abort_flag);
          if (!ok) break;
          const float2 f = xch[row_in_tile];
          ca = f.x;
          cb = f.y;
        } else {
          ok = mbar_wait_warp(bar(BAR_XML), o_it & 1, abort_flag);
          if (!ok) break;
          const float2 o1 = xch[row_in_tile];
          const float mm = fmaxf(m, o1.x);
          const float fa = ex2_approx(m - mm);
          const float fb = o1.x == -INFINITY ? 0.f : ex2_approx(o1.x - mm);
          const float inv = 1.f / (l * fa + o1.y * fb);
          ca = fa * inv;
          cb = fb * inv;
          xch[row_in_tile] = make_float2(ca, cb);
          mbar_arrive(bar(BAR_XF));
        }
        ++o_it;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t oa[32], ob[32];
          tmem_ld32(tOa + wg * kHalfN + c * 32, oa);
          tmem_ld32(tOb + wg * kHalfN + c * 32, ob);
          tmem_wait_ld();
          if (row_ok) {
            float v[32];
            if (cb != 0.f) {
#pragma unroll
              for (int e = 0; e < 32; ++e)
                v[e] = fmaf(__uint_as_float(oa[e]), ca, __uint_as_float(ob[e]) * cb);
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(oa[e]) * ca;
            }
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w4;
              w4.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
              w4.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
              w4.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
              w4.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
              dst[q] = w4;
            }
          }
        }
        // O is read out; the next unit's first PV may overwrite it once every
        // softmax warp arrives on its first P barrier (program order + fence).
        tc_fence_before();
      } else if (row_ok) {
        // No keys at all: the output row is zero.
        uint4* dst = reinterpret_cast<uint4*>(orow);
        for (int v = 0; v < kHalfN / 8; ++v) dst[v] = make_uint4(0, 0, 0, 0);
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

}  // namespace split

cudaError_t launch_attn_fwd_split(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                            const CUtensorMap& tmKc, const CUtensorMap& tmVc,
                            const AttnKernelArgs& args, int max_q, int num_sms,
                            cudaStream_t stream) {
  // The smem opt-in is per device and instantiation; remember it for up to 64 devices.
  static std::atomic<bool> attr_set[2][64];
  const bool rope = args.positions != nullptr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[rope][dev]) {
    e = rope ? cudaFuncSetAttribute(split::attn_fwd_split_kernel<true>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)split::kSmemBytes)
             : cudaFuncSetAttribute(split::attn_fwd_split_kernel<false>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)split::kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[rope][dev] = true;
  }
  AttnKernelArgs a = args;
  long long units;
  if (a.qpack > 1) {
    if (max_q > split::kTileM / a.qpack) return cudaErrorInvalidValue;
    a.qunits = (a.group + a.qpack - 1) / a.qpack;
    units = (long long)a.B * a.Hkv * a.qunits;
  } else {
    a.qunits = (max_q + split::kTileM - 1) / split::kTileM;
    if (a.head_idx == nullptr) a.n_heads = a.Hq;
    units = (long long)a.B * a.n_heads * a.qunits;
  }
  if (units == 0) return cudaSuccess;
  if (units > 0x7fffffffLL) return cudaErrorInvalidValue;
  a.total_units = (int)units;
  const int grid = (int)(units < num_sms ? units : num_sms);
  // Programmatic dependent launch: this grid may start while the previous
  // kernel in the stream finishes; it waits for it in griddep_wait().
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(rope ? split::kThreadsRope : split::kThreads, 1, 1);
  cfg.dynamicSmemBytes = split::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return rope ? cudaLaunchKernelEx(&cfg, split::attn_fwd_split_kernel<true>, tmQ, tmK, tmV, tmKc, tmVc, a)
              : cudaLaunchKernelEx(&cfg, split::attn_fwd_split_kernel<false>, tmQ, tmK, tmV, tmKc, tmVc, a);
}

}  // namespace dllm
