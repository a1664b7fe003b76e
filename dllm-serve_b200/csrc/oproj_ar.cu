// Row-parallel o_proj fused with its all-reduce over NVLink peer memory, sm_100a.
//
// Replaces, under tensor parallelism, RowParallelLinear.forward's
// `y = F.linear(x, W_r)` followed by `dist.all_reduce(y)`
// (dllmserve/layers/linear.py:186-190): every rank r holds x_r [M, K] (the
// attention output of its heads) and W_r [N, K] (its column slice of W_o);
// the result y = sum_r x_r W_r^T [M, N] lands on every rank.
//
// One persistent kernel per rank, a CTA per SM:
//   A) GEMM: 128 x 256 output tiles, K in 64-column chunks (TMA -> shared
//      memory, SW128), tcgen05.mma into a double-buffered TMEM accumulator;
//      the epilogue turns a finished tile into bf16 and writes it, with
//      coalesced 512-byte row stores, into the tile owner's receive buffer
//      (owner = tile index mod tp; plain stores through an IPC mapping of the
//      owner's memory, or local), then raises the tile's flag on the owner
//      (system-scope release, value = this call's epoch).
//   B) Meanwhile two warps of each CTA take the tiles the rank owns: they
//      wait for the tp partials (bounded), sum them in rank order in fp32,
//      round once to bf16 and write the result to every rank's output (plain
//      peer stores), then raise the tile's final flag on every other rank.
//   C) The rank waits for the final flags of the tiles it does not own, so
//      its output is complete when the kernel ends.
// With tp == 1 the epilogue writes the result directly (a plain GEMM).
// Phase A waits on nothing outside the GPU, so no cycle of waits exists
// across ranks; every wait is bounded (kWaitLimitNs) and a timeout anywhere
// raises DLLM_DEV_WAIT_TIMEOUT in the status word, which every other wait
// of this GPU's CTAs also watches. No TMA and no library code reads peer
// memory, and no multicast is used.
#include "common.cuh"
#include "oproj_ar.h"

namespace dllm {

namespace {

constexpr int kTM = 128, kTN = 256, kTK = 64;
constexpr int kStages = 4;
constexpr uint32_t kABytes = kTM * kTK * 2;                 // 16 KB
constexpr uint32_t kBBytes = kTN * kTK * 2;                 // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;         // 48 KB
constexpr uint32_t kOffOut = kStages * kStageBytes;         // bf16 staging of half a tile, 32 KB
constexpr uint32_t kOutBytes = kTM * (kTN / 2) * 2;
constexpr uint32_t kOffBar = kOffOut + kOutBytes;
constexpr int BAR_FULL = 0, BAR_EMPTY = kStages, BAR_ACCF = 2 * kStages, BAR_ACCE = 2 * kStages + 2;
constexpr int BAR_DRAIN = 2 * kStages + 4;
constexpr int kNumBars = 2 * kStages + 5;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 64 + 1024;       // + alignment slack
constexpr int kThreads = 256;  // warp 0 TMA, warp 1 MMA, warps 2-3 reduce, warps 4-7 epilogue
constexpr int kReduceBatch = 8;  // 16-byte vectors in flight per reducing thread

// Spin (bounded) until *flag == epoch. False on timeout or when another CTA of
// this GPU gave up (status word set); a timeout sets the status word.
DLLM_DEVICE bool wait_flag(const int32_t* flag, int32_t epoch, int32_t* err) {
  if (ld_acquire_sys(flag) == epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    if (ld_acquire_sys(flag) == epoch) return true;
    if (err != nullptr && *reinterpret_cast<volatile int32_t*>(err) != 0) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_error(err, kDevWaitTimeout);
      return false;
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    oproj_ar_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    OprojArArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t bar0 = base + kOffBar;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc + 16);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(BAR_FULL + s), 1);
      mbar_init(bar(BAR_EMPTY + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(BAR_ACCF + i), 1);
      mbar_init(bar(BAR_ACCE + i), 4);  // one arrival per epilogue warp
    }
    mbar_init(bar(BAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int kchunks = a.K / kTK;
  const int64_t MN = (int64_t)a.M * a.N;

  // ---------------------------------------------------------------- phase A
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_first(), pol_b = policy_evict_last();
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x) {
        const int tm = t / a.tiles_n, tn = t - tm * a.tiles_n;
        for (int kc = 0; kc < kchunks; ++kc, ++it) {
          const int st = it % kStages;
          if (it >= (uint32_t)kStages) ok = mbar_wait(bar(BAR_EMPTY + st), (it / kStages - 1) & 1, abort_flag);
          if (!ok) break;
          const uint32_t sa = base + st * kStageBytes;
          mbar_arrive_expect_tx(bar(BAR_FULL + st), kStageBytes);
          tma_load_2d(sa, &tmA, bar(BAR_FULL + st), kc * kTK, tm * kTM, pol_a);
          tma_load_2d(sa + kABytes, &tmB, bar(BAR_FULL + st), kc * kTK, tn * kTN, pol_b);
        }
      }
      if (*abort_flag) {
        for (uint32_t n = (it > (uint32_t)kStages ? it - kStages : 0); n < it; ++n)
          mbar_wait_drain(bar(BAR_FULL + n % kStages), (n / kStages) & 1, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(kTM, kTN, false);
      uint32_t it = 0, acc_it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x, ++acc_it) {
        const int buf = acc_it & 1;
        if (acc_it >= 2) ok = mbar_wait(bar(BAR_ACCE + buf), (acc_it / 2 - 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kTN;
        for (int kc = 0; kc < kchunks; ++kc, ++it) {
          const int st = it % kStages;
          ok = mbar_wait(bar(BAR_FULL + st), (it / kStages) & 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sa = base + st * kStageBytes;
          const uint64_t da = make_sw128_desc(sa, 16, 1024);
          const uint64_t db = make_sw128_desc(sa + kABytes, 16, 1024);
#pragma unroll
          for (int s = 0; s < kTK / 16; ++s)
            umma_ss(d, da + (uint64_t)(2 * s), db + (uint64_t)(2 * s), idesc, (kc > 0 || s > 0) ? 1u : 0u);
          umma_commit(bar(BAR_EMPTY + st));
        }
        if (!ok) break;
        umma_commit(bar(BAR_ACCF + buf));
      }
      // every issued MMA has finished before TMEM is released
      umma_commit(bar(BAR_DRAIN));
      mbar_wait_drain(bar(BAR_DRAIN), 0, 100000000ull);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------ epilogue (A)
    const int wq = warp & 3;
    const int rr = wq * 32 + lane;  // tile row held by this thread (TMEM lane)
    uint4* stage_out = reinterpret_cast<uint4*>(smem + kOffOut);
    uint32_t acc_it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x, ++acc_it) {
      const int tm = t / a.tiles_n, tn = t - tm * a.tiles_n;
      const int buf = acc_it & 1;
      ok = mbar_wait_warp(bar(BAR_ACCF + buf), (acc_it / 2) & 1, abort_flag);
      // the four epilogue warps leave together (named barriers follow)
      ok = named_barrier_and(1, 128, ok);
      if (!ok) break;
      tc_fence_after();
      // tp == 1: the tile is the result; else the partial goes to its owner
      const int owner = t % a.tp;
      __nv_bfloat16* dst = a.tp == 1
                               ? a.y[0] + (int64_t)(tm * kTM) * a.N + tn * kTN
                               : a.recv[owner] + (int64_t)a.rank * MN + (int64_t)(tm * kTM) * a.N + tn * kTN;
      for (int h = 0; h < 2; ++h) {
        // TMEM -> bf16 -> staging (row rr: 16 chunks of 16 B, chunk j at j ^ (rr & 7))
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + buf * kTN + h * (kTN / 2) + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * q + 0]), __uint_as_float(v[8 * q + 1]));
            w.y = pack_bf16x2(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3]));
            w.z = pack_bf16x2(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5]));
            w.w = pack_bf16x2(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7]));
            const int j = c * 4 + q;
            stage_out[rr * 16 + (j ^ (rr & 7))] = w;
          }
        }
        if (h == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(BAR_ACCE + buf));  // TMEM buffer free for the next tile
        }
        named_barrier(1, 128);
        // staging -> destination: two 256-byte row halves per warp step
        for (int i = wq * 32 + lane; i < kTM * 16; i += 128) {
          const int r = i >> 4, ch = i & 15;
          if (tm * kTM + r >= a.M) break;
          reinterpret_cast<uint4*>(dst + (int64_t)r * a.N + h * (kTN / 2))[ch] = stage_out[r * 16 + (ch ^ (r & 7))];
        }
        named_barrier(1, 128);  // staging read before the next half overwrites it
      }
      if (a.tp > 1) {
        __threadfence_system();
        named_barrier(1, 128);
        if (wq == 0 && lane == 0) st_release_sys(a.flags[owner] + (int64_t)a.rank * a.num_tiles + t, a.epoch);
      }
    }
  } else if (a.tp > 1) {
    // -------------------------------------- warps 2-3: reduction (B), overlapping A
    // Tiles owned by this rank, t = rank + tp * k for k = blockIdx.x,
    // blockIdx.x + gridDim.x, ...: wait for the tp partials, sum them in rank
    // order, push the result to every rank, raise the final flags.
    const int tid = threadIdx.x - 64;
    const int64_t fin = (int64_t)a.tp * a.num_tiles;
    const __nv_bfloat16* own = a.recv[a.rank];
    bool ok = true;
    for (int t = a.rank + a.tp * (int)blockIdx.x; t < a.num_tiles && ok; t += a.tp * (int)gridDim.x) {
      bool got = true;
      if (tid == 0)
        for (int src = 0; src < a.tp && got; ++src)
          got = wait_flag(a.flags[a.rank] + (int64_t)src * a.num_tiles + t, a.epoch, a.err);
      ok = named_barrier_and(2, 64, got);
      if (!ok) break;
      const int tm = t / a.tiles_n, tn = t - tm * a.tiles_n;
      for (int v0 = tid; v0 < kTM * (kTN / 8); v0 += 64 * kReduceBatch) {
        float acc[kReduceBatch][8];
        int64_t off[kReduceBatch];
        bool in[kReduceBatch];
#pragma unroll
        for (int b = 0; b < kReduceBatch; ++b) {
          const int v = v0 + b * 64;
          const int r = v / (kTN / 8), cc = v - r * (kTN / 8);
          in[b] = v < kTM * (kTN / 8) && tm * kTM + r < a.M;
          off[b] = (int64_t)(tm * kTM + r) * a.N + tn * kTN + cc * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[b][e] = 0.f;
        }
        for (int src = 0; src < a.tp; ++src) {
          uint4 w[kReduceBatch];
#pragma unroll
          for (int b = 0; b < kReduceBatch; ++b)
            w[b] = in[b] ? __ldcg(reinterpret_cast<const uint4*>(own + (int64_t)src * MN + off[b]))
                         : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int b = 0; b < kReduceBatch; ++b) {
            float x[8];
            bf16x8_to_f32(w[b], x);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[b][e] += x[e];
          }
        }
#pragma unroll
        for (int b = 0; b < kReduceBatch; ++b) {
          if (!in[b]) continue;
          uint4 o;
          o.x = pack_bf16x2(acc[b][0], acc[b][1]);
          o.y = pack_bf16x2(acc[b][2], acc[b][3]);
          o.z = pack_bf16x2(acc[b][4], acc[b][5]);
          o.w = pack_bf16x2(acc[b][6], acc[b][7]);
          for (int p = 0; p < a.tp; ++p) *reinterpret_cast<uint4*>(a.y[p] + off[b]) = o;
        }
      }
      __threadfence_system();
      named_barrier(2, 64);
      if (tid == 0)
        for (int p = 0; p < a.tp; ++p)
          if (p != a.rank) st_release_sys(a.flags[p] + fin + t, a.epoch);
    }
  }
  // ---------------------------------------------------------------- phase C
  // Final tiles of the other owners, spread over the CTAs (thread 0, once
  // this CTA's GEMM tiles are out).
  if (a.tp > 1 && threadIdx.x == 0 && *abort_flag == 0) {
    const int64_t fin = (int64_t)a.tp * a.num_tiles;
    for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
      if (t % a.tp == a.rank) continue;
      if (!wait_flag(a.flags[a.rank] + fin + t, a.epoch, a.err)) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) set_error(a.err, kDevWaitTimeout);
}

uint32_t oproj_ar_smem_bytes() { return kSmemBytes; }

cudaError_t launch_oproj_ar(const CUtensorMap& tmA, const CUtensorMap& tmB, const OprojArArgs& args,
                            int num_sms, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(oproj_ar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  // Every CTA must be resident at once (a CTA waits for tiles other CTAs of
  // this GPU write): one CTA per SM, at most as many CTAs as SMs.
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, oproj_ar_kernel, kThreads, kSmemBytes);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int grid = args.num_tiles < num_sms ? args.num_tiles : num_sms;
  oproj_ar_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmA, tmB, args);
  return cudaGetLastError();
}

}  // namespace dllm
