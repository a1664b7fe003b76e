// Device-side helpers shared by the sm_100a kernels of the attention path:
// mbarriers with bounded waits, TMA (cp.async.bulk.tensor, per-CTA only, never
// multicast), tcgen05 (TMEM alloc / MMA / ld / st / commit) and the UMMA
// shared-memory and instruction descriptors.
//
// All inline PTX here is hand-written from the public PTX ISA description of
// these instructions.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#define DLLM_DEVICE __device__ __forceinline__

namespace dllm {

// ---------------------------------------------------------------------------
// Error flag codes written by kernels into the caller's optional status word.
// ---------------------------------------------------------------------------
enum DeviceError : int32_t {
  kDevOk = 0,
  kDevSlotOutOfRange = 1,     // a slot index >= num_slots (write skipped)
  kDevWaitTimeout = 2,        // an mbarrier wait exceeded its time limit
  kDevBadSequence = 3,        // inconsistent per-sequence metadata
  kDevPositionOutOfRange = 4, // a rotary position outside the cos/sin cache (row zeroed)
};

DLLM_DEVICE void set_error(int32_t* err, int32_t code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

DLLM_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DLLM_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
DLLM_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

DLLM_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DLLM_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

DLLM_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

DLLM_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the phase with the given parity (no suspend).
DLLM_DEVICE bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Time limit for any single mbarrier wait. A healthy wait in these kernels
// lasts microseconds; the limit only ends a wait that can never complete.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or ~hint ns pass, instead of spinning in software (a
// spinning warp steals issue slots from the warps that do the work).
DLLM_DEVICE bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and
// raises *abort) when the time limit passes or another role already aborted;
// callers then stop their loop and drain.
DLLM_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 200000u)) return true;  // <= 0.2 ms per sleep
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      return false;
    }
  }
}

// mbar_wait called by all 32 lanes of a warp: the lanes agree on the outcome,
// so a timeout seen by one lane cannot split the warp before a warp-wide
// operation (shuffle, vote, __syncwarp) that would then never complete.
DLLM_DEVICE bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}

// Bounded wait used while draining after an abort: never raises abort.
DLLM_DEVICE bool mbar_wait_drain(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// TMA (tensor maps live in kernel parameter space: __grid_constant__)
// ---------------------------------------------------------------------------
DLLM_DEVICE void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// Programmatic dependent launch: wait until the grids this one depends on have
// completed (and their memory is visible); allow the next grid in the stream
// to start launching (it still waits in its own griddep_wait).
DLLM_DEVICE void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DLLM_DEVICE void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: launches `kernel` with programmatic stream serialization (it may start
// while the previous grid in the stream finishes; the kernel calls
// griddep_wait() before reading anything that grid wrote) and, when
// cluster_x > 1, thread-block clusters of cluster_x CTAs along x.
template <typename Kernel, typename... Args>
inline cudaError_t launch_pdl_cluster(Kernel kernel, dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename Kernel, typename... Args>
inline cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  return launch_pdl_cluster(kernel, grid, block, smem, stream, 1, args...);
}
// 3-D tiled load, completes tx bytes on `bar`. No multicast.
DLLM_DEVICE void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1, int c2,
                             uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(cache_hint)
      : "memory");
}

// 2-D tiled load (coordinates: innermost first), completes tx bytes on `bar`.
// No multicast; the tensor map covers this GPU's own memory.
DLLM_DEVICE void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1,
                             uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "l"(cache_hint)
      : "memory");
}

// System-scope flag access (flags written by another GPU over NVLink).
DLLM_DEVICE int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
DLLM_DEVICE void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Barrier among `count` threads (whole warps) on hardware barrier `id` (1..15).
DLLM_DEVICE void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Barrier among `count` threads on hardware barrier `id` that also returns
// whether `pred` held for every one of them: warps that took a bounded wait
// agree on its outcome before any of them leaves a loop with barriers in it.
DLLM_DEVICE bool named_barrier_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// L2 eviction policies (createpolicy) for TMA cache hints.
DLLM_DEVICE uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
DLLM_DEVICE uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

DLLM_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads/stores, fences
// ---------------------------------------------------------------------------
// Whole warp must execute alloc / relinquish / dealloc.
DLLM_DEVICE void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
DLLM_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
DLLM_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

DLLM_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
DLLM_DEVICE void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)
DLLM_DEVICE void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc)
DLLM_DEVICE void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// mbarrier arrives once all previously issued tcgen05 async ops of this thread
// complete.
DLLM_DEVICE void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

DLLM_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
DLLM_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 32 consecutive columns per thread.
DLLM_DEVICE void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

DLLM_DEVICE void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
      "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}

DLLM_DEVICE void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (sm_100 tcgen05 format)
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle.
//   bits [0,14)  start address >> 4
//   bits [16,30) leading-dimension byte offset >> 4
//   bits [32,46) stride-dimension byte offset >> 4
//   bits [46,48) version = 1
//   bits [61,64) layout: 2 = SWIZZLE_128B
DLLM_DEVICE uint64_t make_sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor, kind::f16 with bf16 inputs and fp32 accumulator.
//   [4,6) D format (1 = f32), [7,10) A format (1 = bf16), [10,13) B format,
//   [15] A major (0 = K), [16] B major (1 = MN), [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------
DLLM_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

DLLM_DEVICE float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 4x4 transpose of 16-byte vectors inside each quad of lanes (j = lane & 3):
// on return v[r] holds what lane r of the quad had in v[j]. Two butterfly
// stages (xor 2 swaps the off-diagonal 2x2 blocks, xor 1 the off-diagonal
// elements inside them); every lane of the warp must take part.
DLLM_DEVICE uint4 shfl_xor_u4(uint4 a, int m) {
  uint4 r;
  r.x = __shfl_xor_sync(0xffffffffu, a.x, m);
  r.y = __shfl_xor_sync(0xffffffffu, a.y, m);
  r.z = __shfl_xor_sync(0xffffffffu, a.z, m);
  r.w = __shfl_xor_sync(0xffffffffu, a.w, m);
  return r;
}
DLLM_DEVICE void quad_transpose16(uint4 (&v)[4], int j) {
  const bool hi = (j & 2) != 0;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const uint4 r = shfl_xor_u4(hi ? v[s] : v[2 + s], 2);
    if (hi) v[s] = r; else v[2 + s] = r;
  }
  const bool odd = (j & 1) != 0;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const uint4 r = shfl_xor_u4(odd ? v[2 * s] : v[2 * s + 1], 1);
    if (odd) v[2 * s] = r; else v[2 * s + 1] = r;
  }
}

DLLM_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// bf16 x 8 (one 16-byte vector) <-> fp32 x 8.
DLLM_DEVICE void bf16x8_to_f32(uint4 w, float (&x)[8]) {
  x[0] = __uint_as_float(w.x << 16);
  x[1] = __uint_as_float(w.x & 0xffff0000u);
  x[2] = __uint_as_float(w.y << 16);
  x[3] = __uint_as_float(w.y & 0xffff0000u);
  x[4] = __uint_as_float(w.z << 16);
  x[5] = __uint_as_float(w.z & 0xffff0000u);
  x[6] = __uint_as_float(w.w << 16);
  x[7] = __uint_as_float(w.w & 0xffff0000u);
}

// NeoX rotation of 8 dimension pairs (x1 from the first half of a head row,
// x2 from the second): y1 = x1*cos - x2*sin, y2 = x2*cos + x1*sin in fp32
// with every product and sum rounded separately (no fused multiply-add), then
// rounded to bf16 -- the reference's elementwise fp32 ops, bit for bit
// (dllmserve/layers/rotary_embedding.py:6-16).
DLLM_DEVICE void rope_rotate8(uint4& w1, uint4& w2, const float (&c)[8], const float (&s)[8]) {
  float x1[8], x2[8];
  bf16x8_to_f32(w1, x1);
  bf16x8_to_f32(w2, x2);
  uint32_t o1[4], o2[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a0 = __fsub_rn(__fmul_rn(x1[2 * i], c[2 * i]), __fmul_rn(x2[2 * i], s[2 * i]));
    const float a1 = __fsub_rn(__fmul_rn(x1[2 * i + 1], c[2 * i + 1]), __fmul_rn(x2[2 * i + 1], s[2 * i + 1]));
    const float b0 = __fadd_rn(__fmul_rn(x2[2 * i], c[2 * i]), __fmul_rn(x1[2 * i], s[2 * i]));
    const float b1 = __fadd_rn(__fmul_rn(x2[2 * i + 1], c[2 * i + 1]), __fmul_rn(x1[2 * i + 1], s[2 * i + 1]));
    o1[i] = pack_bf16x2(a0, a1);
    o2[i] = pack_bf16x2(b0, b1);
  }
  w1 = make_uint4(o1[0], o1[1], o1[2], o1[3]);
  w2 = make_uint4(o2[0], o2[1], o2[2], o2[3]);
}

}  // namespace dllm
