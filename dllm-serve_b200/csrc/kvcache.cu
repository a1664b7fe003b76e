// Paged KV-cache store / load (slot-mapped row copies), sm_100a.
//
// store: cache[slot[i]] <- key[i], value[i]   (reference: dllmserve/layers/attention.py:11-50)
// load:  key[i], value[i] <- cache[slot[i]]   (reference: attention.py:53-92)
//
// One warp moves one token row of K and one of V with 16-byte vector accesses
// (the row is num_kv_heads*head_dim bf16 = 8 KB at LLaDA shapes, 512 vectors).
// Rows are independent, so the grid is sized to keep every SM busy with
// several warps in flight; each lane keeps 4 vectors outstanding per array.
#include "common.cuh"
#include "kvcache.h"

namespace dllm {

namespace {

template <typename V>
DLLM_DEVICE V ldg_nc(const V* p) {
  return __ldg(p);
}
template <>
DLLM_DEVICE uint4 ldg_nc<uint4>(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename V>
DLLM_DEVICE void copy_row(V* __restrict__ dst, const V* __restrict__ src, int64_t nvec, int lane) {
  constexpr int kU = 4;
  int64_t i = lane;
  for (; i + (kU - 1) * 32 < nvec; i += kU * 32) {
    V t[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) t[u] = ldg_nc(src + i + u * 32);
#pragma unroll
    for (int u = 0; u < kU; ++u) dst[i + u * 32] = t[u];
  }
  for (; i < nvec; i += 32) dst[i] = ldg_nc(src + i);
}

template <typename V>
DLLM_DEVICE void zero_row(V* dst, int64_t nvec, int lane) {
  V z;
  memset(&z, 0, sizeof(V));
  for (int64_t i = lane; i < nvec; i += 32) dst[i] = z;
}

// kStore: rows go token -> slot; otherwise slot -> token.
template <typename V, bool kStore>
__global__ void __launch_bounds__(256) kv_copy_kernel(KvCopyArgs a) {
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nvec = a.row_bytes / (int64_t)sizeof(V);
  griddep_wait();  // inputs are read only after the previous grid in the stream finished
  griddep_launch_dependents();
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < a.n_tokens;
       t += warps_total) {
    const int64_t slot = a.slots[t];
    const bool in_range = slot >= 0 && slot < a.num_slots;
    if (!in_range && slot >= 0 && lane == 0) set_error(a.err, kDevSlotOutOfRange);
    char* krow = (char*)a.key + t * a.key_stride_bytes;
    char* vrow = (char*)a.value + t * a.value_stride_bytes;
    char* kc = (char*)a.k_cache + slot * a.row_bytes;
    char* vc = (char*)a.v_cache + slot * a.row_bytes;
    if (kStore) {
      if (!in_range) continue;
      copy_row(reinterpret_cast<V*>(kc), reinterpret_cast<const V*>(krow), nvec, lane);
      copy_row(reinterpret_cast<V*>(vc), reinterpret_cast<const V*>(vrow), nvec, lane);
    } else {
      if (!in_range) {
        zero_row(reinterpret_cast<V*>(krow), nvec, lane);
        zero_row(reinterpret_cast<V*>(vrow), nvec, lane);
        continue;
      }
      copy_row(reinterpret_cast<V*>(krow), reinterpret_cast<const V*>(kc), nvec, lane);
      copy_row(reinterpret_cast<V*>(vrow), reinterpret_cast<const V*>(vc), nvec, lane);
    }
  }
}

template <typename V, bool kStore>
cudaError_t launch_typed(const KvCopyArgs& a, int num_sms, cudaStream_t stream) {
  constexpr int kWarps = 8;
  int64_t blocks = (a.n_tokens + kWarps - 1) / kWarps;
  // enough warps to cover HBM latency, grid-stride beyond that
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return launch_pdl(kv_copy_kernel<V, kStore>, dim3((unsigned)blocks), dim3(kWarps * 32), 0, stream, a);
}

}  // namespace

cudaError_t launch_kv_copy(const KvCopyArgs& a, bool store, int vec_bytes, int num_sms,
                           cudaStream_t stream) {
  if (a.n_tokens == 0) return cudaSuccess;
  switch (vec_bytes) {
    case 16:
      return store ? launch_typed<uint4, true>(a, num_sms, stream)
                   : launch_typed<uint4, false>(a, num_sms, stream);
    case 8:
      return store ? launch_typed<uint2, true>(a, num_sms, stream)
                   : launch_typed<uint2, false>(a, num_sms, stream);
    case 4:
      return store ? launch_typed<uint32_t, true>(a, num_sms, stream)
                   : launch_typed<uint32_t, false>(a, num_sms, stream);
    case 2:
      return store ? launch_typed<uint16_t, true>(a, num_sms, stream)
                   : launch_typed<uint16_t, false>(a, num_sms, stream);
    default:
      return store ? launch_typed<uint8_t, true>(a, num_sms, stream)
                   : launch_typed<uint8_t, false>(a, num_sms, stream);
  }
}

}  // namespace dllm
