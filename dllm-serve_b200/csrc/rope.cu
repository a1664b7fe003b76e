// NeoX-style rotary embedding of q and k, sm_100a.
//
// Restates RotaryEmbedding.forward (dllmserve/layers/rotary_embedding.py:41-57)
// with apply_rotary_emb (:6-16): per token, cos, sin = cos_sin_cache[pos]
// (the cache rows hold [cos | sin] of the 64 rotation angles); per head, with
// x1 = x[0:64], x2 = x[64:128] in fp32,
//   y1 = x1*cos - x2*sin,   y2 = x2*cos + x1*sin,
// rounded to bf16. Products and sums are separately rounded (no fused
// multiply-add), as the reference's elementwise fp32 ops are, so the bf16
// result matches it bit for bit. HBM-bound: one read and one write of every
// q/k element; the cache rows are reused across heads from registers.
//
// Layout: thread group of 8 lanes per head (lane j covers dims 8j..8j+7 of
// each half, 16-byte loads), 32 heads per 256-thread pass; a CTA walks tokens.
#include "common.cuh"
#include "rope.h"

namespace dllm {

namespace {

constexpr int kD = 128;
constexpr int kHalf = 64;
constexpr int kThreads = 256;
constexpr int kHeadsPerPass = kThreads / 8;

// Row of head h (q heads first, then k heads) of token t, input or output.
DLLM_DEVICE const __nv_bfloat16* head_row(const RopeArgs& a, int64_t t, int h, bool out) {
  const bool isq = h < a.Hq;
  const int hh = isq ? h : h - a.Hq;
  if (isq) return (out ? a.q_out : a.q_in) + t * (out ? a.q_out_stride : a.q_in_stride) + (int64_t)hh * kD;
  return (out ? a.k_out : a.k_in) + t * (out ? a.k_out_stride : a.k_in_stride) + (int64_t)hh * kD;
}

__global__ void __launch_bounds__(kThreads) rope_kernel(RopeArgs a) {
  const int lane8 = threadIdx.x & 7;   // dims [8*lane8, 8*lane8 + 8) of each half
  const int hslot = threadIdx.x >> 3;  // head within a pass
  const int nh = a.Hq + a.Hkv;
  // Programmatic dependent launch: inputs are read only after the previous
  // grid in the stream finished; the next grid may start its prologue now.
  griddep_wait();
  griddep_launch_dependents();
  for (int64_t t = blockIdx.x; t < a.n_tokens; t += gridDim.x) {
    const int64_t pos = a.positions[t];
    const bool pos_ok = pos >= 0 && pos < a.max_position;
    float c[8], s[8];
    if (pos_ok) {
      const float4* row = reinterpret_cast<const float4*>(a.cos_sin + pos * kD);
      const float4 c0 = __ldg(row + 2 * lane8), c1 = __ldg(row + 2 * lane8 + 1);
      const float4 s0 = __ldg(row + kHalf / 4 + 2 * lane8), s1 = __ldg(row + kHalf / 4 + 2 * lane8 + 1);
      c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w;
      c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
      s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w;
      s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
    } else {
      if (threadIdx.x == 0) set_error(a.err, kDevPositionOutOfRange);
#pragma unroll
      for (int i = 0; i < 8; ++i) c[i] = s[i] = 0.f;  // the rows become zero
    }
    for (int h = hslot; h < nh; h += kHeadsPerPass) {
      const __nv_bfloat16* src = head_row(a, t, h, false);
      __nv_bfloat16* dst = const_cast<__nv_bfloat16*>(head_row(a, t, h, true));
      uint4 w1 = *reinterpret_cast<const uint4*>(src + 8 * lane8);
      uint4 w2 = *reinterpret_cast<const uint4*>(src + kHalf + 8 * lane8);
      rope_rotate8(w1, w2, c, s);
      *reinterpret_cast<uint4*>(dst + 8 * lane8) = w1;
      *reinterpret_cast<uint4*>(dst + kHalf + 8 * lane8) = w2;
    }
  }
}

}  // namespace

cudaError_t launch_rope(const RopeArgs& a, int num_sms, cudaStream_t stream) {
  if (a.n_tokens <= 0) return cudaSuccess;
  const int64_t cap = (int64_t)num_sms * 8;  // 8 CTAs of 256 threads per SM
  const int grid = (int)(a.n_tokens < cap ? a.n_tokens : cap);
  return launch_pdl(rope_kernel, dim3(grid), dim3(kThreads), 0, stream, a);
}

}  // namespace dllm
