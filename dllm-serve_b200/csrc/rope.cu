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

DLLM_DEVICE uint4 f32x8_to_bf16(const float (&y)[8]) {
  uint4 w;
  w.x = pack_bf16x2(y[0], y[1]);
  w.y = pack_bf16x2(y[2], y[3]);
  w.z = pack_bf16x2(y[4], y[5]);
  w.w = pack_bf16x2(y[6], y[7]);
  return w;
}

__global__ void __launch_bounds__(kThreads) rope_kernel(RopeArgs a) {
  const int lane8 = threadIdx.x & 7;   // dims [8*lane8, 8*lane8 + 8) of each half
  const int hslot = threadIdx.x >> 3;  // head within a pass
  const int nh = a.Hq + a.Hkv;
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
      const bool isq = h < a.Hq;
      const int hh = isq ? h : h - a.Hq;
      const __nv_bfloat16* src = isq ? a.q_in + t * a.q_in_stride + (int64_t)hh * kD
                                     : a.k_in + t * a.k_in_stride + (int64_t)hh * kD;
      __nv_bfloat16* dst = isq ? a.q_out + t * a.q_out_stride + (int64_t)hh * kD
                               : a.k_out + t * a.k_out_stride + (int64_t)hh * kD;
      const uint4 w1 = *reinterpret_cast<const uint4*>(src + 8 * lane8);
      const uint4 w2 = *reinterpret_cast<const uint4*>(src + kHalf + 8 * lane8);
      float x1[8], x2[8], y1[8], y2[8];
      bf16x8_to_f32(w1, x1);
      bf16x8_to_f32(w2, x2);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        y1[i] = __fsub_rn(__fmul_rn(x1[i], c[i]), __fmul_rn(x2[i], s[i]));
        y2[i] = __fadd_rn(__fmul_rn(x2[i], c[i]), __fmul_rn(x1[i], s[i]));
      }
      *reinterpret_cast<uint4*>(dst + 8 * lane8) = f32x8_to_bf16(y1);
      *reinterpret_cast<uint4*>(dst + kHalf + 8 * lane8) = f32x8_to_bf16(y2);
    }
  }
}

}  // namespace

cudaError_t launch_rope(const RopeArgs& a, int num_sms, cudaStream_t stream) {
  if (a.n_tokens <= 0) return cudaSuccess;
  const int64_t cap = (int64_t)num_sms * 8;  // 8 CTAs of 256 threads per SM
  const int grid = (int)(a.n_tokens < cap ? a.n_tokens : cap);
  rope_kernel<<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace dllm
