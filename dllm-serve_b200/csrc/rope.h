// Internal launch interface of the rotary-embedding kernel.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace dllm {

struct RopeArgs {
  const int64_t* positions;        // [n_tokens]
  const __nv_bfloat16* q_in;
  __nv_bfloat16* q_out;
  const __nv_bfloat16* k_in;
  __nv_bfloat16* k_out;
  int64_t q_in_stride, q_out_stride, k_in_stride, k_out_stride;  // elements between tokens
  const float* cos_sin;            // [max_position, head_dim]: cos | sin halves
  int64_t max_position;
  int64_t n_tokens;
  int Hq, Hkv;
  int32_t* err;
};

cudaError_t launch_rope(const RopeArgs& a, int num_sms, cudaStream_t stream);

}  // namespace dllm
