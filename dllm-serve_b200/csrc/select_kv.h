// Internal launch interface of the scoring / top-k / store kernel.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace dllm {

struct SelectArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_tok_stride, k_tok_stride, v_tok_stride;  // elements
  const int32_t* seq_desc;                           // [n_seqs, 8]
  int max_klen;
  int Hq, Hkv, group;
  float sqrt_d;                                      // fp32(sqrt(head_dim))
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t cache_tok_stride;                          // elements between slots
  int64_t num_slots;
  const int32_t* slots;
  int64_t* top_idx;                                  // optional
  int32_t* err;
};

size_t select_kv_smem_bytes(int nq, int max_klen);
cudaError_t launch_select_kv(const SelectArgs& a, bool head_select, int n_seqs, cudaStream_t stream);

}  // namespace dllm
