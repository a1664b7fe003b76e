// Internal launch interface of the fused row-parallel o_proj + all-reduce
// (oproj_ar.cu); the public C ABI is dllm_oproj_allreduce in include/dllm_attn.h.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace dllm {

constexpr int kOprojMaxRanks = 8;

struct OprojArArgs {
  int M, N, K;             // y[M, N] = sum over ranks of x_r[M, K] W_r[N, K]^T
  int rank, tp;
  int32_t epoch;           // this call's flag value (every rank passes the same)
  int tiles_m, tiles_n, num_tiles;
  __nv_bfloat16* recv[kOprojMaxRanks];  // rank p's receive buffer [tp][M][N] (this rank's address of it)
  __nv_bfloat16* y[kOprojMaxRanks];     // rank p's output [M][N]
  int32_t* flags[kOprojMaxRanks];       // rank p's flags: partial [tp][num_tiles], final [num_tiles]
  int32_t* err;            // status word (also the cross-CTA abort signal)
};

uint32_t oproj_ar_smem_bytes();
cudaError_t launch_oproj_ar(const CUtensorMap& tmA, const CUtensorMap& tmB, const OprojArArgs& args,
                            int num_sms, cudaStream_t stream);

}  // namespace dllm
