// Internal launch interface of the KV-cache copy kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dllm {

struct KvCopyArgs {
  void* key;                  // token rows (source for store, destination for load)
  void* value;
  int64_t key_stride_bytes;
  int64_t value_stride_bytes;
  void* k_cache;              // slot rows, row_bytes apart
  void* v_cache;
  const int32_t* slots;
  int64_t n_tokens;
  int64_t row_bytes;
  int64_t num_slots;
  int32_t* err;
};

// vec_bytes: 16, 8, 4, 2 or 1 - the widest access every pointer/stride allows.
cudaError_t launch_kv_copy(const KvCopyArgs& a, bool store, int vec_bytes, int num_sms,
                           cudaStream_t stream);

}  // namespace dllm
