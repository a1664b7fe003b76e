// Device-side step-metadata builder (step_plan.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dllm {

constexpr int kPlanSeqFields = 10;  // int64 fields per sequence (DLLM_PLAN_SEQ_FIELDS)
constexpr int kPlanDescInts = 8;    // int32 per selection descriptor (DLLM_SEQ_DESC_INTS)

struct StepPlanArgs {
  const int64_t* seqs;  // [batch, kPlanSeqFields] device
  int batch;
  int num_kv_heads;
  int32_t* out;         // cu at 0 (batch + 1), then the sections below
  int off_cu_c;
  int off_desc_hs, cap_desc_hs;
  int off_desc_sh, cap_desc_sh;
  int off_slots_c, cap_slots_c;
  int off_slots_hs, cap_slots_hs;
  int off_slots_sh, cap_slots_sh;
  int32_t* err;
};

int step_plan_max_batch();
cudaError_t launch_step_plan(const StepPlanArgs& a, cudaStream_t stream);

}  // namespace dllm
