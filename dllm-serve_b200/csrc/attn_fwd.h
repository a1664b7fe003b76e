// Internal launch interface of the sm_100a attention kernel (not part of the
// public C ABI; see include/dllm_attn.h for that).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace dllm {

struct AttnKernelArgs {
  __nv_bfloat16* o;        // output rows, indexed like q
  int64_t o_tok_stride;    // elements between consecutive output rows
  int64_t o_head_stride;   // elements between heads inside a row
  const int32_t* cu_q;     // [B+1] query rows (and output rows) per sequence
  const int32_t* cu_k;     // [B+1] fresh key/value rows per sequence
  const int32_t* cu_c;     // [B+1] cached key/value rows per sequence, or null
  int B;
  int Hq;
  int Hkv;
  int group;               // Hq / Hkv
  float scale_log2;        // softmax_scale * log2(e)
  int32_t* err;            // optional device status word
  // Paged cached segment (optional): when `slots` is set, the cached rows of
  // sequence b are cache rows slots[cu_c[b] .. cu_c[b+1]) of kc/vc.
  const int32_t* slots;
  int64_t num_slots;
  const __nv_bfloat16* kc;
  const __nv_bfloat16* vc;
  int64_t c_tok_stride;    // elements between cache slots
  // Optional scheduler workspace (pair kernel): two int32 words, zero on entry,
  // zero again when the kernel exits. Launches that may run at the same time
  // need distinct workspaces. Null: static round-robin unit order.
  int32_t* sched;
  // Split kernel: query heads packed into one 128-row tile (GQA, every query
  // segment <= 128 / qpack rows; the Q tensor map's box is then (64, qpack,
  // 128 / qpack)). 1: one head per tile. The pair kernel requires 1.
  int qpack;
  // Query heads of the launch: head_idx[0 .. n_heads) when head_idx is set
  // (units are numbered over that list, so heads left out cost nothing; an
  // index outside [0, Hq) flags kDevBadSequence and its units are skipped),
  // else all Hq heads (n_heads = Hq). Requires qpack == 1.
  const int32_t* head_idx;
  int n_heads;
  int qunits;              // query units per (sequence, head): 256-row tile pairs (pair
                           // kernel) or 128-row tiles (split kernel); set by the launcher
  int total_units;         // B * n_heads * qunits; set by the launcher
  // Pair kernel: 1 = hand out the units of the sequences with the most key
  // tiles first (ties by sequence index), 0 = in sequence order. Set by the
  // launcher; it changes only which CTA computes a unit and when.
  int long_first;
  // Rotary embedding applied on chip (split kernel only; null positions: off).
  // Query row r and fresh key row r are rotated by cos_sin[positions[r]]
  // between their TMA arrival and the MMA that reads them; cached rows are
  // taken as already rotated.
  const int64_t* positions;
  const float* cos_sin;    // [max_position, 128] fp32: cos | sin halves
  int64_t max_position;
};

uint32_t attn_fwd_smem_bytes();
int attn_fwd_kv_rows_per_tile();  // rows of a key/value TMA box

// "Pair" kernel (attn_fwd.cu): a unit is two 128-row query tiles, one per
// softmax warpgroup. Used when some query segment is longer than 128 rows.
cudaError_t launch_attn_fwd(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                            const CUtensorMap& tmKc, const CUtensorMap& tmVc,
                            const AttnKernelArgs& args, int max_q, int num_sms,
                            cudaStream_t stream);

// "Split" kernel (attn_fwd_split.cu): a unit is one 128-row query tile and the
// two softmax warpgroups split each KV tile's columns. Used when max_q <= 128.
constexpr int kSplitMaxQ = 128;
cudaError_t launch_attn_fwd_split(const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                  const CUtensorMap& tmV, const CUtensorMap& tmKc,
                                  const CUtensorMap& tmVc, const AttnKernelArgs& args, int max_q,
                                  int num_sms, cudaStream_t stream);

}  // namespace dllm
