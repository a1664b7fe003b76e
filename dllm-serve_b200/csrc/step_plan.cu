// Per-step metadata of the diffusion attention path, built on the device.
//
// Restates the per-sequence decisions the reference takes inside every layer
// (dllmserve/layers/attention.py:168-304, with the sizing rules of
// dllmserve/sparse/state.py:44-62 and dllmserve/engine/sequence.py:98-152)
// once per step, in one launch: from each sequence's raw state it derives the
// rows the sequence contributes, its current block, the cached rows it
// attends (reuse state) or the rows it selects (compute-cache state), writes
// the row offsets, the cached-row offsets and the selection descriptors, and
// gathers the sequences' slot lists into the concatenated lists the attention
// and selection launches read. One CTA; a sequence per thread.
#include "common.cuh"
#include "step_plan.h"

namespace dllm {

namespace {

constexpr int kPlanThreads = 1024;

struct SeqPlan {
  int rows, blk_start, blk_len, n_sel, n_cached, state, hs, pool;
};

// num_keep(n, r) = min(max(1, int(n * r)), n) for n > 0, else 0
// (attention.py:396-399, sequence.py:119-123); the product is a float64 and
// int() truncates toward zero, as in the reference's Python.
DLLM_DEVICE int num_keep_dev(int n, double r) {
  if (n <= 0) return 0;
  const long long k = (long long)((double)n * r);
  return (int)min((long long)n, max(1ll, k));
}

DLLM_DEVICE SeqPlan plan_of(const int64_t* row, int32_t* err) {
  SeqPlan p = {};
  const int state = (int)row[0];
  const int L = (int)row[1], P = (int)row[2], bidx = (int)row[3], blen_cfg = (int)row[4];
  const double ratio = __longlong_as_double(row[5]);
  p.pool = (int)(row[6] & 0xffffffff);
  p.hs = (int)(row[6] >> 32) & 1;
  p.state = state;
  // block boundaries (state.py:44-62)
  if (L - P <= 0) {
    p.blk_start = P;
    p.blk_len = 0;
  } else {
    p.blk_start = P + bidx * blen_cfg;
    p.blk_len = min(blen_cfg, L - p.blk_start);
  }
  if (state == 2) {
    // reuse: only the block's rows; keys = the cached selection + the block
    p.rows = p.blk_len;
    const int unused = max(0, p.blk_start) + max(0, L - (p.blk_start + p.blk_len));
    p.n_cached = num_keep_dev(unused, ratio);
  } else {
    p.rows = L;
    if (state == 1) {
      if (p.blk_len <= 0) set_error(err, kDevBadSequence);  // nothing to score
      p.n_sel = num_keep_dev(L - p.blk_len, ratio);
    } else if (state != 0) {
      set_error(err, kDevBadSequence);
    }
  }
  return p;
}

// Exclusive block-wide scan of v (every thread calls it); total in *total.
DLLM_DEVICE int block_scan_excl(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) warp_sums[lane] = s;  // inclusive warp prefix
  }
  __syncthreads();
  const int before = warp > 0 ? warp_sums[warp - 1] : 0;
  *total = warp_sums[(blockDim.x >> 5) - 1];
  __syncthreads();  // warp_sums is reused by the next scan
  return before + x - v;
}

__global__ void __launch_bounds__(kPlanThreads, 1) step_plan_kernel(StepPlanArgs a) {
  __shared__ int warp_sums[32];
  __shared__ int64_t src_ptr[kPlanThreads];
  __shared__ int dst_off[kPlanThreads];
  __shared__ int cnt[kPlanThreads];
  griddep_wait();
  griddep_launch_dependents();
  const int i = threadIdx.x;
  const bool in = i < a.batch;
  SeqPlan p = {};
  if (in) p = plan_of(a.seqs + (int64_t)i * kPlanSeqFields, a.err);
  const bool sel_hs = in && p.state == 1 && p.hs;
  const bool sel_sh = in && p.state == 1 && !p.hs;
  int total;
  const int row0 = block_scan_excl(in ? p.rows : 0, warp_sums, &total);
  const int c0 = block_scan_excl(in && p.state == 2 ? p.n_cached : 0, warp_sums, &total);
  const int d_hs = block_scan_excl(sel_hs ? 1 : 0, warp_sums, &total);
  const int d_sh = block_scan_excl(sel_sh ? 1 : 0, warp_sums, &total);
  const int s_hs = block_scan_excl(sel_hs ? p.n_sel : 0, warp_sums, &total);
  const int s_sh = block_scan_excl(sel_sh ? p.n_sel : 0, warp_sums, &total);
  const int x_hs = block_scan_excl(sel_hs ? p.n_sel * a.num_kv_heads : 0, warp_sums, &total);
  int32_t* out = a.out;
  if (in) {
    out[i] = row0;
    if (i == a.batch - 1) out[a.batch] = row0 + p.rows;
    int32_t* cu_c = out + a.off_cu_c;
    cu_c[i] = c0;
    if (i == a.batch - 1) cu_c[a.batch] = c0 + (p.state == 2 ? p.n_cached : 0);
    if (p.state == 1) {
      const int k = p.hs ? d_hs : d_sh;
      if (k < (p.hs ? a.cap_desc_hs : a.cap_desc_sh)) {
        int32_t* d = out + (p.hs ? a.off_desc_hs : a.off_desc_sh) + (int64_t)k * kPlanDescInts;
        d[0] = row0;
        d[1] = p.rows;
        d[2] = p.blk_start;
        d[3] = p.blk_len;
        d[4] = p.n_sel;
        d[5] = p.hs ? s_hs : s_sh;
        d[6] = p.hs ? x_hs : s_sh;  // top_idx offset: [Hkv, n_keep] per sequence with head_select, else [n_keep]
        d[7] = p.pool;
      } else {
        set_error(a.err, kDevBadSequence);
      }
    }
  }
  // slot lists into their concatenated sections (a warp per sequence)
  const int need = in ? (p.state == 2 ? p.n_cached : (p.state == 1 ? p.n_sel : 0)) : 0;
  const int64_t have = in ? a.seqs[(int64_t)i * kPlanSeqFields + 8] : 0;
  int off = 0, cap = 0;
  if (p.state == 2) {
    off = c0, cap = a.cap_slots_c;
  } else if (p.state == 1) {
    off = p.hs ? s_hs : s_sh;
    cap = p.hs ? a.cap_slots_hs : a.cap_slots_sh;
  }
  const bool ok = in && need > 0 && have == need && off + need <= cap;
  if (in && need > 0 && !ok) set_error(a.err, kDevBadSequence);
  src_ptr[i] = ok ? a.seqs[(int64_t)i * kPlanSeqFields + 7] : 0;
  cnt[i] = ok ? need : 0;
  dst_off[i] = !ok ? 0 : (p.state == 2 ? a.off_slots_c : (p.hs ? a.off_slots_hs : a.off_slots_sh)) + off;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int s = warp; s < a.batch; s += kPlanThreads / 32) {
    const int32_t* src = reinterpret_cast<const int32_t*>(src_ptr[s]);
    if (src == nullptr) continue;
    int32_t* dst = out + dst_off[s];
    for (int j = lane; j < cnt[s]; j += 32) dst[j] = src[j];
  }
}

}  // namespace

int step_plan_max_batch() { return kPlanThreads; }

cudaError_t launch_step_plan(const StepPlanArgs& a, cudaStream_t stream) {
  if (a.batch == 0) return cudaSuccess;
  return launch_pdl(step_plan_kernel, dim3(1), dim3(kPlanThreads), 0, stream, a);
}

}  // namespace dllm
