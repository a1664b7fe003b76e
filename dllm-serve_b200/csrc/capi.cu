// extern "C" entry points of libdllm_attn.so (declared in include/dllm_attn.h):
// argument validation, TMA tensor-map encoding and kernel dispatch.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "dllm_attn.h"
#include "attn_fwd.h"
#include "kvcache.h"
#include "select_kv.h"
#include "rope.h"
#include "step_plan.h"
#include "oproj_ar.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DLLM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// SM count per device, queried once (host threads racing on the first query
// store the same value).
int num_sms_of_current_device() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D map over [rows, heads, 128] bf16: dims (d, head, row), box (64,
// box_heads, box_rows), 128-byte swizzle (matches the UMMA SW128 K-major /
// MN-major smem layout: the box lands as box_rows * box_heads rows of 128 B,
// row r of head h at r * box_heads + h). Queries use 128-row boxes (or
// packed GQA boxes of 128 / m rows x m heads), keys/values 128-row boxes.
int encode_rows_map(CUtensorMap* m, const void* ptr, int64_t rows, int heads, int64_t tok_stride,
                    int box_rows, int box_heads = 1) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return fail(DLLM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)(rows > 0 ? rows : 1)};
  cuuint64_t strides[2] = {128 * 2, (cuuint64_t)tok_stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_heads, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DLLM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DLLM_OK;
}

// 2-D map over a row-major bf16 matrix [rows, cols] (row stride in elements):
// box (64 columns, box_rows rows), 128-byte swizzle (UMMA SW128 K-major).
int encode_matrix_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t row_stride,
                      int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return fail(DLLM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DLLM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DLLM_OK;
}

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn get_address_range_fn() {
  static std::atomic<GetAddressRangeFn> fn{nullptr};
  GetAddressRangeFn f = fn.load();
  if (f == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f = reinterpret_cast<GetAddressRangeFn>(p);
    fn.store(f);
  }
  return f;
}

int check_rows(const char* name, const void* p, int64_t tok_stride, int heads, int64_t rows) {
  if (rows > 0 && p == nullptr) return fail(DLLM_ERR_INVALID_ARG, "%s is null", name);
  if (!aligned(p, 16)) return fail(DLLM_ERR_ALIGNMENT, "%s is not 16-byte aligned", name);
  if (tok_stride < (int64_t)heads * 128)
    return fail(DLLM_ERR_INVALID_ARG, "%s token stride %lld < heads*head_dim", name,
                (long long)tok_stride);
  if (tok_stride % 8 != 0)
    return fail(DLLM_ERR_ALIGNMENT, "%s token stride %lld is not a multiple of 8 elements", name,
                (long long)tok_stride);
  if (rows < 0) return fail(DLLM_ERR_INVALID_ARG, "%s has negative rows", name);
  if (rows >= (int64_t)1 << 31) return fail(DLLM_ERR_TOO_LARGE, "%s has too many rows", name);
  return DLLM_OK;
}

// kc/vc are either row tensors of total_c rows (slots == nullptr) or paged
// caches of total_c = num_slots slots addressed through `slots` (cu_c then
// indexes the slot list).
int attn_common(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                const void* v, int64_t v_tok_stride, const void* kc, int64_t kc_tok_stride,
                const void* vc, int64_t vc_tok_stride, void* o, int64_t o_tok_stride,
                const int32_t* cu_q, const int32_t* cu_k, const int32_t* cu_c, int batch,
                int max_q, int64_t total_q, int64_t total_k, int64_t total_c, int Hq, int Hkv,
                int head_dim, float scale, int32_t* sched, int32_t* err, void* stream,
                const int32_t* slots = nullptr, const int64_t* positions = nullptr,
                const float* cos_sin = nullptr, int64_t max_position = 0,
                const int32_t* head_idx = nullptr, int n_heads = -1) {
  if (head_dim != 128)
    return fail(DLLM_ERR_UNSUPPORTED, "head_dim %d not supported (only 128)", head_dim);
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0)
    return fail(DLLM_ERR_UNSUPPORTED, "num_heads %d must be a positive multiple of num_kv_heads %d",
                Hq, Hkv);
  if (batch < 0 || max_q < 0 || total_q < 0 || total_k < 0 || total_c < 0)
    return fail(DLLM_ERR_INVALID_ARG, "negative size");
  if (!(scale > 0.f)) return fail(DLLM_ERR_INVALID_ARG, "softmax_scale must be > 0");
  if (!aligned(sched, 4)) return fail(DLLM_ERR_ALIGNMENT, "sched_workspace is not 4-byte aligned");
  if (positions != nullptr) {
    if (cos_sin == nullptr) return fail(DLLM_ERR_INVALID_ARG, "cos_sin_cache is null");
    if (!aligned(cos_sin, 16)) return fail(DLLM_ERR_ALIGNMENT, "cos_sin_cache must be 16-byte aligned");
    if (max_position < 0) return fail(DLLM_ERR_INVALID_ARG, "negative size");
    if (max_q > dllm::kSplitMaxQ)
      return fail(DLLM_ERR_UNSUPPORTED,
                  "on-chip rotary needs max_seqlen_q <= %d (got %d); rotate first, then attend",
                  dllm::kSplitMaxQ, max_q);
    if (total_q != total_k)
      return fail(DLLM_ERR_INVALID_ARG, "on-chip rotary needs total_q == total_k (one position per row)");
  }
  if (head_idx != nullptr) {
    if (n_heads < 0 || n_heads > Hq)
      return fail(DLLM_ERR_INVALID_ARG, "num_selected_heads %d outside [0, %d]", n_heads, Hq);
    if (!aligned(head_idx, 4)) return fail(DLLM_ERR_ALIGNMENT, "head_idx is not 4-byte aligned");
    if (positions != nullptr) return fail(DLLM_ERR_UNSUPPORTED, "a head list with on-chip rotary");
    if (n_heads == 0) return DLLM_OK;
  }
  if (batch == 0 || total_q == 0 || max_q == 0) return DLLM_OK;
  if (cu_q == nullptr || cu_k == nullptr) return fail(DLLM_ERR_INVALID_ARG, "cu_seqlens is null");
  int rc;
  if ((rc = check_rows("q", q, q_tok_stride, Hq, total_q)) != DLLM_OK) return rc;
  if ((rc = check_rows("o", o, o_tok_stride, Hq, total_q)) != DLLM_OK) return rc;
  if ((rc = check_rows("k", k, k_tok_stride, Hkv, total_k)) != DLLM_OK) return rc;
  if ((rc = check_rows("v", v, v_tok_stride, Hkv, total_k)) != DLLM_OK) return rc;
  if (cu_c != nullptr) {
    if ((rc = check_rows("k_cached", kc, kc_tok_stride, Hkv, total_c)) != DLLM_OK) return rc;
    if ((rc = check_rows("v_cached", vc, vc_tok_stride, Hkv, total_c)) != DLLM_OK) return rc;
    if (slots != nullptr && kc_tok_stride != vc_tok_stride)
      return fail(DLLM_ERR_INVALID_ARG, "k_cache and v_cache slot strides differ");
  }
  CUtensorMap tq, tk, tv, tkc, tvc;
  const int kv_rows = dllm::attn_fwd_kv_rows_per_tile();
  // GQA launches whose query segments are short (the reuse steps' blocks) pack
  // m query heads of a KV group into one 128-row tile of the split kernel.
  int qpack = 1;
  if (max_q <= dllm::kSplitMaxQ && head_idx == nullptr) {
    for (int m = 4; m >= 2; m >>= 1) {
      if (Hq / Hkv >= m && max_q <= 128 / m) {
        qpack = m;
        break;
      }
    }
  }
  if ((rc = encode_rows_map(&tq, q, total_q, Hq, q_tok_stride, 128 / qpack, qpack)) != DLLM_OK) return rc;
  if ((rc = encode_rows_map(&tk, k, total_k, Hkv, k_tok_stride, kv_rows)) != DLLM_OK) return rc;
  if ((rc = encode_rows_map(&tv, v, total_k, Hkv, v_tok_stride, kv_rows)) != DLLM_OK) return rc;
  if (cu_c != nullptr && total_c > 0) {
    if ((rc = encode_rows_map(&tkc, kc, total_c, Hkv, kc_tok_stride, kv_rows)) != DLLM_OK) return rc;
    if ((rc = encode_rows_map(&tvc, vc, total_c, Hkv, vc_tok_stride, kv_rows)) != DLLM_OK) return rc;
  } else {
    tkc = tk;
    tvc = tv;
    if (total_c == 0) cu_c = nullptr;
  }
  dllm::AttnKernelArgs a;
  a.o = reinterpret_cast<__nv_bfloat16*>(o);
  a.o_tok_stride = o_tok_stride;
  a.o_head_stride = 128;
  a.cu_q = cu_q;
  a.cu_k = cu_k;
  a.cu_c = cu_c;
  a.B = batch;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.group = Hq / Hkv;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = err;
  a.slots = slots;
  a.num_slots = slots != nullptr ? total_c : 0;
  a.kc = reinterpret_cast<const __nv_bfloat16*>(kc);
  a.vc = reinterpret_cast<const __nv_bfloat16*>(vc);
  a.c_tok_stride = kc_tok_stride;
  a.sched = sched;
  a.qpack = qpack;
  a.qunits = 0;
  a.total_units = 0;
  a.long_first = 0;
  a.positions = positions;
  a.cos_sin = cos_sin;
  a.max_position = max_position;
  a.head_idx = head_idx;
  a.n_heads = head_idx != nullptr ? n_heads : Hq;
  // Query segments that fit one tile (the reuse steps' fresh blocks) go to the
  // split kernel, which keeps both softmax warpgroups busy on a lone tile.
  const int sms = num_sms_of_current_device();
  cudaError_t e =
      max_q <= dllm::kSplitMaxQ
          ? dllm::launch_attn_fwd_split(tq, tk, tv, tkc, tvc, a, max_q, sms,
                                        reinterpret_cast<cudaStream_t>(stream))
          : dllm::launch_attn_fwd(tq, tk, tv, tkc, tvc, a, max_q, sms,
                                  reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd launch");
  return DLLM_OK;
}

int kv_copy_common(bool store, const void* key, int64_t key_stride, const void* value,
                   int64_t value_stride, const void* k_cache, const void* v_cache,
                   const int32_t* slots, int64_t n_tokens, int64_t row_elems, int elem_bytes,
                   int64_t num_slots, int32_t* err, void* stream) {
  if (n_tokens < 0 || row_elems <= 0 || num_slots < 0)
    return fail(DLLM_ERR_INVALID_ARG, "negative size");
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(DLLM_ERR_INVALID_ARG, "elem_bytes %d not in {1,2,4,8}", elem_bytes);
  if (n_tokens == 0) return DLLM_OK;
  if (!key || !value || !k_cache || !v_cache || !slots)
    return fail(DLLM_ERR_INVALID_ARG, "null pointer");
  if (key_stride < row_elems || value_stride < row_elems)
    return fail(DLLM_ERR_INVALID_ARG, "token stride smaller than the cache row");
  dllm::KvCopyArgs a;
  a.key = const_cast<void*>(key);
  a.value = const_cast<void*>(value);
  a.key_stride_bytes = key_stride * elem_bytes;
  a.value_stride_bytes = value_stride * elem_bytes;
  a.k_cache = const_cast<void*>(k_cache);
  a.v_cache = const_cast<void*>(v_cache);
  a.slots = slots;
  a.n_tokens = n_tokens;
  a.row_bytes = row_elems * elem_bytes;
  a.num_slots = num_slots;
  a.err = err;
  int vec = 16;
  auto fits = [&](int w) {
    return aligned(key, w) && aligned(value, w) && aligned(k_cache, w) && aligned(v_cache, w) &&
           a.key_stride_bytes % w == 0 && a.value_stride_bytes % w == 0 && a.row_bytes % w == 0;
  };
  while (vec > 1 && !fits(vec)) vec >>= 1;
  cudaError_t e = dllm::launch_kv_copy(a, store, vec, num_sms_of_current_device(),
                                       reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, store ? "store_kvcache launch" : "load_kvcache launch");
  return DLLM_OK;
}

// Scheduler workspace of dllm_attn_varlen_fwd_static_ws: file-scope device
// memory (one copy per device, zero when the module loads). The attention
// kernel uses the first DLLM_SCHED_WORKSPACE_INTS words and leaves them zero;
// each call also clears them on its stream before the launch.
constexpr int kStaticWsInts = 64;
static __device__ __align__(256) int32_t g_static_sched_ws[kStaticWsInts];

// Device address of g_static_sched_ws on the current device, looked up once
// per device (host threads racing on the first lookup store the same value);
// nullptr (and the CUDA error in *e) if the lookup fails. The address stays
// valid until the device's context is destroyed (cudaDeviceReset, process exit).
int32_t* static_sched_ws(int dev, cudaError_t* e) {
  static std::atomic<int32_t*> addr[64];
  *e = cudaSuccess;
  if (dev >= 0 && dev < 64) {
    int32_t* p = addr[dev].load(std::memory_order_acquire);
    if (p != nullptr) return p;
  }
  void* p = nullptr;
  *e = cudaGetSymbolAddress(&p, g_static_sched_ws);
  if (*e != cudaSuccess) return nullptr;
  if (dev >= 0 && dev < 64) addr[dev].store(static_cast<int32_t*>(p), std::memory_order_release);
  return static_cast<int32_t*>(p);
}

}  // namespace

extern "C" {

int dllm_version(void) { return 100; }

const char* dllm_last_error(void) { return g_last_error.c_str(); }

int dllm_store_kvcache(const void* key, int64_t key_stride, const void* value, int64_t value_stride,
                       void* k_cache, void* v_cache, const int32_t* slot_mapping, int64_t n_tokens,
                       int64_t row_elems, int elem_bytes, int64_t num_slots, int32_t* err_flag,
                       void* stream) {
  return kv_copy_common(true, key, key_stride, value, value_stride, k_cache, v_cache, slot_mapping,
                        n_tokens, row_elems, elem_bytes, num_slots, err_flag, stream);
}

int dllm_load_kvcache(void* key, int64_t key_stride, void* value, int64_t value_stride,
                      const void* k_cache, const void* v_cache, const int32_t* slot_mapping,
                      int64_t n_tokens, int64_t row_elems, int elem_bytes, int64_t num_slots,
                      int32_t* err_flag, void* stream) {
  return kv_copy_common(false, key, key_stride, value, value_stride, k_cache, v_cache,
                        slot_mapping, n_tokens, row_elems, elem_bytes, num_slots, err_flag, stream);
}

int dllm_attn_varlen_fwd(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                         const void* v, int64_t v_tok_stride, void* o, int64_t o_tok_stride,
                         const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int batch,
                         int max_seqlen_q, int64_t total_q, int64_t total_k, int num_heads,
                         int num_kv_heads, int head_dim, float softmax_scale,
                         int32_t* sched_workspace, int32_t* err_flag, void* stream) {
  return attn_common(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, nullptr, 0, nullptr, 0, o,
                     o_tok_stride, cu_seqlens_q, cu_seqlens_k, nullptr, batch, max_seqlen_q,
                     total_q, total_k, 0, num_heads, num_kv_heads, head_dim, softmax_scale,
                     sched_workspace, err_flag, stream);
}

int dllm_attn_varlen_fwd_static_ws(const void* q, int64_t q_tok_stride, const void* k,
                                   int64_t k_tok_stride, const void* v, int64_t v_tok_stride,
                                   void* o, int64_t o_tok_stride, const int32_t* cu_seqlens_q,
                                   const int32_t* cu_seqlens_k, int batch, int max_seqlen_q,
                                   int64_t total_q, int64_t total_k, int num_heads,
                                   int num_kv_heads, int head_dim, float softmax_scale,
                                   int32_t* err_flag, void* stream) {
  static_assert(DLLM_SCHED_WORKSPACE_INTS <= kStaticWsInts, "static workspace too small");
  if (DLLM_SCHED_WORKSPACE_INTS > kStaticWsInts)
    return fail(DLLM_ERR_TOO_LARGE, "scheduler workspace needs %d words > %d", DLLM_SCHED_WORKSPACE_INTS,
                kStaticWsInts);
  // The array lives on the current device; a stream of another device would
  // run the kernel there with this device's address.
  int dev = 0, stream_dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaStreamGetDevice(reinterpret_cast<cudaStream_t>(stream), &stream_dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamGetDevice");
  if (stream_dev != dev)
    return fail(DLLM_ERR_INVALID_ARG,
                "stream belongs to device %d but device %d is current; make the stream's device current",
                stream_dev, dev);
  int32_t* ws = static_sched_ws(dev, &e);
  if (ws == nullptr) return cuda_fail(e, "cudaGetSymbolAddress(static scheduler workspace)");
  // The words are shared by every call on this device and keep what the last
  // launch left (zero when it ran to its end); clear them on the stream so this
  // launch starts from zero whatever an earlier call did.
  e = cudaMemsetAsync(ws, 0, sizeof(int32_t) * DLLM_SCHED_WORKSPACE_INTS, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "clearing the static scheduler workspace");
  return attn_common(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, nullptr, 0, nullptr, 0, o,
                     o_tok_stride, cu_seqlens_q, cu_seqlens_k, nullptr, batch, max_seqlen_q,
                     total_q, total_k, 0, num_heads, num_kv_heads, head_dim, softmax_scale, ws,
                     err_flag, stream);
}

int dllm_attn_varlen_cached_fwd(const void* q, int64_t q_tok_stride, const void* k,
                                int64_t k_tok_stride, const void* v, int64_t v_tok_stride,
                                const void* kc, int64_t kc_tok_stride, const void* vc,
                                int64_t vc_tok_stride, void* o, int64_t o_tok_stride,
                                const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                                const int32_t* cu_seqlens_c, int batch, int max_seqlen_q,
                                int64_t total_q, int64_t total_k, int64_t total_c, int num_heads,
                                int num_kv_heads, int head_dim, float softmax_scale,
                                int32_t* sched_workspace, int32_t* err_flag, void* stream) {
  if (cu_seqlens_c == nullptr) return fail(DLLM_ERR_INVALID_ARG, "cu_seqlens_c is null");
  return attn_common(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, kc, kc_tok_stride, vc,
                     vc_tok_stride, o, o_tok_stride, cu_seqlens_q, cu_seqlens_k, cu_seqlens_c,
                     batch, max_seqlen_q, total_q, total_k, total_c, num_heads, num_kv_heads,
                     head_dim, softmax_scale, sched_workspace, err_flag, stream);
}

int dllm_attn_varlen_paged_fwd(const void* q, int64_t q_tok_stride, const void* k,
                               int64_t k_tok_stride, const void* v, int64_t v_tok_stride,
                               const void* k_cache, const void* v_cache, int64_t cache_tok_stride,
                               int64_t num_slots, const int32_t* slots,
                               const int32_t* cu_seqlens_slots, void* o, int64_t o_tok_stride,
                               const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int batch,
                               int max_seqlen_q, int64_t total_q, int64_t total_k, int num_heads,
                               int num_kv_heads, int head_dim, float softmax_scale,
                               int32_t* sched_workspace, int32_t* err_flag, void* stream) {
  if (cu_seqlens_slots == nullptr || slots == nullptr)
    return fail(DLLM_ERR_INVALID_ARG, "slots / cu_seqlens_slots is null");
  if (num_slots <= 0) return fail(DLLM_ERR_INVALID_ARG, "num_slots must be > 0");
  return attn_common(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, k_cache, cache_tok_stride,
                     v_cache, cache_tok_stride, o, o_tok_stride, cu_seqlens_q, cu_seqlens_k,
                     cu_seqlens_slots, batch, max_seqlen_q, total_q, total_k, num_slots, num_heads,
                     num_kv_heads, head_dim, softmax_scale, sched_workspace, err_flag, stream, slots);
}

int dllm_attn_varlen_rope_fwd(const int64_t* positions, const float* cos_sin_cache,
                              int64_t max_position, const void* q, int64_t q_tok_stride,
                              const void* k, int64_t k_tok_stride, const void* v,
                              int64_t v_tok_stride, const void* k_cache, const void* v_cache,
                              int64_t cache_tok_stride, int64_t num_slots, const int32_t* slots,
                              const int32_t* cu_seqlens_slots, void* o, int64_t o_tok_stride,
                              const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int batch,
                              int max_seqlen_q, int64_t total_q, int64_t total_k, int num_heads,
                              int num_kv_heads, int head_dim, float softmax_scale,
                              int32_t* err_flag, void* stream) {
  if (positions == nullptr) return fail(DLLM_ERR_INVALID_ARG, "positions is null");
  if ((slots == nullptr) != (cu_seqlens_slots == nullptr))
    return fail(DLLM_ERR_INVALID_ARG, "slots and cu_seqlens_slots must both be given or both be null");
  if (slots != nullptr && num_slots <= 0) return fail(DLLM_ERR_INVALID_ARG, "num_slots must be > 0");
  return attn_common(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, k_cache, cache_tok_stride,
                     v_cache, cache_tok_stride, o, o_tok_stride, cu_seqlens_q, cu_seqlens_k,
                     cu_seqlens_slots, batch, max_seqlen_q, total_q, total_k,
                     slots != nullptr ? num_slots : 0, num_heads, num_kv_heads, head_dim,
                     softmax_scale, nullptr, err_flag, stream, slots, positions, cos_sin_cache,
                     max_position);
}

int dllm_attn_varlen_heads_fwd(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                               const void* v, int64_t v_tok_stride, const void* k_cache,
                               const void* v_cache, int64_t cache_tok_stride, int64_t num_slots,
                               const int32_t* slots, const int32_t* cu_seqlens_slots, void* o,
                               int64_t o_tok_stride, const int32_t* cu_seqlens_q,
                               const int32_t* cu_seqlens_k, int batch, int max_seqlen_q, int64_t total_q,
                               int64_t total_k, int num_heads, int num_kv_heads, int head_dim,
                               float softmax_scale, const int32_t* head_idx, int num_selected_heads,
                               int32_t* sched_workspace, int32_t* err_flag, void* stream) {
  if (head_idx == nullptr && num_selected_heads > 0) return fail(DLLM_ERR_INVALID_ARG, "head_idx is null");
  if ((slots == nullptr) != (cu_seqlens_slots == nullptr))
    return fail(DLLM_ERR_INVALID_ARG, "slots and cu_seqlens_slots must both be given or both be null");
  if (slots != nullptr && num_slots <= 0) return fail(DLLM_ERR_INVALID_ARG, "num_slots must be > 0");
  if (num_selected_heads == 0) return DLLM_OK;
  return attn_common(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, k_cache, cache_tok_stride,
                     v_cache, cache_tok_stride, o, o_tok_stride, cu_seqlens_q, cu_seqlens_k,
                     cu_seqlens_slots, batch, max_seqlen_q, total_q, total_k,
                     slots != nullptr ? num_slots : 0, num_heads, num_kv_heads, head_dim,
                     softmax_scale, sched_workspace, err_flag, stream, slots, nullptr, nullptr, 0,
                     head_idx, num_selected_heads);
}

int dllm_rope_neox(const int64_t* positions, const void* q_in, int64_t q_in_stride, void* q_out,
                   int64_t q_out_stride, const void* k_in, int64_t k_in_stride, void* k_out,
                   int64_t k_out_stride, const float* cos_sin_cache, int64_t max_position,
                   int64_t n_tokens, int num_heads, int num_kv_heads, int head_dim,
                   int32_t* err_flag, void* stream) {
  if (head_dim != 128)
    return fail(DLLM_ERR_UNSUPPORTED, "head_dim %d not supported (only 128)", head_dim);
  if (n_tokens < 0 || num_heads < 0 || num_kv_heads < 0 || max_position < 0)
    return fail(DLLM_ERR_INVALID_ARG, "negative size");
  if (n_tokens == 0 || num_heads + num_kv_heads == 0) return DLLM_OK;
  if (positions == nullptr || cos_sin_cache == nullptr)
    return fail(DLLM_ERR_INVALID_ARG, "positions / cos_sin_cache is null");
  if ((reinterpret_cast<uintptr_t>(cos_sin_cache) & 15) != 0)
    return fail(DLLM_ERR_ALIGNMENT, "cos_sin_cache must be 16-byte aligned");
  int rc;
  if (num_heads > 0) {
    if ((rc = check_rows("q_in", q_in, q_in_stride, num_heads, n_tokens)) != DLLM_OK) return rc;
    if ((rc = check_rows("q_out", q_out, q_out_stride, num_heads, n_tokens)) != DLLM_OK) return rc;
  }
  if (num_kv_heads > 0) {
    if ((rc = check_rows("k_in", k_in, k_in_stride, num_kv_heads, n_tokens)) != DLLM_OK) return rc;
    if ((rc = check_rows("k_out", k_out, k_out_stride, num_kv_heads, n_tokens)) != DLLM_OK) return rc;
  }
  dllm::RopeArgs a;
  a.positions = positions;
  a.q_in = reinterpret_cast<const __nv_bfloat16*>(q_in);
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out);
  a.k_in = reinterpret_cast<const __nv_bfloat16*>(k_in);
  a.k_out = reinterpret_cast<__nv_bfloat16*>(k_out);
  a.q_in_stride = q_in_stride;
  a.q_out_stride = q_out_stride;
  a.k_in_stride = k_in_stride;
  a.k_out_stride = k_out_stride;
  a.cos_sin = cos_sin_cache;
  a.max_position = max_position;
  a.n_tokens = n_tokens;
  a.Hq = num_heads;
  a.Hkv = num_kv_heads;
  a.err = err_flag;
  cudaError_t e = dllm::launch_rope(a, num_sms_of_current_device(), reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  return DLLM_OK;
}

int dllm_select_kv_store(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                         const void* v, int64_t v_tok_stride, const int32_t* seq_desc, int n_seqs,
                         int max_klen, int num_heads, int num_kv_heads, int head_dim,
                         int head_select, void* k_cache, void* v_cache, int64_t cache_tok_stride,
                         int64_t num_slots, const int32_t* slots, int64_t* top_idx,
                         int32_t* err_flag, void* stream) {
  if (head_dim != 128)
    return fail(DLLM_ERR_UNSUPPORTED, "head_dim %d not supported (only 128)", head_dim);
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return fail(DLLM_ERR_UNSUPPORTED, "num_heads must be a positive multiple of num_kv_heads");
  if (n_seqs < 0 || max_klen < 0) return fail(DLLM_ERR_INVALID_ARG, "negative size");
  if (max_klen > 16384) return fail(DLLM_ERR_TOO_LARGE, "max_klen %d > 16384", max_klen);
  if (n_seqs == 0 || max_klen == 0) return DLLM_OK;
  if (!q || !k || !v || !seq_desc || !k_cache || !v_cache || !slots)
    return fail(DLLM_ERR_INVALID_ARG, "null pointer");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(k_cache, 16) ||
      !aligned(v_cache, 16) || q_tok_stride % 8 || k_tok_stride % 8 || v_tok_stride % 8 ||
      cache_tok_stride % 8)
    return fail(DLLM_ERR_ALIGNMENT, "q/k/v/cache must be 16-byte aligned with strides %% 8 == 0");
  if (cache_tok_stride < (int64_t)num_kv_heads * 128)
    return fail(DLLM_ERR_INVALID_ARG, "cache_tok_stride smaller than num_kv_heads*head_dim");
  dllm::SelectArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k = reinterpret_cast<const __nv_bfloat16*>(k);
  a.v = reinterpret_cast<const __nv_bfloat16*>(v);
  a.q_tok_stride = q_tok_stride;
  a.k_tok_stride = k_tok_stride;
  a.v_tok_stride = v_tok_stride;
  a.seq_desc = seq_desc;
  a.max_klen = max_klen;
  a.Hq = num_heads;
  a.Hkv = num_kv_heads;
  a.group = num_heads / num_kv_heads;
  a.sqrt_d = (float)sqrt((double)head_dim);
  a.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache);
  a.cache_tok_stride = cache_tok_stride;
  a.num_slots = num_slots;
  a.slots = slots;
  a.top_idx = top_idx;
  a.err = err_flag;
  const size_t smem = dllm::select_kv_smem_bytes(head_select ? a.group : a.Hq, max_klen);
  if (smem > 227 * 1024) return fail(DLLM_ERR_TOO_LARGE, "select_kv needs %zu B smem", smem);
  cudaError_t e = dllm::launch_select_kv(a, head_select != 0, n_seqs,
                                         reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "select_kv launch");
  return DLLM_OK;
}

int dllm_build_step_plan(const int64_t* seqs, int batch, int num_kv_heads, int32_t* out,
                         const int64_t* layout, int32_t* err_flag, void* stream) {
  static_assert(DLLM_PLAN_SEQ_FIELDS == dllm::kPlanSeqFields, "plan row layout");
  static_assert(DLLM_SEQ_DESC_INTS == dllm::kPlanDescInts, "descriptor layout");
  if (batch < 0 || num_kv_heads <= 0) return fail(DLLM_ERR_INVALID_ARG, "negative batch or num_kv_heads <= 0");
  if (batch > dllm::step_plan_max_batch() || batch > DLLM_PLAN_MAX_BATCH)
    return fail(DLLM_ERR_TOO_LARGE, "batch %d > %d", batch, DLLM_PLAN_MAX_BATCH);
  if (batch == 0) return DLLM_OK;
  if (seqs == nullptr || out == nullptr || layout == nullptr) return fail(DLLM_ERR_INVALID_ARG, "null pointer");
  if (!aligned(seqs, 8) || !aligned(out, 4)) return fail(DLLM_ERR_ALIGNMENT, "seqs / out misaligned");
  // sections in order, inside the buffer: cu | cu_c | desc_hs | desc_sh | slots_c | slots_hs | slots_sh
  const int64_t total = layout[0];
  const int64_t sec[6][2] = {{layout[1], batch + 1},
                             {layout[2], layout[3] * DLLM_SEQ_DESC_INTS},
                             {layout[4], layout[5] * DLLM_SEQ_DESC_INTS},
                             {layout[6], layout[7]},
                             {layout[8], layout[9]},
                             {layout[10], layout[11]}};
  int64_t end = batch + 1;
  for (int i = 0; i < 6; ++i) {
    if (sec[i][1] < 0 || sec[i][0] < end) return fail(DLLM_ERR_INVALID_ARG, "plan layout section %d overlaps", i);
    end = sec[i][0] + sec[i][1];
  }
  if (end > total || total >= ((int64_t)1 << 31)) return fail(DLLM_ERR_INVALID_ARG, "plan layout exceeds the buffer");
  dllm::StepPlanArgs a;
  a.seqs = seqs;
  a.batch = batch;
  a.num_kv_heads = num_kv_heads;
  a.out = out;
  a.off_cu_c = (int)layout[1];
  a.off_desc_hs = (int)layout[2];
  a.cap_desc_hs = (int)layout[3];
  a.off_desc_sh = (int)layout[4];
  a.cap_desc_sh = (int)layout[5];
  a.off_slots_c = (int)layout[6];
  a.cap_slots_c = (int)layout[7];
  a.off_slots_hs = (int)layout[8];
  a.cap_slots_hs = (int)layout[9];
  a.off_slots_sh = (int)layout[10];
  a.cap_slots_sh = (int)layout[11];
  a.err = err_flag;
  cudaError_t e = dllm::launch_step_plan(a, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "step plan launch");
  return DLLM_OK;
}

int dllm_oproj_allreduce(const void* x, int64_t x_stride, const void* w, int64_t w_stride, int M, int N,
                         int K, void* const* recv, void* const* y, int32_t* const* flags, int rank,
                         int tp, int epoch, int32_t* err_flag, void* stream) {
  if (tp < 1 || tp > DLLM_OPROJ_MAX_RANKS || rank < 0 || rank >= tp)
    return fail(DLLM_ERR_INVALID_ARG, "rank %d / tp %d (tp must be 1..%d)", rank, tp, DLLM_OPROJ_MAX_RANKS);
  if (M < 0 || N <= 0 || K <= 0) return fail(DLLM_ERR_INVALID_ARG, "bad sizes M=%d N=%d K=%d", M, N, K);
  if (N % 256 != 0 || K % 64 != 0)
    return fail(DLLM_ERR_UNSUPPORTED, "N %% 256 == 0 and K %% 64 == 0 required (N=%d K=%d)", N, K);
  if (epoch == 0) return fail(DLLM_ERR_INVALID_ARG, "epoch must be nonzero (flags start at 0)");
  if (M == 0) return DLLM_OK;
  if (!x || !w || !recv || !y || !flags) return fail(DLLM_ERR_INVALID_ARG, "null pointer");
  if (!aligned(x, 16) || !aligned(w, 16) || x_stride % 8 || w_stride % 8 || x_stride < K || w_stride < K)
    return fail(DLLM_ERR_ALIGNMENT, "x / w must be 16-byte aligned with row strides %% 8 == 0 and >= K");
  dllm::OprojArArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.rank = rank;
  a.tp = tp;
  a.epoch = epoch;
  a.tiles_m = (M + 127) / 128;
  a.tiles_n = N / 256;
  const int64_t tiles = (int64_t)a.tiles_m * a.tiles_n;
  if (tiles >= ((int64_t)1 << 30)) return fail(DLLM_ERR_TOO_LARGE, "too many tiles");
  a.num_tiles = (int)tiles;
  for (int p = 0; p < tp; ++p) {
    if (!recv[p] || !y[p] || !flags[p]) return fail(DLLM_ERR_INVALID_ARG, "null buffer of rank %d", p);
    if (!aligned(recv[p], 16) || !aligned(y[p], 16) || !aligned(flags[p], 4))
      return fail(DLLM_ERR_ALIGNMENT, "buffers of rank %d misaligned", p);
    a.recv[p] = reinterpret_cast<__nv_bfloat16*>(recv[p]);
    a.y[p] = reinterpret_cast<__nv_bfloat16*>(y[p]);
    a.flags[p] = flags[p];
  }
  a.err = err_flag;
  CUtensorMap tmA, tmB;
  int rc;
  if ((rc = encode_matrix_map(&tmA, x, M, K, x_stride, 128)) != DLLM_OK) return rc;
  if ((rc = encode_matrix_map(&tmB, w, N, K, w_stride, 256)) != DLLM_OK) return rc;
  cudaError_t e = dllm::launch_oproj_ar(tmA, tmB, a, num_sms_of_current_device(),
                                        reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "oproj_allreduce launch");
  return DLLM_OK;
}

int dllm_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return fail(DLLM_ERR_INVALID_ARG, "null pointer");
  GetAddressRangeFn range = get_address_range_fn();
  if (range == nullptr) return fail(DLLM_ERR_CUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr b = 0;
  size_t size = 0;
  CUresult r = range(&b, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(DLLM_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(b));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) <= DLLM_IPC_HANDLE_BYTES, "handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - b);
  return DLLM_OK;
}

int dllm_ipc_open(const void* handle, void** base) {
  if (handle == nullptr || base == nullptr) return fail(DLLM_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return DLLM_OK;
}

int dllm_ipc_close(void* base) {
  if (base == nullptr) return DLLM_OK;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return DLLM_OK;
}

}  // extern "C"
