/*
 * dllm_attn.h - C ABI of the B200 (sm_100a) attention-path library
 * (libdllm_attn.so) for diffusion-LLM serving.
 *
 * Each entry point replaces one piece of the reference's per-denoising-step
 * attention path (chosen-ox/dLLM-Serve, dllmserve/layers/attention.py):
 *
 *   dllm_store_kvcache        <- store_kvcache + store_kvcache_kernel   (attention.py:11-50)
 *   dllm_load_kvcache         <- load_kvcache + load_kvcache_kernel     (attention.py:53-92)
 *   dllm_attn_varlen_fwd      <- flash_attn_varlen_func(..., causal=False) (attention.py:289-299)
 *   dllm_attn_varlen_fwd_static_ws
 *                             (no reference counterpart) dllm_attn_varlen_fwd for callers
 *                                that cannot allocate device memory: its scheduler workspace
 *                                is a small array inside the library (see its declaration)
 *   dllm_attn_varlen_cached_fwd
 *                             <- reuse-state K/V assembly + varlen call (attention.py:235-299):
 *                                keys are [cached selected rows ; fresh block rows]
 *   dllm_attn_varlen_paged_fwd
 *                             <- the same with the cached rows read from the paged cache by
 *                                slot (load_kvcache fused in, attention.py:241-263)
 *   dllm_attn_varlen_rope_fwd <- RotaryEmbedding.forward (rotary_embedding.py:41-57) on q and
 *                                the fresh k, fused into the attention of a launch whose
 *                                query segments fit one 128-row tile (the reuse steps'
 *                                blocks): llada.py:81-84 / dream.py:90-93 in one call
 *   dllm_rope_neox            <- RotaryEmbedding.forward / apply_rotary_emb
 *                                (dllmserve/layers/rotary_embedding.py:6-16, 41-57), the
 *                                op the decoder layers apply to q, k just before attention
 *   dllm_attn_varlen_heads_fwd  attention for a list of query heads only (no reference
 *                                counterpart: the head-level form of the sparse path)
 *   dllm_oproj_allreduce      <- RowParallelLinear.forward: F.linear + dist.all_reduce
 *                                (linear.py:186-190), one kernel over NVLink peer memory
 *   dllm_build_step_plan      <- the per-sequence metadata of attention.py:168-304 /
 *                                model_runner.py:240-321, on the device
 *   dllm_select_kv_store      <- _select_important_head_kv (attention.py:344-413) or
 *                                _select_important_kv (attention.py:308-342), followed by
 *                                the k_prefix_suffix[idx] gather and store_kvcache of the
 *                                selected rows (attention.py:204-233)
 *
 * Conventions
 *   - Every pointer except `err_flag`/`top_idx` arguments documented as optional is a
 *     device pointer owned by the caller. The library never allocates or frees memory,
 *     never synchronises the stream and never reads device data on the host, so a call
 *     of any entry point that works only on caller buffers can be captured in a CUDA
 *     graph (this statement does not cover dllm_attn_varlen_fwd_static_ws, whose
 *     workspace is a library array).
 *   - `stream` is a cudaStream_t passed as void*. NULL means the legacy default stream.
 *   - Strides are in ELEMENTS unless the name ends in `_bytes`.
 *   - bf16 tensors are laid out [tokens, heads, head_dim] with head_dim contiguous and
 *     heads packed (head stride == head_dim); the token stride is free (views of a fused
 *     qkv projection are accepted) but must be a multiple of 8 elements.
 *   - Return value: DLLM_OK or one of the DLLM_ERR_* codes; dllm_last_error() gives a
 *     one-line message for the calling thread.
 *   - `err_flag` (optional, int32 device word) receives a device-side status: the first
 *     nonzero DLLM_DEV_* code seen by any kernel thread. The caller clears and reads it.
 *   - `sched_workspace` (optional, attention entry points): DLLM_SCHED_WORKSPACE_INTS int32
 *     device words, zero before their first use. With it, launches whose query segments
 *     exceed 128 rows hand out their work units dynamically (an atomic counter) instead of
 *     round-robin, which evens out batches of unequal lengths; the kernel returns the words
 *     to zero when it exits. Launches that may run at the same time (other streams) need
 *     distinct workspaces. NULL: round-robin order (same results, bit for bit).
 */
#ifndef DLLM_ATTN_H_
#define DLLM_ATTN_H_

#include <stdint.h>

#if defined(__GNUC__)
#define DLLM_API __attribute__((visibility("default")))
#else
#define DLLM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* host-side return codes */
#define DLLM_OK 0
#define DLLM_ERR_INVALID_ARG 1   /* null pointer, negative size, inconsistent sizes */
#define DLLM_ERR_UNSUPPORTED 2   /* head_dim / head ratio not supported */
#define DLLM_ERR_ALIGNMENT 3     /* pointer or stride not aligned for vector/TMA access */
#define DLLM_ERR_TOO_LARGE 4     /* a size beyond the kernel's limit */
#define DLLM_ERR_CUDA 5          /* CUDA launch / driver error */

/* int32 words of an attention scheduler workspace */
#define DLLM_SCHED_WORKSPACE_INTS 2

/* device-side status codes written to err_flag */
#define DLLM_DEV_SLOT_OUT_OF_RANGE 1
#define DLLM_DEV_WAIT_TIMEOUT 2
#define DLLM_DEV_BAD_SEQUENCE 3
#define DLLM_DEV_POSITION_OUT_OF_RANGE 4

/* Library version (major*10000 + minor*100 + patch). */
DLLM_API int dllm_version(void);

/* Message describing the last failing call on this thread ("" if none). */
DLLM_API const char* dllm_last_error(void);

/*
 * cache[slot_mapping[i]] <- key[i], value[i]  for i in [0, n_tokens)
 * Replaces store_kvcache (attention.py:33-50) and its Triton kernel (:11-30).
 * A cache row (one slot) holds `row_elems` contiguous elements (= num_kv_heads*head_dim),
 * `elem_bytes` wide. key/value row i starts at key + i*key_stride elements.
 * Slots < 0 are skipped; slots >= num_slots are skipped and flag
 * DLLM_DEV_SLOT_OUT_OF_RANGE in err_flag.
 */
DLLM_API int dllm_store_kvcache(const void* key, int64_t key_stride, const void* value,
                       int64_t value_stride, void* k_cache, void* v_cache,
                       const int32_t* slot_mapping, int64_t n_tokens, int64_t row_elems,
                       int elem_bytes, int64_t num_slots, int32_t* err_flag, void* stream);

/*
 * key[i], value[i] <- cache[slot_mapping[i]]  for i in [0, n_tokens)
 * Replaces load_kvcache (attention.py:77-92) and its Triton kernel (:53-74).
 * Out-of-range slots produce zero rows (negative: silently; >= num_slots: also flag).
 */
DLLM_API int dllm_load_kvcache(void* key, int64_t key_stride, void* value, int64_t value_stride,
                      const void* k_cache, const void* v_cache, const int32_t* slot_mapping,
                      int64_t n_tokens, int64_t row_elems, int elem_bytes, int64_t num_slots,
                      int32_t* err_flag, void* stream);

/*
 * Non-causal varlen attention, bf16 in/out, fp32 accumulation:
 *   o[q rows of seq b] = softmax(Q_b K_b^T * softmax_scale) V_b
 * Replaces flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
 * max_seqlen_k, softmax_scale, causal=False) as called at attention.py:289-299.
 * q: [total_q, num_heads, head_dim]; k, v: [total_k, num_kv_heads, head_dim];
 * o: [total_q, num_heads, head_dim]. cu_seqlens_*: int32 [batch+1], device.
 * max_seqlen_q must be >= every query length (it sizes the grid). GQA when
 * num_heads is a multiple of num_kv_heads. head_dim must be 128.
 */
DLLM_API int dllm_attn_varlen_fwd(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                         const void* v, int64_t v_tok_stride, void* o, int64_t o_tok_stride,
                         const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int batch,
                         int max_seqlen_q, int64_t total_q, int64_t total_k, int num_heads,
                         int num_kv_heads, int head_dim, float softmax_scale,
                         int32_t* sched_workspace, int32_t* err_flag, void* stream);

/*
 * dllm_attn_varlen_fwd for callers that cannot allocate device memory. It
 * allocates nothing: the scheduler workspace that dllm_attn_varlen_fwd takes
 * from the caller lives instead in a file-scope static device array of the
 * library, 64 int32 words per device (every device that loads the library
 * holds it until the process exits; the call uses the first
 * DLLM_SCHED_WORKSPACE_INTS words and returns DLLM_ERR_TOO_LARGE if a
 * workspace would not fit). Typical callers: a plugin whose host application
 * owns all device memory through its own pool and hands it only input/output
 * pointers, and launch loops that must not call cudaMalloc, which can
 * synchronise the device and would stall the stream they are feeding.
 * The caller still passes every input and output.
 *
 * Set-up: the first call on a device (with that device current) looks up the
 * array's device address with cudaGetSymbolAddress and keeps it for later
 * calls; make that first call before any stream capture. The kept address
 * belongs to the device's current context: after cudaDeviceReset on that
 * device, do not call this entry point again in the same process. The stream must
 * belong to the current device (DLLM_ERR_INVALID_ARG otherwise). Each call
 * clears the words it uses on its stream (cudaMemsetAsync, no allocation)
 * before the launch, so it starts from zero whatever an earlier call left;
 * calls that overlap in time on one device (several streams or host threads)
 * share the words and race: run them one after another.
 * No counterpart in the reference (its flash_attn_varlen_func takes no
 * workspace).
 */
DLLM_API int dllm_attn_varlen_fwd_static_ws(const void* q, int64_t q_tok_stride, const void* k,
                                   int64_t k_tok_stride, const void* v, int64_t v_tok_stride,
                                   void* o, int64_t o_tok_stride, const int32_t* cu_seqlens_q,
                                   const int32_t* cu_seqlens_k, int batch, int max_seqlen_q,
                                   int64_t total_q, int64_t total_k, int num_heads,
                                   int num_kv_heads, int head_dim, float softmax_scale,
                                   int32_t* err_flag, void* stream);

/*
 * As dllm_attn_varlen_fwd, but the keys/values of sequence b are the
 * concatenation [cached rows cu_seqlens_c[b]..cu_seqlens_c[b+1] of kc/vc ;
 * fresh rows cu_seqlens_k[b]..cu_seqlens_k[b+1] of k/v], without materialising
 * the concatenation. Replaces the reuse-state assembly of attention.py:235-265
 * (zeros + load_kvcache + torch.cat) feeding the varlen call at :289-299.
 * kc, vc: [total_c, num_kv_heads, head_dim] with token strides kc_tok_stride/vc_tok_stride.
 */
DLLM_API int dllm_attn_varlen_cached_fwd(const void* q, int64_t q_tok_stride, const void* k,
                                int64_t k_tok_stride, const void* v, int64_t v_tok_stride,
                                const void* kc, int64_t kc_tok_stride, const void* vc,
                                int64_t vc_tok_stride, void* o, int64_t o_tok_stride,
                                const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                                const int32_t* cu_seqlens_c, int batch, int max_seqlen_q,
                                int64_t total_q, int64_t total_k, int64_t total_c,
                                int num_heads, int num_kv_heads, int head_dim,
                                float softmax_scale, int32_t* sched_workspace, int32_t* err_flag,
                                void* stream);

/*
 * As dllm_attn_varlen_cached_fwd, but the cached keys/values of sequence b are read
 * straight from the paged KV cache: rows slots[cu_seqlens_slots[b] .. cu_seqlens_slots[b+1])
 * of k_cache / v_cache (num_slots slots, cache_tok_stride elements apart, the layout of
 * model_runner.py:192-206). Replaces zeros + load_kvcache + torch.cat of the reuse state
 * (attention.py:241-263) and the varlen call (:289-299) with one launch. Runs of 128
 * consecutive slots (the runner's 256-token pages) are copied with TMA; other slot lists are
 * gathered row by row. Slots outside [0, num_slots) read as zero rows and flag
 * DLLM_DEV_SLOT_OUT_OF_RANGE. Cache rows must hold finite values (the reference allocates
 * the cache with torch.zeros).
 */
DLLM_API int dllm_attn_varlen_paged_fwd(const void* q, int64_t q_tok_stride, const void* k,
                               int64_t k_tok_stride, const void* v, int64_t v_tok_stride,
                               const void* k_cache, const void* v_cache, int64_t cache_tok_stride,
                               int64_t num_slots, const int32_t* slots,
                               const int32_t* cu_seqlens_slots, void* o, int64_t o_tok_stride,
                               const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int batch,
                               int max_seqlen_q, int64_t total_q, int64_t total_k, int num_heads,
                               int num_kv_heads, int head_dim, float softmax_scale,
                               int32_t* sched_workspace, int32_t* err_flag, void* stream);

/*
 * Rotary embedding fused into attention: the result equals dllm_rope_neox(positions, q, k)
 * followed by dllm_attn_varlen_paged_fwd (or dllm_attn_varlen_fwd when slots is NULL) on the
 * rotated q and k, bit for bit, but q and k are never rewritten: each query tile and each
 * fresh key tile is rotated in shared memory between its load and the matrix multiply that
 * reads it. Replaces the decoder layers' `q, k = self.rotary_emb(positions, q, k)` followed
 * by `self.attn(q, k, v)` (llada.py:81-84, dream.py:90-93) for the diffusion reuse steps.
 * positions: int64 [total_q], the position of query row r and of fresh key row r (so
 * total_k must equal total_q). cos_sin_cache: fp32 [max_position, 128], cos | sin halves,
 * 16-byte aligned. Cached rows (k_cache/v_cache through slots/cu_seqlens_slots, both NULL
 * for none) are taken as already rotated, as store_kvcache wrote them. max_seqlen_q must be
 * <= 128 (DLLM_ERR_UNSUPPORTED otherwise: rotate with dllm_rope_neox, then attend).
 * Positions outside [0, max_position) give zero rows and flag
 * DLLM_DEV_POSITION_OUT_OF_RANGE. No scheduler workspace (units are handed out round-robin).
 */
DLLM_API int dllm_attn_varlen_rope_fwd(const int64_t* positions, const float* cos_sin_cache,
                                       int64_t max_position, const void* q, int64_t q_tok_stride,
                                       const void* k, int64_t k_tok_stride, const void* v,
                                       int64_t v_tok_stride, const void* k_cache,
                                       const void* v_cache, int64_t cache_tok_stride,
                                       int64_t num_slots, const int32_t* slots,
                                       const int32_t* cu_seqlens_slots, void* o,
                                       int64_t o_tok_stride, const int32_t* cu_seqlens_q,
                                       const int32_t* cu_seqlens_k, int batch, int max_seqlen_q,
                                       int64_t total_q, int64_t total_k, int num_heads,
                                       int num_kv_heads, int head_dim, float softmax_scale,
                                       int32_t* err_flag, void* stream);

/*
 * NeoX rotary embedding of q and k (RotaryEmbedding.forward, rotary_embedding.py:41-57,
 * with apply_rotary_emb :6-16): for token t at position p = positions[t], every head row
 * x (head_dim 128, bf16) becomes [x1*cos - x2*sin, x2*cos + x1*sin] where x1, x2 are its
 * halves in fp32 and cos, sin the halves of cos_sin_cache[p] (fp32 [max_position, 128],
 * cos | sin, as the reference builds it). Products and sums are rounded separately, so
 * the result equals the reference's bit for bit. q_in/q_out: [n_tokens, num_heads, 128],
 * k_in/k_out: [n_tokens, num_kv_heads, 128], token strides in elements (multiples of 8);
 * out may equal in (in place). Positions outside [0, max_position) give zero rows and
 * flag DLLM_DEV_POSITION_OUT_OF_RANGE.
 */
DLLM_API int dllm_rope_neox(const int64_t* positions, const void* q_in, int64_t q_in_stride,
                            void* q_out, int64_t q_out_stride, const void* k_in,
                            int64_t k_in_stride, void* k_out, int64_t k_out_stride,
                            const float* cos_sin_cache, int64_t max_position, int64_t n_tokens,
                            int num_heads, int num_kv_heads, int head_dim, int32_t* err_flag,
                            void* stream);

/*
 * Per-sequence descriptor for dllm_select_kv_store: 8 int32 values per sequence.
 *   [0] tok_start   row of the sequence's first token in q/k/v
 *   [1] seq_len     tokens of the sequence in q/k/v (L)
 *   [2] blk_start   start of the current diffusion block, relative to tok_start
 *   [3] blk_len     tokens in the block; candidates are the other L-blk_len tokens
 *   [4] n_keep      rows to keep: min(max(1, int(Klen*retention_ratio)), Klen), 0 if Klen==0
 *   [5] slot_off    offset of this sequence's n_keep slots in `slots`
 *   [6] idx_off     offset of this sequence's indices in `top_idx` (elements)
 *   [7] pool_kernel max-pool window over candidate scores (<=1: none)
 */
#define DLLM_SEQ_DESC_INTS 8

/*
 * Importance scoring + top-k selection + gather + KV-cache store, for every
 * sequence of the step that is in the "compute cache" state.
 *   q_avg[h]   = mean of the block's query rows (fp32)
 *   head_select != 0 (attention.py:344-413): per KV head h,
 *       s[h,c] = max over the head's query group g of q_avg[g].k[c,h] / sqrt(head_dim)
 *     else (attention.py:308-342): one shared ranking,
 *       s[c]   = sum over all query heads g of q_avg[g].k[c, g/group] / sqrt(head_dim)
 *   s <- max_pool1d(s, pool_kernel, stride 1, padding pool_kernel/2)[:Klen]
 *   idx = the n_keep largest scores, ordered by descending score, ties by ascending
 *         candidate index
 *   k_cache[slots[j]] (head h, or all heads) <- k[candidate idx[j]], same for v.
 * Candidates are the sequence's tokens outside [blk_start, blk_start+blk_len), in order.
 * top_idx (optional, int64, device): per sequence [num_kv_heads, n_keep] (head_select)
 * or [n_keep] at idx_off. max_klen must be >= every Klen and <= 16384.
 * `cache_tok_stride` is the element stride between cache slots (num_kv_heads*head_dim
 * for the reference layout).
 */
DLLM_API int dllm_select_kv_store(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                         const void* v, int64_t v_tok_stride, const int32_t* seq_desc,
                         int n_seqs, int max_klen, int num_heads, int num_kv_heads, int head_dim,
                         int head_select, void* k_cache, void* v_cache, int64_t cache_tok_stride,
                         int64_t num_slots, const int32_t* slots, int64_t* top_idx,
                         int32_t* err_flag, void* stream);

/*
 * Head-compacted attention: dllm_attn_varlen_fwd (or, with k_cache/v_cache/slots/
 * cu_seqlens_slots, dllm_attn_varlen_paged_fwd) computed only for the query heads
 * head_idx[0 .. num_selected_heads) (device int32, each in [0, num_heads); with GQA the
 * KV head of query head h is h / (num_heads / num_kv_heads)). Work units are numbered
 * over the list, so heads left out cost nothing; their output rows are not written.
 * An index outside [0, num_heads) sets DLLM_DEV_BAD_SEQUENCE in err_flag and its units
 * are skipped. The slots / cu_seqlens_slots pair is optional (both null: no cached
 * segment). No counterpart in the reference, which keeps every head and selects tokens
 * per KV head (attention.py:344-413); this is the head-level form of the sparse path.
 */
DLLM_API int dllm_attn_varlen_heads_fwd(const void* q, int64_t q_tok_stride, const void* k,
                                        int64_t k_tok_stride, const void* v, int64_t v_tok_stride,
                                        const void* k_cache, const void* v_cache,
                                        int64_t cache_tok_stride, int64_t num_slots,
                                        const int32_t* slots, const int32_t* cu_seqlens_slots, void* o,
                                        int64_t o_tok_stride, const int32_t* cu_seqlens_q,
                                        const int32_t* cu_seqlens_k, int batch, int max_seqlen_q,
                                        int64_t total_q, int64_t total_k, int num_heads, int num_kv_heads,
                                        int head_dim, float softmax_scale, const int32_t* head_idx,
                                        int num_selected_heads, int32_t* sched_workspace, int32_t* err_flag,
                                        void* stream);

/*
 * Per-step metadata of the diffusion attention path, built on the device in one
 * launch. Replaces the per-sequence host loop that the reference runs inside every
 * layer (attention.py:168-304: which rows a sequence contributes, its block, the
 * cached rows it attends or the rows it selects) with the sizing rules of
 * sparse/state.py:44-62 (block boundaries) and engine/sequence.py:98-152 (n_keep),
 * and the packing of ModelRunner._run_diffusion (model_runner.py:240-321).
 * seqs: device int64 [batch, DLLM_PLAN_SEQ_FIELDS], per sequence in batch order:
 *   [0] cache state: 0 dense, 1 compute cache, 2 reuse cache
 *   [1] num_tokens L    [2] num_prompt_tokens P    [3] current block index
 *   [4] block length (SparseConfig.default_block_len)
 *   [5] retention ratio as the bits of an IEEE float64
 *   [6] pool_kernel | head_select << 32
 *   [7] device pointer of the sequence's slot list (int32), 0 for a dense sequence
 *   [8] its number of slots (must equal n_keep: min(max(1, int(Klen*r)), Klen))
 *   [9] 0
 * out: device int32 buffer; layout: HOST int64[DLLM_PLAN_LAYOUT_INTS] = {total ints,
 *   offset of cu_c, offset and capacity (rows) of the head_select descriptors, of the
 *   shared-ranking descriptors, offset and capacity of the reuse slots, of the
 *   head_select slots, of the shared-ranking slots}. cu (batch+1 row offsets) is at 0.
 * Written: cu [batch+1], cu_c [batch+1] (cached rows of reuse sequences), one
 * DLLM_SEQ_DESC_INTS descriptor per compute-cache sequence of each head_select flavour
 * (batch order; idx_off for a top_idx laid out [num_kv_heads, n_keep] per sequence with
 * head_select), and the concatenated slot lists of the reuse sequences and of each
 * selection flavour. A slot count that differs from the rule, an empty block in the
 * compute-cache state or an overflowing section sets DLLM_DEV_BAD_SEQUENCE in err_flag.
 * batch <= DLLM_PLAN_MAX_BATCH.
 */
#define DLLM_PLAN_SEQ_FIELDS 10
#define DLLM_PLAN_LAYOUT_INTS 12
#define DLLM_PLAN_MAX_BATCH 1024
DLLM_API int dllm_build_step_plan(const int64_t* seqs, int batch, int num_kv_heads, int32_t* out,
                                  const int64_t* layout, int32_t* err_flag, void* stream);

/*
 * Row-parallel o_proj fused with its all-reduce over NVLink peer memory
 * (replaces RowParallelLinear.forward: F.linear then dist.all_reduce,
 * linear.py:186-190). Every rank r of a tp-way group calls it, in the same order
 * and with the same epoch, for its x_r [M, K] (bf16, row stride x_stride) and
 * W_r [N, K] (its column slice of W_o, bf16, row stride w_stride); afterwards
 * y[rank] holds y = sum_r x_r W_r^T [M, N] (bf16; fp32 GEMM accumulation, each
 * rank's partial rounded to bf16, partials summed in rank order in fp32 and
 * rounded once). recv[p], y[p], flags[p] (HOST arrays of tp device pointers) are
 * rank p's buffers as addressed from this rank (its own, or a mapping of the
 * peer's from dllm_ipc_open): recv [tp, M, N] bf16 receive buffer, y [M, N] bf16
 * output, flags int32 [(tp + 1) * ceil(M/128) * N/256], zero before the first call.
 * epoch: nonzero, distinct from the previous call's (a counter). A rank can run at
 * most one call ahead of its peers, so alternate two y buffers between calls if
 * the output of a call is read after the next call started on a peer.
 * Bounded waits: a peer that does not take part makes the call end with
 * DLLM_DEV_WAIT_TIMEOUT in err_flag. N % 256 == 0, K % 64 == 0, tp <= 8.
 * No multicast, and no TMA or library code reads peer memory.
 */
#define DLLM_OPROJ_MAX_RANKS 8
DLLM_API int dllm_oproj_allreduce(const void* x, int64_t x_stride, const void* w, int64_t w_stride,
                                  int M, int N, int K, void* const* recv, void* const* y,
                                  int32_t* const* flags, int rank, int tp, int epoch,
                                  int32_t* err_flag, void* stream);

/*
 * CUDA IPC for the buffers of dllm_oproj_allreduce: dllm_ipc_export writes the
 * handle (DLLM_IPC_HANDLE_BYTES) of the allocation holding `ptr` and ptr's offset in
 * it; a peer process opens it with dllm_ipc_open (base address of the mapping; add
 * the offset) and releases it with dllm_ipc_close. These map memory the peer
 * owns; they allocate nothing.
 */
#define DLLM_IPC_HANDLE_BYTES 64
DLLM_API int dllm_ipc_export(const void* ptr, void* handle, int64_t* offset);
DLLM_API int dllm_ipc_open(const void* handle, void** base);
DLLM_API int dllm_ipc_close(void* base);

#ifdef __cplusplus
}
#endif

#endif /* DLLM_ATTN_H_ */
