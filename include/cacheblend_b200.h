/*
 * cacheblend_b200.h -- C ABI of the B200 (sm_100a) CacheBlend hot path.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, int64
 * sizes/strides (strides in BYTES unless stated otherwise) and a
 * `cudaStream_t` passed as `void*`, and returns an int status:
 *
 *   CB_OK (0)              success (work is enqueued on `stream`)
 *   CB_ERR_INVALID (-1)    invalid argument / shape / alignment
 *   CB_ERR_UNSUPPORTED (-2) dtype or layout the kernels do not implement
 *   CB_ERR_CUDA (-3)       a CUDA runtime/driver call failed
 *
 * `cb_last_error()` returns a thread-local message for the last failure on
 * the calling thread.  The library allocates no device or host memory and
 * keeps no global mutable state besides that per-thread string (and the
 * per-context caches of kernel attributes and of cb_sparse_q_scores_static's
 * array address), so it is
 * re-entrant and may be called from several host threads on several streams.
 * Kernels run on the device that owns `stream`; for the legacy NULL stream,
 * on the device that holds the call's output buffer.
 *
 * KV rows.  One token of one K (or V) plane is `num_heads` rows of
 * `head_bytes` contiguous bytes; consecutive heads are `head_stride` bytes
 * apart.  A paged plane addresses token slot s at
 *     base + (s / block_size) * block_stride + (s % block_size) * slot_stride
 * which covers vLLM's FlashAttention layout [2, blocks, block_size, H, D],
 * FlashInfer's [blocks, 2, block_size, H, D], the HND stride orders and the
 * separate (K, V) tuple layout.  A dense plane addresses token t at
 *     base + plane * plane_stride + (t / chunk_tokens) * chunk_stride
 *          + (t % chunk_tokens) * token_stride
 * (chunk_tokens <= 0 disables chunking), which covers the contiguous
 * [2, T, H, D] tensors of the reference and the chunk-major store staging.
 */
#ifndef CACHEBLEND_B200_H_
#define CACHEBLEND_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CB_OK 0
#define CB_ERR_INVALID (-1)
#define CB_ERR_UNSUPPORTED (-2)
#define CB_ERR_CUDA (-3)

/* Element types of KV / query tensors. */
#define CB_DTYPE_BF16 0
#define CB_DTYPE_FP16 1
#define CB_DTYPE_FP32 2

/* ABI revision; bumped whenever a signature below changes. */
CB_API int cb_abi_version(void);

/* Thread-local description of the last failure ("" if none). */
CB_API const char* cb_last_error(void);

/*
 * Paged gather: out[plane, t] = cache_plane[slots[t]] for plane in {K, V}.
 * Replaces `gather_paged_kv(kv_layer, slot_mapping, block_size, out)`
 * (cacheblend_vllm/kv_layout.py:90-122) and the Store-path gather into
 * staging (cacheblend_vllm/connector.py:408-419).  Negative slots wrap once
 * by num_blocks*block_size exactly like torch advanced indexing; any slot
 * still out of range makes the kernel skip that row and is reported by the
 * host wrapper's validation (kernels never touch memory out of range).
 */
CB_API int cb_paged_gather(const void* k_cache, const void* v_cache,
                    int64_t block_stride, int64_t slot_stride, int64_t head_stride,
                    int64_t num_blocks, int64_t block_size,
                    int64_t num_heads, int64_t head_bytes,
                    const int64_t* slots, int64_t num_tokens,
                    void* out, int64_t out_plane_stride, int64_t out_token_stride,
                    int64_t out_head_stride, int64_t out_chunk_tokens,
                    int64_t out_chunk_stride, void* stream);

/*
 * Paged scatter: cache_plane[slots[t]] = src[plane, t].
 * Replaces `scatter_paged_kv(contiguous, kv_layer, slot_mapping, block_size)`
 * (cacheblend_vllm/kv_layout.py:125-161) and `PagedBlendLoader.commit`
 * (cacheblend_vllm/ascend.py:385-407).  Duplicate slots: the last writer in
 * token order is not guaranteed (as with torch index_put on CUDA).
 */
CB_API int cb_paged_scatter(const void* src, int64_t src_plane_stride, int64_t src_token_stride,
                     int64_t src_head_stride, int64_t src_chunk_tokens,
                     int64_t src_chunk_stride,
                     void* k_cache, void* v_cache,
                     int64_t block_stride, int64_t slot_stride, int64_t head_stride,
                     int64_t num_blocks, int64_t block_size,
                     int64_t num_heads, int64_t head_bytes,
                     const int64_t* slots, int64_t num_tokens, void* stream);

/*
 * Strided device -> host copy (copy engine) on `stream`: `rows` rows of
 * `row_bytes`, `src_pitch` bytes apart in device memory and `dst_pitch` bytes
 * apart in pinned host memory.  The Store path's batch transfer
 * (cacheblend_vllm/connector.py:384-447, the D2H of `_enqueue_store_batch`)
 * into consecutive pinned-arena entries: one transfer per run of entries,
 * row pitch = the entry size.
 */
CB_API int cb_copy_rows_d2h(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                            int64_t row_bytes, int64_t rows, void* stream);

/*
 * Diagnostics: each of the library's four bounded-wait helpers waits on a
 * barrier that is never completed, gives up after its bound (about 2 s) and
 * ORs its bit (1, 2, 4, 8) into *result (device memory, zeroed by the caller)
 * on `stream`.  A result of 15 shows that a stuck pipeline stage ends in an
 * error word instead of a hang, and the context stays usable.
 */
CB_API int cb_wait_selftest(int32_t* result, void* stream);

/*
 * Host function (no GPU): the 64-bit polynomial fingerprint of every full
 * `window` of `tokens` (n - window + 1 values into `out`), identical to
 * cacheblend_vllm/hashing.py:42-53 (rolling_hash_values) in O(n).
 */
CB_API int cb_window_hashes(const int64_t* tokens, int64_t n, int64_t window, uint64_t* out);

/*
 * Host function (no GPU): ascending offsets i < n with hashes[i] in `known`
 * (ascending, distinct); at most `max_out` are written, *count receives the
 * total.  The candidate scan of TokenRangeMatcher.match
 * (cacheblend_vllm/matcher.py:80-125) before token verification.
 */
CB_API int cb_hash_candidates(const uint64_t* hashes, int64_t n, const uint64_t* known,
                              int64_t num_known, int64_t* out, int64_t max_out, int64_t* count);

/*
 * Number of common entries of two strictly ascending int64 index lists
 * (device memory), written to *count (device memory) on `stream`.  The
 * overlap of the two selections that the `compare` strategy reports
 * (cacheblend_vllm/ascend.py:713-747: overlap_tokens, and with the list
 * lengths the union and Jaccard index) without building the reference's two
 * boolean masks.
 */
CB_API int cb_sorted_overlap(const int64_t* a, int64_t na, const int64_t* b, int64_t nb,
                             int64_t* count, void* stream);

/*
 * Failure word of the bulk-copy paged gather/scatter kernels on the stream's
 * device (0: none; 1: a bounded wait for a bulk copy gave up and the launch
 * stopped early).  Synchronizes `stream`, stores the word in *value and
 * clears it when `reset` is non-zero.  Diagnostic entry point with no
 * counterpart in cacheblend_vllm (torch indexing cannot fail this way).
 */
CB_API int cb_paged_copy_error(void* stream, int32_t* value, int reset);

/*
 * RoPE relocation of an already rotated key: out = R(new) R(old)^-1 key,
 * evaluated op by op in the key dtype exactly like
 * `relocate_key(rotary_emb, old_positions, new_positions, key)`
 * (cacheblend_vllm/ascend.py:52-103, the cos_sin_cache branch).
 * key/out: [num_tokens, num_heads, head_size] with row stride
 * `token_stride` bytes and head stride `head_size` elements.  cos_sin:
 * [max_position, rotary_dim] in the key dtype (cos half, then sin half).
 * In-place (out == key) is allowed.
 */
CB_API int cb_relocate_key(const void* key, void* out, int64_t token_stride, int64_t out_token_stride,
                    int64_t num_tokens, int64_t num_heads, int64_t head_size,
                    int64_t rotary_dim, int is_neox, int dtype,
                    const void* cos_sin, int64_t max_position,
                    const int64_t* old_positions, const int64_t* new_positions,
                    void* stream);

/*
 * One hit segment of a blend plan for one layer.  k_src / v_src are device
 * addresses (device memory, or mapped pinned host memory for the zero-copy
 * load) of the segment's first token; token t of the segment is at
 * src + t * src_token_stride, heads `src_head_stride` apart.
 */
typedef struct cb_segment_t {
  uint64_t k_src;
  uint64_t v_src;
  int64_t src_token_stride;
  int64_t src_head_stride;
  int32_t source_start; /* token position the chunk was cached at */
  int32_t target_start; /* token position inside this request */
  int32_t length;       /* tokens */
  int32_t rotate;       /* nonzero: relocate K from source to target position */
} cb_segment_t;

/*
 * Fused per-layer blend load into the staging buffer `out` ([2, alloc_end,
 * H, D] dense plane description):
 *   t <  apc_prefix            : gathered from the paged cache (slots[t])
 *   token_segment[t] == -1     : zero (gap)
 *   token_segment[t] == s >= 0 : segment s, K relocated when rotate != 0
 * Replaces PagedBlendLoader.prefetch's body: the APC prefix gather, _zero_gaps,
 * _load_segments_fused and _load_segments_individually
 * (cacheblend_vllm/ascend.py:224-370).  token_segment is int32[alloc_end]
 * (entries below apc_prefix are ignored); segments is cb_segment_t[num_segments]
 * in device memory.  max_ctas > 0 caps the grid: a load that reads mapped
 * host memory is PCIe-bound and needs only a few SMs' worth of loads in
 * flight, leaving the rest of the GPU to the serving stream.  With
 * max_ctas == 0 and 16-byte aligned rows the load is staged through shared
 * memory by TMA bulk copies; its pipeline waits are bounded (2 s) and a wait
 * that runs out stores a nonzero code into *device_error (nullable, device
 * memory; 1 = producer, 2 = consumer) instead of hanging.
 */
CB_API int cb_blend_load_layer(void* out, int64_t out_plane_stride, int64_t out_token_stride,
                        int64_t out_head_stride, int64_t alloc_end, int64_t apc_prefix,
                        const void* k_cache, const void* v_cache,
                        int64_t block_stride, int64_t slot_stride, int64_t head_stride,
                        int64_t num_blocks, int64_t block_size, const int64_t* slots,
                        int64_t num_heads, int64_t head_size, int dtype,
                        const int32_t* token_segment, const cb_segment_t* segments,
                        int64_t num_segments,
                        const void* cos_sin, int64_t max_position, int64_t rotary_dim,
                        int is_neox, int64_t max_ctas, int32_t* device_error, void* stream);

/*
 * K-deviation score: scores[i] = sum_j (fresh[i, j] - cached[abs_i, j])^2 in
 * fp32, abs_i = abs_index ? abs_index[i] : abs_offset + i; a row whose abs_i
 * falls outside [0, cached_rows) scores NaN and is not read.  Replaces the
 * inline expression of Qwen3BlendExecutor._compute_layer
 * (cacheblend_vllm/ascend.py:535-538).  The reduction order is fixed (see
 * the oracle): lane l of a warp accumulates 16-byte vectors l, l+32, ... with
 * fmaf, then a xor-butterfly 16,8,4,2,1 combines the 32 partial sums.
 * Strides are in bytes; width in elements.
 */
CB_API int cb_kv_deviation(const void* fresh, int64_t fresh_row_stride,
                    const void* cached, int64_t cached_row_stride, int64_t cached_rows,
                    const int64_t* abs_index, int64_t abs_offset,
                    int64_t num_tokens, int64_t width, int dtype,
                    float* scores, void* stream);

/*
 * Masked top-k selection (Qwen3BlendExecutor._select,
 * cacheblend_vllm/ascend.py:757-796, after the TP all-reduce): writes the
 * ascending indices of base_mask[i] != 0 united with the k largest scores
 * among the remaining entries.  `k` must already follow the reference's
 * budget formula (computed by the host: it depends only on mask counts).
 * Exactly (#base + k) indices are written to out_index (never more than
 * out_capacity).  Ties at the k-th value keep the lowest indices; NaN ranks
 * above +inf (torch.topk order).  One CTA; no workspace.
 */
CB_API int cb_select_topk(const float* scores, const uint8_t* base_mask, int64_t n, int64_t k,
                   int64_t* out_index, int64_t out_capacity, void* stream);

/*
 * Tensor-parallel selection with the score reduction done over NVLink peer
 * memory: the TP all-reduce of the partial scores and `_select`
 * (cacheblend_vllm/ascend.py:764-770 tensor_model_parallel_all_reduce, then
 * 771-796) in one launch of one 8-CTA cluster per rank, replacing the NCCL
 * all-reduce + cb_select_topk pair.  Every rank owns an exchange buffer
 * (cb_peer_select_buffer_size bytes for its world size and the largest token
 * count it will select over) that every rank maps: the owner creates it with
 * cb_peer_buffer_create (zeroed; the 64-byte CUDA IPC handle goes to the other
 * ranks), the others open it with cb_peer_buffer_open.  `buffers` is a HOST
 * array of `world` device addresses, indexed by rank (this rank's own buffer
 * and the opened mappings of the others').  Each call stores this rank's
 * partial scores into every rank's buffer, waits (bounded, 2 s) for every
 * rank's scores of the same call, sums them in rank order (rank 0 first: the
 * same fp32 sum on every rank, so every rank selects the same tokens), writes
 * the sum to `summed` (may be NULL) and selects exactly like cb_select_topk.
 * All ranks size their buffers for the same world and max_tokens and make
 * the same sequence of calls with the same n, k and base mask, on streams that
 * run them in call order; n <= max_tokens <= 344,064.  `device`: the CUDA
 * device the buffer lives on (create) or is mapped into (open, close).
 * `protocol` 0: the partial scores as fp32 rows, one system fence, then a
 * flag per (rank, cluster CTA); 1 (low latency): every score as a 64-bit word
 * carrying the call number, polled by the reader, with no fence or flag.  All
 * ranks must use the same protocol for a call.  A wait that gives up stores 5
 * in *device_error (if not NULL): that call's result is wrong, later calls are
 * right again once the late rank catches up.
 * cb_peer_buffer_reset zeroes the whole buffer (all ranks, at a quiescent
 * point, e.g. after an error); close opened mappings before the owners
 * destroy their buffers.
 */
#define CB_IPC_HANDLE_BYTES 64
CB_API int cb_peer_select_buffer_size(int world, int64_t max_tokens, int64_t* bytes);
CB_API int cb_peer_buffer_create(int device, int64_t bytes, void** buffer, void* ipc_handle);
CB_API int cb_peer_buffer_open(int device, const void* ipc_handle, void** buffer);
CB_API int cb_peer_buffer_close(int device, void* buffer);
CB_API int cb_peer_buffer_destroy(int device, void* buffer);
CB_API int cb_peer_buffer_reset(void* buffer, int world, int64_t max_tokens, void* stream);
CB_API int cb_select_topk_peer(const float* partial, const uint8_t* base_mask, int64_t n, int64_t k,
                               int64_t* out_index, int64_t out_capacity, const uint64_t* buffers,
                               int rank, int world, int64_t max_tokens, int protocol, float* summed,
                               int32_t* device_error, void* stream);
/*
 * The same exchange with every rank played by one cooperative launch on one
 * GPU (cluster r is rank r; `buffers` are all local): partial is
 * [world][n] fp32, out_index [world][out_capacity], summed [world][n].  The
 * single-GPU check of the multi-rank protocol.
 */
CB_API int cb_select_topk_peer_all_ranks(const float* partial, const uint8_t* base_mask, int64_t n,
                                         int64_t k, int64_t* out_index, int64_t out_capacity,
                                         const uint64_t* buffers, int world, int64_t max_tokens,
                                         int protocol, float* summed, int32_t* device_error,
                                         void* stream);

/*
 * Bytes of the workspace cb_kv_deviation_select needs (a 2048-bin histogram
 * and a completion ticket).
 */
CB_API int cb_kv_deviation_select_workspace_size(int64_t* bytes);

/*
 * K-deviation score and recompute selection of a single-rank check layer in
 * one launch: cb_kv_deviation's scores (bit-identical, written to `scores`)
 * and cb_select_topk's ascending index set of base_mask[i] != 0 united with
 * the k largest non-base scores (out_index, at most out_capacity entries).
 * Replaces the deviation expression and `_select`
 * (cacheblend_vllm/ascend.py:534-543, 757-796) when no TP all-reduce sits
 * between them.  8-CTA clusters score the tokens and histogram the top 11
 * bits of the non-base scores into `workspace`; the cluster that finishes
 * last (a ticket in the workspace) runs the remaining radix passes and the
 * ordered compaction.  `workspace` (16-byte aligned device memory,
 * cb_kv_deviation_select_workspace_size bytes) must be zero before its first
 * use; every call leaves it zero again, and calls sharing one workspace must
 * not overlap on the GPU.  Rows that are not 16-byte aligned, more than
 * 327,680 tokens, or a NULL workspace fall back to the two launches
 * (cb_kv_deviation, then cb_select_topk) with the same results.
 */
CB_API int cb_kv_deviation_select(const void* fresh, int64_t fresh_row_stride, const void* cached,
                                  int64_t cached_row_stride, int64_t cached_rows,
                                  const int64_t* abs_index, int64_t abs_offset,
                                  int64_t num_tokens, int64_t width, int dtype,
                                  const uint8_t* base_mask, int64_t k, float* scores,
                                  int64_t* out_index, int64_t out_capacity, void* workspace,
                                  int64_t workspace_bytes, void* stream);

/*
 * Workspace bytes cb_blend_attention needs (row positions, tile bounds and the
 * rows' log2-sum-exps).  Same shape limits as
 * Sparse-Q: head_size 128, bf16 or fp16, (q heads / KV heads) dividing 128.
 */
CB_API int cb_blend_attention_workspace_size(int64_t num_queries, int64_t num_keys,
                                             int64_t num_q_heads, int64_t num_kv_heads,
                                             int64_t head_size, int dtype, int64_t* bytes);

/*
 * Causal attention of the computed queries over the whole staging context
 * (Qwen3BlendExecutor._attention, cacheblend_vllm/ascend.py:798-846, its
 * einsum path): query [num_queries][num_q_heads][head_size] at absolute
 * positions query_positions[i] (device int64; a position >= num_keys sees
 * every key, as the reference's mask does; a negative one gives zeros), key and
 * value [num_keys][num_kv_heads][head_size] (staging rows = positions),
 * query head h attends KV head h / (num_q_heads / num_kv_heads):
 *   w = T(T(q . k) * scale), p = softmax over keys k <= pos of w (fp32),
 *   out = T(sum_k T(p) v).
 * exact_rounding = 1 follows that order: one launch computes each row's
 * log2-sum-exp of w, a second rounds the normalized p to T before P V.
 * exact_rounding = 2 keeps the roundings of w in one launch (flash order: the
 * unnormalized exp2 values rounded to T, O divided by the row sum at the end;
 * within one T ulp per probability).  exact_rounding = 0 computes
 * w = (q . k) * scale in fp32, flash order (the reference's fused attention
 * kernel, ascend.py:814-830); it needs scale > 0.
 * Strides in bytes, rows and heads 16-byte aligned, heads contiguous within a
 * row.  On the tensor cores: QK^T and PV with tcgen05.mma, accumulators in
 * TMEM, operands staged by TMA; device_error (optional) receives a code if a
 * bounded wait gives up.
 */
CB_API int cb_blend_attention(const void* query, int64_t query_token_stride, const void* key,
                              int64_t key_token_stride, const void* value,
                              int64_t value_token_stride, int64_t num_keys, int64_t num_q_heads,
                              int64_t num_kv_heads, int64_t head_size, int dtype,
                              const int64_t* query_positions, int64_t num_queries, float scale,
                              int exact_rounding, void* out, int64_t out_token_stride,
                              void* workspace, int64_t workspace_bytes, int32_t* device_error,
                              void* stream);

/*
 * Workspace bytes cb_sparse_q_scores needs for `num_queries` sparse queries
 * (dense per-KV-head query rows, per-row log-sum-exp, row positions, tile
 * position bounds).  head_size must be 128, dtype bf16 or fp16, and the query
 * heads a multiple of the KV heads with (q heads / KV heads) dividing 128.
 */
CB_API int cb_sparse_q_workspace_size(int64_t num_queries, int64_t num_q_heads,
                               int64_t num_kv_heads, int64_t head_size, int dtype,
                               int64_t* bytes);

/*
 * Sparse-Q attention mass per key (Qwen3BlendExecutor._sparse_q_scores,
 * cacheblend_vllm/ascend.py:638-711, the score part): for every KV head,
 * query group head and sparse query i (query row query_rows[i] of `query`,
 * position query_positions[i]) the causal softmax over keys 0..position of
 * round_dtype(q . k) * scale is added into scores[key] (fp32, [num_keys]).
 * query: [num_query_tokens, num_q_heads, 128] rows `query_token_stride` bytes
 * apart; key: [num_keys, num_kv_heads, 128] rows `key_token_stride` bytes
 * apart.  query_rows and query_positions are device int64 [num_queries].  A
 * position >= num_keys sees every key (the reference's mask); a query row
 * outside [0, num_query_tokens) or a negative position is not read, adds
 * nothing and stores code 4 into *device_error.  Runs on the tcgen05 tensor
 * cores in two passes (row log-sum-exp, then per-key mass); `workspace` (1 KiB
 * aligned, device memory, cb_sparse_q_workspace_size bytes) holds the
 * intermediate state.  Pipeline waits are bounded (2 s); a timeout stores a
 * nonzero code (1-3) into *device_error (nullable).
 */
CB_API int cb_sparse_q_scores(const void* query, int64_t query_token_stride,
                              int64_t num_query_tokens, const void* key,
                              int64_t key_token_stride, int64_t num_keys, int64_t num_q_heads,
                              int64_t num_kv_heads, int64_t head_size, int dtype,
                              const int64_t* query_rows, const int64_t* query_positions,
                              int64_t num_queries, float scale, float* scores, void* workspace,
                              int64_t workspace_bytes, int32_t* device_error, void* stream);

/*
 * cb_sparse_q_scores without a workspace argument.  No counterpart in the
 * reference.  For callers that cannot allocate device memory when they score
 * -- a serving worker whose free memory was claimed by the KV cache after
 * profiling, or an FFI host holding buffers of another runtime without an
 * allocator -- the workspace is a 32 MiB array inside this library (one per
 * GPU that loads it, held until the process exits); the function allocates
 * nothing.  Requests whose workspace (cb_sparse_q_workspace_size) exceeds
 * 32 MiB - 1 KiB are rejected with CB_ERR_INVALID.  The array's device address
 * is looked up (cudaGetSymbolAddress) on every call made outside a stream
 * capture and recorded per CUDA context; a call inside a capture uses the
 * recorded address, so make one call on EACH device (each context) outside
 * capture before capturing there -- otherwise the captured call returns
 * CB_ERR_INVALID.  All calls on a device share the array: calls whose
 * executions overlap on the GPU race and must be serialized (one stream, or
 * events).  Nothing in the array needs to start at zero: every call rewrites
 * the parts it reads.
 */
CB_API int cb_sparse_q_scores_static(const void* query, int64_t query_token_stride,
                                     int64_t num_query_tokens, const void* key,
                                     int64_t key_token_stride, int64_t num_keys,
                                     int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                                     int dtype, const int64_t* query_rows,
                                     const int64_t* query_positions, int64_t num_queries,
                                     float scale, float* scores, int32_t* device_error,
                                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CACHEBLEND_B200_H_ */
