/*
 * qsa_b200.h -- C ABI of the B200-native (sm_100a) QSA sparse-attention hot path.
 *
 * Three stages, one entry point each, plus plain helpers:
 *   1. qsa_indexer_scores    dense q.k of every visible compressed index key,
 *                            fused ReLU / head-weight / head-sum epilogue
 *   2. qsa_topk_expand       exact per-row top-k of fp32 scores, expanded to
 *                            token (or physical slot) ids plus the causal tail
 *   3. qsa_sparse_attention  paged BF16 GQA attention over the selected tokens
 *
 * Conventions (every entry point):
 *   - All pointers are device pointers of the current CUDA device, except
 *     where a comment says otherwise.  bf16 tensors are passed as void*.
 *   - Strides are in ELEMENTS of the pointed-to type, as torch reports them.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Nothing
 *     synchronises the host; every launch is CUDA-graph capturable.
 *   - No entry point allocates device memory.  Attention takes a
 *     caller-provided workspace sized by qsa_sparse_attention_workspace_bytes.
 *   - Return value: QSA_OK or a QSA_ERR_* code; qsa_last_error() gives the
 *     detail for the calling host thread.  Invalid metadata VALUES (a -1 page,
 *     an out-of-range index) are not errors: they are masked exactly as the
 *     reference masks them.
 *   - Per-device state (the device error word's address, kernel attributes,
 *     the SM count) is looked up once per device and kept for the process:
 *     the library expects each device's context to outlive its use, as torch
 *     keeps the primary context; a process that resets a device
 *     (cudaDeviceReset) must not call the library on it afterwards.
 *     (The static-scratch entry point looks its array up on every call.)
 */
#ifndef QSA_B200_H_
#define QSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QSA_API __attribute__((visibility("default")))
#else
#define QSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum qsa_status {
  QSA_OK = 0,
  QSA_ERR_INVALID = 1,     /* null pointer, negative size, misaligned / inconsistent strides */
  QSA_ERR_UNSUPPORTED = 2, /* shape outside the compiled range (head dim, GQA group, width) */
  QSA_ERR_WORKSPACE = 3,   /* workspace smaller than the matching *_workspace_bytes query */
  QSA_ERR_CUDA = 4,        /* a CUDA runtime call or kernel launch failed */
  QSA_ERR_DEVICE = 5,      /* the current device is not an sm_100 (B200) GPU */
  QSA_ERR_TIMEOUT = 6      /* a bounded device-side wait expired (see qsa_device_error_poll) */
};

/* Human-readable name of a status code (static storage). */
QSA_API const char* qsa_status_string(int status);
/* Detail of the last failure on the calling host thread (thread-local storage). */
QSA_API const char* qsa_last_error(void);
/* Library version string. */
QSA_API const char* qsa_version(void);
/*
 * Number of kernels this library has launched (or recorded into a CUDA graph)
 * in this process, counted on the host at each successful launch.  No
 * counterpart in the reference; used by benchmarks to report launches per step.
 */
QSA_API uint64_t qsa_kernel_launches(void);
/*
 * Measurement hook, no counterpart in the reference: while set (non-NULL),
 * qsa_sparse_attention* records the cudaEvent_t `before` on its stream right
 * before launching the main attention kernel and `after` right after it (before
 * the split merge), so a caller can time that kernel alone with
 * cudaEventElapsedTime.  Per host thread; NULL, NULL clears it.
 */
QSA_API int qsa_set_attention_timing_events(void* before, void* after);
/* QSA_OK when the current device is sm_100; QSA_ERR_DEVICE otherwise. */
QSA_API int qsa_device_check(void);
/*
 * Reads and clears the device-side error word of the current device
 * (synchronous: waits for the device).  0 = no error; otherwise a bit set of
 * QSA_DEVICE_ERR_* recorded by kernels whose bounded waits expired.
 */
QSA_API int qsa_device_error_poll(int32_t* error_bits);
/*
 * Self-test of the bounded-wait error path, no counterpart in the reference:
 * launches one CTA that waits on a barrier phase nothing completes.  The wait
 * gives up after its 1 s limit and sets QSA_DEVICE_ERR_WAIT_TIMEOUT in the
 * device error word (read it with qsa_device_error_poll); the kernel returns
 * normally and the context stays usable.  Takes about one second of GPU time.
 */
QSA_API int qsa_selftest_wait_timeout(void* stream);
enum {
  QSA_DEVICE_ERR_WAIT_TIMEOUT = 1, /* a bounded wait expired */
  QSA_DEVICE_ERR_OUT_OF_RANGE = 2  /* a slot / position / request outside its buffer was skipped */
};

/*
 * Top-k selection + expansion.
 * Replaces torch.ops.yulan_qsa_kernels.topk_expand
 * (reference ops/csrc/topk.cu:503-525, schema :550-552; Python wrapper
 * ops/topk.py:29-39; callers ops/indexer.py:273-279 and :336-343).
 *
 * For each row r: with L = min(lengths[r], score_width) and K = output_width / ratio,
 * selects the K columns of scores[r, :L] with the largest fp32 BIT PATTERNS
 * (uint32 order; ties to the lowest column), in ascending column order
 * (all of 0..L-1 when L <= K), and expands selected block b to the tokens
 * b*ratio .. b*ratio+ratio-1, followed by the causal tail of positions[r].
 * physical != 0 maps tokens to slots page*page_size+offset through
 * table[token_to_req[r]]; counts (nullable) receives the per-row valid count.
 * scores: fp32 [rows, score_width] (unit column stride).
 * positions: int64 [rows]; sequence_lengths: int32 [num_requests];
 * token_to_req, lengths: int32 [rows]; output: int32 [rows, output_width].
 * lengths may be NULL: each row's length is then its visible block count
 * min((positions[r] + 1) // ratio, sequence_lengths[req] // ratio) (0 for an
 * unmapped row), as qsa_visible_blocks computes it.
 * Limits (QSA_ERR_UNSUPPORTED beyond them): score_width up to 524288 columns
 * (16-CTA clusters of 1024 threads x 32 keys), K up to 49152 blocks (one
 * row's selection in 192 KB of shared memory); the same for qsa_topk.
 */
QSA_API int qsa_topk_expand(const float* scores, int64_t score_row_stride, int32_t rows,
                    int32_t score_width, const int32_t* lengths, const int64_t* positions,
                    const int32_t* sequence_lengths, int32_t num_requests,
                    const int32_t* token_to_req, const int32_t* table,
                    int64_t table_row_stride, int32_t table_width, int32_t* output,
                    int64_t output_row_stride, int64_t output_col_stride,
                    int32_t output_width, int32_t* counts, int32_t ratio, int32_t page_size,
                    int32_t physical, void* stream);

/*
 * Plain top-k ids (no expansion).
 * Replaces torch.ops.yulan_qsa_kernels.topk (reference ops/csrc/topk.cu:527-545,
 * schema :549; wrapper ops/topk.py:25-26).  output: int32 [rows, topk], unit
 * column stride; ids ascending, -1 padded when lengths[r] <= topk.
 */
QSA_API int qsa_topk(const float* scores, int64_t score_row_stride, int32_t rows, int32_t score_width,
             const int32_t* lengths, int32_t* output, int64_t output_row_stride, int32_t topk,
             void* stream);

/*
 * Indexer scores.
 * Replaces the launches of _qsa_mqa_paged_uniform_kernel (reference
 * ops/indexer.py:24-114, launched at :260-272) when query_start_loc == NULL,
 * and of _qsa_mqa_paged_prefill_kernel (ops/indexer.py:117-223, launched by
 * _prefill_logits :282-302) otherwise.
 *
 * logits[r - query_offset, c] = scale * sum_h w[r,h] * max(q[r,h,:] . key(c), 0)
 * for packed rows r in [query_offset, query_offset + num_rows) and columns
 * c < min(visible[r], table_width * page_size, logits_width); other logits are
 * not written.  key(c) = k_cache[page_table[req(r), c / page_size], c % page_size].
 * Decode (query_start_loc == NULL): req(r) = r / decode_query_len.
 * Prefill: req(r) is the request whose [qsl[req]-qsl[0], qsl[req+1]-qsl[0])
 * contains r; max_query_len bounds the rows of one request.
 * q: bf16 [rows, num_heads, head_dim] (unit dim stride); k_cache: bf16
 * [num_blocks, page_size, 1, head_dim] (unit dim stride); weights: fp32
 * [rows, num_heads] or NULL for all ones (the reference's weighting);
 * reference scale = head_dim ** -0.5.  head_dim must be 64 or 128.
 * visible may be NULL: row r's count is then derived as qsa_visible_blocks
 * does from positions (int64, indexed like visible), sequence_lengths
 * [num_sequences] and token_to_req (indexed like visible) with `ratio`; these
 * four are ignored when visible is given.
 */
QSA_API int qsa_indexer_scores(const void* q, int64_t q_row_stride, int64_t q_head_stride,
                       int32_t num_heads, int32_t head_dim, const void* k_cache,
                       int64_t cache_block_stride, int64_t cache_token_stride,
                       int32_t num_blocks, int32_t page_size, const int32_t* page_table,
                       int64_t table_row_stride, int32_t table_width, int32_t num_requests,
                       const int32_t* visible, const int64_t* positions,
                       const int32_t* sequence_lengths, int32_t num_sequences,
                       const int32_t* token_to_req, int32_t ratio,
                       const int32_t* query_start_loc,
                       int32_t decode_query_len, int32_t max_query_len, int32_t query_offset,
                       int32_t num_rows, const float* weights, int64_t weight_row_stride,
                       int64_t weight_head_stride, float scale, float* logits,
                       int64_t logits_row_stride, int32_t logits_width, void* stream);

/*
 * Fused decode selection: indexer scores -> top-k -> expansion in ONE launch.
 * Replaces, for decode rows, the scoring launch + topk_expand pair of the
 * reference's qsa_select_paged_decode (ops/indexer.py:227-279: the kernel at
 * :24-114 fills an fp32 logits chunk, then ops/csrc/topk.cu:503-525 selects
 * from it); the scores never leave the chip.
 *
 * The results are, bit for bit, those of qsa_indexer_scores (decode,
 * query_start_loc NULL, logits_width = score_width) followed by
 * qsa_topk_expand on those scores with lengths = each row's visible count,
 * score_width, and the expansion arguments below.  The arguments mean what
 * they mean in those two calls; num_sequences is the length of
 * sequence_lengths.  scores_out (nullable, [num_rows, score_width] fp32, row
 * stride scores_row_stride) receives the scores as qsa_indexer_scores would
 * write them.  Returns QSA_ERR_UNSUPPORTED, launching nothing, for shapes
 * outside the fused kernel's range (the two-call path covers them): pages
 * not a multiple of 8 rows, a head count that is not a power of two,
 * decode_query_len * num_heads > 32, top-k blocks above 8192, or more
 * requests than fit the GPU at once as thread-block clusters (at most one
 * request per SM).  The visible counts (or the positions, sequence lengths
 * and request ids they are derived from when visible is NULL) and the page
 * table are read before waiting on the preceding kernel of the stream (see
 * the programmatic-dependent-launch contract in INTEGRATION.md).
 */
QSA_API int qsa_select_decode(
    const void* q, int64_t q_row_stride, int64_t q_head_stride, int32_t num_heads,
    int32_t head_dim, const void* k_cache, int64_t cache_block_stride,
    int64_t cache_token_stride, int32_t num_blocks, int32_t page_size,
    const int32_t* page_table, int64_t table_row_stride, int32_t table_width,
    int32_t num_requests, const int32_t* visible, const int64_t* positions,
    const int32_t* sequence_lengths, int32_t num_sequences, const int32_t* token_to_req,
    int32_t ratio, int32_t decode_query_len, int32_t num_rows, const float* weights,
    int64_t weight_row_stride, int64_t weight_head_stride, float scale, int32_t score_width,
    const int32_t* main_table, int64_t main_table_row_stride, int32_t main_table_width,
    int32_t main_page_size, int32_t physical, int32_t* output, int64_t output_row_stride,
    int64_t output_col_stride, int32_t output_width, int32_t* counts, float* scores_out,
    int64_t scores_row_stride, void* stream);

/*
 * Visible compressed blocks per query row.
 * Replaces the torch computation in select_paged_tokens (reference
 * ops/indexer.py:363-369) with one launch:
 *   visible[r] = token_to_req[r] in [0, num_requests)
 *              ? min((positions[r] + 1) // ratio, sequence_lengths[req] // ratio) : 0
 * with floor division as in torch.  positions: int64 [rows]; the rest int32.
 * (The reference raises on token_to_req >= num_requests; here such rows get 0.)
 */
QSA_API int qsa_visible_blocks(const int64_t* positions, const int32_t* sequence_lengths,
                               int32_t num_requests, const int32_t* token_to_req, int32_t rows,
                               int32_t ratio, int32_t* visible, void* stream);

/*
 * Indexer preparation and main K/V cache writes, one launch.
 * Replaces qsa_prepare / _qsa_prepare_kernel (reference ops/prepare.py:169-228,
 * kernel :49-166, norm + RoPE :16-46); bound from Python by
 * qsa_vllm_b200.prepare.qsa_prepare with the reference's signature.
 *
 * index_qk: bf16 [num_tokens, >= (num_index_heads + 1) * index_head_dim], row
 *   stride index_row_stride (elements): the heads' query rows, then the raw key.
 * positions: int64 (stride positions_stride); q/k_norm_weight: bf16 [dim];
 * cos_sin_cache: bf16 [cos_sin_rows, rotary_dim] (cosines, then sines; row p
 *   at p * rotary_dim, as the reference indexes it).
 * index_q_out: bf16 [num_tokens, num_index_heads, index_head_dim] contiguous:
 *   RMSNorm(eps) * q weight, then rotate-half RoPE of the first rotary_dim dims,
 *   with bf16 rounding after each post-norm step.
 * Key compression, per k_work item (int32 [num_k_work, 2] = (request, work
 *   item in request); request < 0 = padding): group `work` of the request's
 *   chunk, the mean of compress_ratio raw keys ending at the group boundary
 *   (this chunk's keys, or the ring state_cache block state_table[request *
 *   state_table_stride] for earlier positions), normed with k_norm_weight and
 *   rotated at the group's first position, stored at
 *   compressed_slots[boundary token] of compressed_cache [compressed_blocks,
 *   compressed_page_size, dim].  Work item 0 then writes the chunk's last
 *   min(query length, state_size) raw keys to state_slots of the ring
 *   state_cache [state_blocks, state_size, dim].
 *   query_start_loc: int32 [num_requests + 1]; logical_positions,
 *   state_slots, compressed_slots: int64 [num_tokens].
 * Main K/V: main_key / main_value bf16 [num_tokens, num_main_kv_heads,
 *   main_head_dim] to main_slots (int64) of the paged caches [main_blocks,
 *   main_page_size, num_main_kv_heads, main_head_dim]; all strides in elements.
 * Slots < 0 are skipped.  Out-of-range slots, positions or requests (which the
 * reference would access out of bounds) are skipped and set
 * QSA_DEVICE_ERR_OUT_OF_RANGE in the device error word.
 * index_head_dim 64 or 128; index rows 4-byte aligned with even strides.
 */
QSA_API int qsa_prepare(
    const void* index_qk, int64_t index_row_stride, int32_t num_tokens, int32_t num_index_heads,
    int32_t index_head_dim, const int64_t* positions, int64_t positions_stride,
    const void* q_norm_weight, const void* k_norm_weight, const void* cos_sin_cache,
    int64_t cos_sin_rows, int32_t rotary_dim, float eps, void* index_q_out, void* state_cache,
    int64_t state_block_stride, int64_t state_token_stride, int64_t state_blocks,
    int32_t state_size, const int64_t* state_slots, const int32_t* state_table,
    int64_t state_table_stride, const int32_t* query_start_loc, int32_t num_requests,
    const int64_t* logical_positions, void* compressed_cache, int64_t compressed_block_stride,
    int64_t compressed_token_stride, int64_t compressed_blocks, int32_t compressed_page_size,
    const int64_t* compressed_slots, const int32_t* k_work, int32_t num_k_work,
    int32_t compress_ratio, const void* main_key, int64_t main_key_token_stride,
    int64_t main_key_head_stride, int64_t main_key_dim_stride, const void* main_value,
    int64_t main_value_token_stride, int64_t main_value_head_stride,
    int64_t main_value_dim_stride, void* main_key_cache, int64_t main_key_cache_block_stride,
    int64_t main_key_cache_token_stride, int64_t main_key_cache_head_stride,
    int64_t main_key_cache_dim_stride, void* main_value_cache,
    int64_t main_value_cache_block_stride, int64_t main_value_cache_token_stride,
    int64_t main_value_cache_head_stride, int64_t main_value_cache_dim_stride,
    int64_t main_blocks, int32_t main_page_size, const int64_t* main_slots,
    int32_t num_main_kv_heads, int32_t main_head_dim, void* stream);

/*
 * Workspace bytes qsa_sparse_attention needs for these shapes on the current
 * device: fp32 per-warp partial outputs + LSE of the (row, KV-head group)
 * pairs that the work split cuts between two or more CTAs, combined by the
 * merge pass.  At most 2 x SMs x 8 x (query heads per KV head, <= 16) x
 * (head_dim + 1) x 4 bytes, whatever the row count (19.6 MB on a 148-SM
 * B200; 9.8 MB at 8 query heads per KV head), and 0 when no pair is cut.
 * 0 as well for shapes qsa_sparse_attention rejects (no rows, non-positive
 * head counts, query heads not a multiple of KV heads, negative width).
 * Deterministic in its arguments for a given device.
 */
QSA_API size_t qsa_sparse_attention_workspace_bytes(int32_t rows, int32_t num_q_heads,
                                            int32_t num_kv_heads, int32_t head_dim,
                                            int32_t topk_width, int32_t use_decode_kernel);

/*
 * Paged sparse GQA attention.
 * Replaces qsa_sparse_paged_attention (reference ops/qsa.py:594-688):
 * _qsa_sparse_paged_gqa_splitk_kernel (:109-303) and _qsa_merge_splitk_kernel
 * (:306-362); called from YuLanQSAImpl.forward (backend.py:39-68).
 *
 * For row r and query head h (kv head h / (num_q_heads / num_kv_heads)):
 *   out[r,h] = softmax_j(q[r,h] . K_j * head_dim^-0.5) . V_j over the columns j
 *   of indices[r, :n] that resolve to a cached token, n = min(valid_counts[r],
 *   topk_width) (topk_width when valid_counts is NULL).  P is rounded to bf16
 *   before P.V; with a gate, out = bf16(out) * sigmoid(gate).  Rows with no
 *   valid token get 0.
 * indices_are_physical != 0: indices are slots page*page_size+offset.
 * Otherwise indices are logical token ids of request token_to_req[r], mapped
 * through block_table.  q, gate, out: bf16 [rows, num_q_heads, head_dim];
 * k_cache / v_cache: bf16 [num_blocks, page_size, num_kv_heads, head_dim]
 * (unit dim stride; typically the two halves of one [.., 2*head_dim] buffer).
 * head_dim must be 64 or 128; num_q_heads / num_kv_heads must be 1..16.
 */
QSA_API int qsa_sparse_attention(const void* q, int64_t q_row_stride, int64_t q_head_stride,
                         int32_t rows, int32_t num_q_heads, int32_t head_dim,
                         const void* k_cache, int64_t k_block_stride, int64_t k_token_stride,
                         int64_t k_head_stride, const void* v_cache, int64_t v_block_stride,
                         int64_t v_token_stride, int64_t v_head_stride, int32_t num_blocks,
                         int32_t page_size, int32_t num_kv_heads, const int32_t* indices,
                         int64_t indices_row_stride, int32_t topk_width,
                         const int32_t* block_table, int64_t table_row_stride,
                         int32_t table_width, int32_t num_requests,
                         const int32_t* token_to_req, const int32_t* valid_counts,
                         const void* gate, int64_t gate_row_stride, int64_t gate_head_stride,
                         int64_t gate_dim_stride, void* out, int64_t out_row_stride,
                         int64_t out_head_stride, int32_t indices_are_physical,
                         int32_t use_decode_kernel, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * qsa_sparse_attention for callers that cannot allocate device memory.
 * No counterpart in the reference.  Such callers are, for example, code that
 * runs while a stream is captured in the global capture mode (a cudaMalloc
 * there is refused and invalidates the capture), serving engines that hand
 * all free device memory to their KV cache at start-up (a later cudaMalloc
 * fails), and C callers without a caching allocator (a cudaMalloc / cudaFree
 * per call synchronises the device and stalls the decode loop).  Same
 * arguments and results as
 * qsa_sparse_attention without (workspace, workspace_bytes): the split-K
 * scratch is a file-scope device array of QSA_STATIC_SCRATCH_BYTES per device,
 * whose address is looked up (cudaGetSymbolAddress, no allocation) on each
 * call with the caller's device current; nothing is allocated.
 *   - The array exists in every context that loads this library's module
 *     (at the first call under lazy module loading, at library load under
 *     CUDA_MODULE_LOADING=EAGER) and is held until the context ends.  Make the
 *     first call on a device before any stream capture, so the module load
 *     does not happen inside a capture.
 *   - Shapes are validated first (QSA_ERR_INVALID / QSA_ERR_UNSUPPORTED).
 *     The scratch need (qsa_sparse_attention_workspace_bytes) does not grow
 *     with the rows and fits QSA_STATIC_SCRATCH_BYTES on GPUs of up to 254
 *     SMs at any shape; a call needing more returns QSA_ERR_WORKSPACE.
 *   - Nothing in the scratch has to start at zero: each call writes every
 *     partial slot it reads (as an empty partial when a bounded wait gave up).
 *   - One scratch array serves all calls on a device: calls whose kernels
 *     overlap on the GPU (other streams or host threads) race on it; the
 *     caller must serialise them.
 */
#define QSA_STATIC_SCRATCH_BYTES ((size_t)32 << 20)
QSA_API int qsa_sparse_attention_static_scratch(
    const void* q, int64_t q_row_stride, int64_t q_head_stride, int32_t rows,
    int32_t num_q_heads, int32_t head_dim, const void* k_cache, int64_t k_block_stride,
    int64_t k_token_stride, int64_t k_head_stride, const void* v_cache, int64_t v_block_stride,
    int64_t v_token_stride, int64_t v_head_stride, int32_t num_blocks, int32_t page_size,
    int32_t num_kv_heads, const int32_t* indices, int64_t indices_row_stride,
    int32_t topk_width, const int32_t* block_table, int64_t table_row_stride,
    int32_t table_width, int32_t num_requests, const int32_t* token_to_req,
    const int32_t* valid_counts, const void* gate, int64_t gate_row_stride,
    int64_t gate_head_stride, int64_t gate_dim_stride, void* out, int64_t out_row_stride,
    int64_t out_head_stride, int32_t indices_are_physical, int32_t use_decode_kernel,
    void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* QSA_B200_H_ */
