// Internal launch interface between the C ABI (capi.cu) and the kernel
// translation units.  Plain structs of pointers, strides and sizes.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace qsa {

// ----------------------------------------------------------------- top-k
struct TopkParams {
  const float* scores;
  int64_t score_row_stride;
  int rows, width;
  const int32_t* lengths;
  const int64_t* positions;
  const int32_t* seq_lens;
  int num_requests;
  const int32_t* token_to_req;
  const int32_t* table;
  int64_t table_row_stride;
  int table_width;
  int32_t* output;
  int64_t out_row_stride, out_col_stride;
  int out_width;
  int32_t* counts;
  int ratio, page_size;
  FastDiv page_div;  // division by page_size
  int physical;   // expansion maps tokens to slots through `table`
  int aligned_blocks;  // physical && page_size % ratio == 0: one lookup per block
  int expand;     // 0: plain ids (torch.ops...topk), 1: expanded tokens
  int topk;       // selected blocks per row
  int slice_cap;  // keys held in shared memory per CTA
  int vec4;       // rows are 16-byte aligned: float4 loads
};
// Chooses the cluster width and launches.  Returns cudaError_t.
cudaError_t launch_topk(const TopkParams& p, cudaStream_t stream, int* plan_cluster);
// Largest score width the shared-memory-resident select supports.
int topk_max_width();
// Largest top-k (in blocks) one row's selection can hold in shared memory.
int topk_max_blocks();

// --------------------------------------------------------------- indexer
struct IndexerParams {
  const void* q;
  int64_t q_row_stride, q_head_stride;
  int heads, dim;
  const void* k_cache;
  int64_t block_stride, token_stride;
  int num_blocks, page_size;
  FastDiv page_div;  // division by page_size
  const int32_t* table;
  int64_t table_row_stride;
  int table_width, num_requests;
  const int32_t* visible;          // nullptr: derived per row from the four fields below
  const int64_t* positions;        // [rows] (same row indexing as q)
  const int32_t* seq_lens;         // [num_sequences]
  const int32_t* token_to_req;     // [rows]
  int num_sequences, ratio;
  const int32_t* query_start_loc;  // nullptr: uniform decode
  int decode_query_len, max_query_len, query_offset, num_rows;
  const float* weights;
  int64_t w_row_stride, w_head_stride;
  float scale;
  float* logits;
  int64_t logits_row_stride;
  int logits_width;
  int* err;
};

// Visible compressed blocks of row r: the caller's count, or derived.
__device__ __forceinline__ int row_visible(const IndexerParams& p, int r) {
  return p.visible != nullptr ? p.visible[r]
                              : visible_of(p.positions, p.seq_lens, p.num_sequences,
                                           p.token_to_req, p.ratio, r);
}
cudaError_t launch_indexer(const IndexerParams& p, cudaStream_t stream);
// tcgen05 + TMA formulation (indexer_tc.cu); launch_indexer dispatches to it
// when indexer_tc_eligible() holds, else runs the mma.sync kernel.
bool indexer_tc_eligible(const IndexerParams& p);
cudaError_t launch_indexer_tc(const IndexerParams& p, cudaStream_t stream);
cudaError_t launch_visible_blocks(const int64_t* positions, const int32_t* seq_lens,
                                  int num_requests, const int32_t* token_to_req, int rows,
                                  int ratio, int32_t* visible, cudaStream_t stream);

// ------------------------------------------- fused decode selection
// Indexer scores -> top-k -> expansion for decode rows in one launch
// (select_decode.cu).  `ix` describes the scoring (decode: query_start_loc is
// nullptr; its logits fields are unused), `tk` the selection and expansion
// (its scores / lengths / width fields are unused: the scores stay on chip and
// each row's length is its visible count, clipped to score_width).
struct SelectParams {
  IndexerParams ix;
  TopkParams tk;
  int score_width;          // logits columns of the two-launch path (decode bucket)
  float* scores_out;        // optional copy of the scores, [rows, score_width]
  int64_t scores_row_stride;
};
// Launches the fused kernel when the shapes allow it; returns
// cudaErrorNotSupported, launching nothing, when they do not, with the
// reason in *why (static string; why may be nullptr).
cudaError_t launch_select_decode(const SelectParams& p, cudaStream_t stream, const char** why);

// ------------------------------------------------------------- attention
// Most pairs a work split can cut: one per boundary between CTA ranges (the
// planner uses at most kMaxSplit + 1 CTAs).
constexpr int kMaxSplit = 255;
struct AttnParams {
  const void* q;
  int64_t q_row_stride, q_head_stride;
  int rows, q_heads, dim;
  const void* k_cache;
  int64_t k_block_stride, k_token_stride, k_head_stride;
  const void* v_cache;
  int64_t v_block_stride, v_token_stride, v_head_stride;
  int num_blocks, page_size, kv_heads;
  uint32_t num_slots;  // num_blocks x page_size (clamped to 2^32 - 1)
  FastDiv page_div;  // division by page_size
  const int32_t* indices;
  int64_t indices_row_stride;
  int topk_width;
  const int32_t* block_table;
  int64_t table_row_stride;
  int table_width, num_requests;
  const int32_t* token_to_req;
  const int32_t* valid_counts;
  const void* gate;
  int64_t gate_row_stride, gate_head_stride, gate_dim_stride;
  void* out;
  int64_t out_row_stride, out_head_stride;
  float scale_log2;  // head_dim^-0.5 * log2(e), rounded once to fp32 (ops/qsa.py:176)
  int physical;
  int kv_fused;     // 2: K||V of consecutive heads contiguous; 1: per head; 0: apart
  int slot_contig;  // consecutive slots are adjacent in memory (block stride = page * token stride)
  int gate_vec;     // gate rows 16-byte aligned with unit dim stride
  int out_vec;      // out rows 16-byte aligned
  // Stream-K work split: the (row, kv-head group) pairs x pair_tiles token
  // tiles form sk_units units of work, cut into sk_ctas contiguous ranges
  // (one per CTA).  A pair met by one CTA is finished by it; a pair that a
  // range boundary splits gets one partial slot from each CTA meeting it.
  int pair_tiles;       // token tiles per pair (upper bound: topk_width / tile)
  int sk_ctas;          // CTAs of the main kernel
  int64_t sk_units;     // pairs * pair_tiles
  int heads_per_unit;   // KV heads per pair
  int partials;         // partial slots per CTA: 2 x (8 / heads_per_unit) when some pair is split, else 0
  int merge_pieces;     // most CTAs meeting one split pair
  float* part_o;    // [sk_ctas, 2, 8 / heads_per_unit, heads of a pair, dim] fp32
  float* part_lse;  // [sk_ctas, 2, 8 / heads_per_unit, heads of a pair] fp32
  int* err;
};
// The split pairs, each named by the CTA holding its first tile: the merge
// kernel's grid columns (kept out of AttnParams, which every attention CTA
// reads).
struct SplitList {
  int n;
  int16_t cta[kMaxSplit];
};
struct AttnPlan {
  int pair_tiles;     // token tiles per (row, kv-head group) pair
  int ctas;           // main-kernel CTAs (contiguous unit ranges)
  int64_t units;      // pairs * pair_tiles
  int heads_per_unit; // KV heads per pair
  int partials;       // partial slots per CTA (2 x 8 / heads_per_unit when some pair is split, else 0)
  int merge_pieces;   // most CTAs meeting one split pair (0: none split)
  SplitList split;    // the split pairs
  size_t lse_offset;  // byte offset of the LSE slots in the workspace
  size_t workspace_bytes;
};
AttnPlan plan_attention(int rows, int q_heads, int kv_heads, int dim, int topk_width,
                        int use_decode_kernel);
cudaError_t launch_attention(const AttnParams& p, const SplitList& split, cudaStream_t stream);

// --------------------------------------------------------------- prepare
struct PrepareParams {
  // index projection [tokens, (heads + 1) * dim]: heads query rows, then the raw key
  const __nv_bfloat16* index_qk;
  int64_t index_row_stride;
  int num_tokens, heads, dim;
  const int64_t* positions;
  int64_t positions_stride;
  const __nv_bfloat16 *q_weight, *k_weight;
  const __nv_bfloat16* cos_sin;  // [cos_sin_rows, rotary]: cosines, then sines
  int64_t cos_sin_rows;
  int rotary;
  float eps;
  __nv_bfloat16* index_q_out;    // [tokens, heads, dim] contiguous
  // raw-key ring: [state_blocks, state_size, dim]
  __nv_bfloat16* state_cache;
  int64_t state_block_stride, state_token_stride;
  int state_size;
  int64_t state_blocks;
  const int64_t* state_slots;
  const int32_t* state_table;
  int64_t state_table_stride;
  const int32_t* query_start_loc;
  int num_requests;
  const int64_t* logical_positions;
  // compressed keys: [comp_blocks, comp_page, dim]
  __nv_bfloat16* compressed_cache;
  int64_t comp_block_stride, comp_token_stride;
  int comp_page;
  int64_t comp_blocks;
  const int64_t* compressed_slots;
  const int32_t* k_work;  // [num_k_work, 2]: (request, work item in request)
  int num_k_work, ratio;
  // main K/V rows [tokens, kv_heads, main_dim] into paged caches
  // [main_blocks, main_page, kv_heads, main_dim]
  const __nv_bfloat16 *main_key, *main_value;
  int64_t mk_stride[3], mv_stride[3];
  __nv_bfloat16 *main_key_cache, *main_value_cache;
  int64_t kc_stride[4], vc_stride[4];
  const int64_t* main_slots;
  int kv_heads, main_dim, main_page;
  int64_t main_blocks;
  int main_vec;   // unit dim strides and 16-byte aligned rows: 16-byte copies
  int* err;
};
cudaError_t launch_prepare(const PrepareParams& p, cudaStream_t stream);

int num_sms();
// One CTA waits on an mbarrier phase nothing completes; the bounded wait
// expires and records kDeviceErrWaitTimeout in *err (selftest.cu).
cudaError_t launch_wait_timeout_selftest(int* err, cudaStream_t stream);
// Records this host thread's attention timing event `which` (0: before the
// main attention kernel, 1: after it) on `stream`, when one is set.
void record_attention_event(int which, cudaStream_t stream);
// Counts `n` kernel launches of this library when `e` reports success (the
// host-side count read by qsa_kernel_launches); returns `e`.
cudaError_t count_launches(cudaError_t e, int n = 1);
// Records a failure message for qsa_last_error() on this host thread and
// returns `status` (for entry points outside capi.cu).
int set_last_error(int status, const char* fmt, ...);
// cudaFuncSetAttribute(fn, attr, value) once per (function, attribute, device);
// later launches (including ones under CUDA-graph capture) skip the call.
cudaError_t set_attr_once(const void* fn, cudaFuncAttribute attr, int value);

}  // namespace qsa
