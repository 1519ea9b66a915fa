// qsa_sparse_attention_static_scratch: paged sparse attention for callers that
// cannot allocate device memory -- code running under a global-mode stream
// capture (cudaMalloc is refused there), engines whose KV cache took all free
// memory at start-up, and C callers without a caching allocator (a cudaMalloc /
// cudaFree per call would synchronise the device).  The split-K workspace (normalised partial
// outputs + LSE) lives in a file-scope device array of QSA_STATIC_SCRATCH_BYTES
// instead of a caller-provided buffer; nothing here allocates.
//
// Nothing in the scratch must start at zero: every partial slot the merge
// reads is written by the main kernel of the same call (as an empty partial
// when a bounded wait gave up), so no clearing pass is needed.  There is one
// scratch array per device, shared by every call on that device: calls whose
// kernels overlap on the GPU (other streams, other host threads) race on it
// and must be serialised by the caller.
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/qsa_b200.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = QSA_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_attention_scratch[kScratchBytes];

// Device address of the current device's scratch.  Looked up on every call
// (the lookup allocates nothing), so it stays right if the context of a
// device is torn down and recreated.  On failure the pending CUDA error is
// cleared, so it does not surface in an unrelated later call.
cudaError_t scratch_address(void** out) {
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_attention_scratch);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  *out = ptr;
  return cudaSuccess;
}

}  // namespace

extern "C" int qsa_sparse_attention_static_scratch(
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
    void* stream) {
  const char* who = "qsa_sparse_attention_static_scratch";
  void* scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess)
    return qsa::set_last_error(QSA_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", who,
                               cudaGetErrorString(e));
  // The caller-workspace entry point validates the shapes first and only then
  // compares the plan's scratch need with the size it is given, so malformed
  // calls get QSA_ERR_INVALID / QSA_ERR_UNSUPPORTED, and well-formed calls
  // above the static maximum get QSA_ERR_WORKSPACE (reworded below).
  const int status = qsa_sparse_attention(
      q, q_row_stride, q_head_stride, rows, num_q_heads, head_dim, k_cache, k_block_stride,
      k_token_stride, k_head_stride, v_cache, v_block_stride, v_token_stride, v_head_stride,
      num_blocks, page_size, num_kv_heads, indices, indices_row_stride, topk_width, block_table,
      table_row_stride, table_width, num_requests, token_to_req, valid_counts, gate,
      gate_row_stride, gate_head_stride, gate_dim_stride, out, out_row_stride, out_head_stride,
      indices_are_physical, use_decode_kernel, scratch, kScratchBytes, stream);
  if (status == QSA_ERR_WORKSPACE) {
    const size_t need = qsa_sparse_attention_workspace_bytes(
        rows, num_q_heads, num_kv_heads, head_dim, topk_width, use_decode_kernel);
    return qsa::set_last_error(
        QSA_ERR_WORKSPACE,
        "%s: this call needs %zu bytes of split-K scratch, above the static maximum of %zu "
        "bytes (QSA_STATIC_SCRATCH_BYTES); use qsa_sparse_attention with a caller workspace",
        who, need, kScratchBytes);
  }
  return status;
}
