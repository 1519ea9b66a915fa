// C ABI of the QSA hot path (declared in include/qsa_b200.h): argument checks,
// error reporting and dispatch to the kernel launchers.  Nothing here
// allocates device memory or synchronises the host (except the explicit
// qsa_device_error_poll).
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <atomic>
#include <mutex>
#include <set>
#include <tuple>

#include "../../include/qsa_b200.h"
#include "kernels.h"

namespace qsa {

namespace {
thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(QSA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Device-side error word, one per device (a __device__ variable is
// instantiated per device context).
__device__ int g_device_error = 0;

constexpr int kMaxDevices = 64;
int* g_err_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
std::mutex g_mu;

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int* device_error_word() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_err_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_error) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    g_err_ptr[dev] = static_cast<int*>(ptr);
  }
  return g_err_ptr[dev];
}
}  // namespace

int set_last_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

std::atomic<uint64_t> g_launches{0};
thread_local cudaEvent_t g_attention_events[2] = {nullptr, nullptr};

void record_attention_event(int which, cudaStream_t stream) {
  cudaEvent_t ev = g_attention_events[which];
  if (ev == nullptr) return;
  // under stream capture the record becomes an event node of the graph, so
  // graph replays time the kernel too
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(stream, &cap);
  cudaEventRecordWithFlags(ev, stream,
                           cap == cudaStreamCaptureStatusActive ? cudaEventRecordExternal
                                                                : cudaEventRecordDefault);
}

cudaError_t count_launches(cudaError_t e, int n) {
  if (e == cudaSuccess) g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed);
  return e;
}

int num_sms() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

cudaError_t set_attr_once(const void* fn, cudaFuncAttribute attr, int value) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int, int>> done;
  const auto key = std::make_tuple(fn, static_cast<int>(attr), value, current_device());
  {
    std::lock_guard<std::mutex> lk(mu);
    if (done.count(key)) return cudaSuccess;
  }
  const cudaError_t e = cudaFuncSetAttribute(fn, attr, value);
  if (e == cudaSuccess) {
    std::lock_guard<std::mutex> lk(mu);
    done.insert(key);
  }
  return e;
}

}  // namespace qsa

using namespace qsa;

extern "C" {

const char* qsa_status_string(int status) {
  switch (status) {
    case QSA_OK: return "ok";
    case QSA_ERR_INVALID: return "invalid argument";
    case QSA_ERR_UNSUPPORTED: return "unsupported shape";
    case QSA_ERR_WORKSPACE: return "workspace too small";
    case QSA_ERR_CUDA: return "CUDA error";
    case QSA_ERR_DEVICE: return "not an sm_100 device";
    case QSA_ERR_TIMEOUT: return "device wait timed out";
  }
  return "unknown status";
}

const char* qsa_last_error(void) { return g_last_error; }

const char* qsa_version(void) { return "qsa_b200 0.1.0 (sm_100a)"; }

uint64_t qsa_kernel_launches(void) { return qsa::g_launches.load(std::memory_order_relaxed); }

int qsa_set_attention_timing_events(void* before, void* after) {
  qsa::g_attention_events[0] = static_cast<cudaEvent_t>(before);
  qsa::g_attention_events[1] = static_cast<cudaEvent_t>(after);
  return QSA_OK;
}

int qsa_device_check(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(QSA_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                major, minor);
  return QSA_OK;
}

int qsa_device_error_poll(int32_t* error_bits) {
  int* w = device_error_word();
  if (w == nullptr) return fail(QSA_ERR_CUDA, "device error word unavailable");
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading device error word");
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "clearing device error word");
  }
  if (error_bits) *error_bits = v;
  return QSA_OK;
}

int qsa_selftest_wait_timeout(void* stream) {
  int* w = device_error_word();
  if (w == nullptr) return fail(QSA_ERR_CUDA, "device error word unavailable");
  cudaError_t e = launch_wait_timeout_selftest(w, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "qsa_selftest_wait_timeout");
  return QSA_OK;
}

// ------------------------------------------------------------------ top-k
static int topk_common(TopkParams& p, void* stream, const char* who) {
  if (p.rows < 0 || p.width < 0) return fail(QSA_ERR_INVALID, "%s: negative rows/width", who);
  if (p.rows == 0) return QSA_OK;
  // lengths may be NULL only when the kernel can derive them (expansion)
  if (!p.scores || (!p.lengths && !p.expand) || !p.output)
    return fail(QSA_ERR_INVALID, "%s: null scores/lengths/output", who);
  if (p.score_row_stride < p.width)
    return fail(QSA_ERR_INVALID, "%s: score row stride %lld < width %d", who,
                (long long)p.score_row_stride, p.width);
  if (p.width > topk_max_width())
    return fail(QSA_ERR_UNSUPPORTED, "%s: score width %d exceeds %d", who, p.width,
                topk_max_width());
  if (p.topk > topk_max_blocks())
    return fail(QSA_ERR_UNSUPPORTED, "%s: top-k of %d blocks exceeds %d", who, p.topk,
                topk_max_blocks());
  p.vec4 = aligned(p.scores, 16) && (p.score_row_stride % 4 == 0);
  int cluster = 0;
  cudaError_t e = launch_topk(p, static_cast<cudaStream_t>(stream), &cluster);
  if (e != cudaSuccess) return cuda_fail(e, who);
  return QSA_OK;
}

int qsa_topk_expand(const float* scores, int64_t score_row_stride, int32_t rows,
                    int32_t score_width, const int32_t* lengths, const int64_t* positions,
                    const int32_t* sequence_lengths, int32_t num_requests,
                    const int32_t* token_to_req, const int32_t* table,
                    int64_t table_row_stride, int32_t table_width, int32_t* output,
                    int64_t output_row_stride, int64_t output_col_stride,
                    int32_t output_width, int32_t* counts, int32_t ratio, int32_t page_size,
                    int32_t physical, void* stream) {
  if (ratio <= 0) return fail(QSA_ERR_INVALID, "qsa_topk_expand: ratio must be positive");
  if (physical && page_size <= 0)
    return fail(QSA_ERR_INVALID, "qsa_topk_expand: page_size must be positive");
  if (rows > 0 && (!positions || !sequence_lengths || !token_to_req))
    return fail(QSA_ERR_INVALID, "qsa_topk_expand: null metadata pointer");
  if (physical && rows > 0 && !table)
    return fail(QSA_ERR_INVALID, "qsa_topk_expand: physical output needs a table");
  if (output_width < 0 || num_requests < 0)
    return fail(QSA_ERR_INVALID, "qsa_topk_expand: negative output width / requests");
  TopkParams p = {};
  p.scores = scores;
  p.score_row_stride = score_row_stride;
  p.rows = rows;
  p.width = score_width;
  p.lengths = lengths;
  p.positions = positions;
  p.seq_lens = sequence_lengths;
  p.num_requests = num_requests;
  p.token_to_req = token_to_req;
  p.table = table;
  p.table_row_stride = table_row_stride;
  p.table_width = physical ? table_width : 0;
  p.output = output;
  p.out_row_stride = output_row_stride;
  p.out_col_stride = output_col_stride;
  p.out_width = output_width;
  p.counts = counts;
  p.ratio = ratio;
  p.page_size = physical ? page_size : 1;
  p.page_div = FastDiv(static_cast<uint32_t>(p.page_size));
  p.physical = physical ? 1 : 0;
  p.aligned_blocks = (physical && page_size % ratio == 0) ? 1 : 0;
  p.expand = 1;
  p.topk = output_width / ratio;
  return topk_common(p, stream, "qsa_topk_expand");
}

int qsa_topk(const float* scores, int64_t score_row_stride, int32_t rows, int32_t score_width,
             const int32_t* lengths, int32_t* output, int64_t output_row_stride, int32_t topk,
             void* stream) {
  if (topk < 0) return fail(QSA_ERR_INVALID, "qsa_topk: negative topk");
  TopkParams p = {};
  p.scores = scores;
  p.score_row_stride = score_row_stride;
  p.rows = rows;
  p.width = score_width;
  p.lengths = lengths;
  p.output = output;
  p.out_row_stride = output_row_stride;
  p.out_col_stride = 1;
  p.out_width = topk;
  p.ratio = 1;
  p.page_size = 1;
  p.expand = 0;
  p.topk = topk;
  return topk_common(p, stream, "qsa_topk");
}

// ---------------------------------------------------------------- indexer
int qsa_indexer_scores(const void* q, int64_t q_row_stride, int64_t q_head_stride,
                       int32_t num_heads, int32_t head_dim, const void* k_cache,
                       int64_t cache_block_stride, int64_t cache_token_stride,
                       int32_t num_blocks, int32_t page_size, const int32_t* page_table,
                       int64_t table_row_stride, int32_t table_width, int32_t num_requests,
                       const int32_t* visible, const int64_t* positions,
                       const int32_t* sequence_lengths, int32_t num_sequences,
                       const int32_t* token_to_req, int32_t ratio,
                       const int32_t* query_start_loc, int32_t decode_query_len,
                       int32_t max_query_len, int32_t query_offset,
                       int32_t num_rows, const float* weights, int64_t weight_row_stride,
                       int64_t weight_head_stride, float scale, float* logits,
                       int64_t logits_row_stride, int32_t logits_width, void* stream) {
  const char* who = "qsa_indexer_scores";
  if (num_rows < 0 || logits_width < 0) return fail(QSA_ERR_INVALID, "%s: negative size", who);
  if (num_rows == 0) return QSA_OK;
  if (!q || !k_cache || !page_table || !logits)
    return fail(QSA_ERR_INVALID, "%s: null pointer", who);
  if (!visible && (!positions || !sequence_lengths || !token_to_req || ratio <= 0 ||
                   num_sequences < 0))
    return fail(QSA_ERR_INVALID,
                "%s: without visible counts, positions / sequence_lengths / token_to_req and a "
                "positive ratio are needed", who);
  if (head_dim != 64 && head_dim != 128)
    return fail(QSA_ERR_UNSUPPORTED, "%s: head_dim %d (supported: 64, 128)", who, head_dim);
  const bool pow2 = num_heads > 0 && num_heads <= 8 && (num_heads & (num_heads - 1)) == 0;
  if (!(pow2 || (num_heads > 0 && num_heads % 8 == 0 && num_heads <= 128)))
    return fail(QSA_ERR_UNSUPPORTED, "%s: %d heads (supported: 1,2,4,8 or a multiple of 8)",
                who, num_heads);
  if (page_size <= 0 || table_width < 0 || num_blocks < 0)
    return fail(QSA_ERR_INVALID, "%s: bad page geometry", who);
  if (!aligned(q, 16) || q_row_stride % 8 || q_head_stride % 8 || !aligned(k_cache, 16) ||
      cache_block_stride % 8 || cache_token_stride % 8)
    return fail(QSA_ERR_INVALID, "%s: q / key cache need 16-byte aligned rows", who);
  if (query_start_loc == nullptr) {
    if (decode_query_len <= 0 || num_rows % decode_query_len)
      return fail(QSA_ERR_INVALID, "%s: %d decode rows not a multiple of query len %d", who,
                  num_rows, decode_query_len);
    if (decode_query_len * num_heads > 128)
      return fail(QSA_ERR_UNSUPPORTED, "%s: decode_query_len*heads > 128", who);
    if (query_offset != 0)
      return fail(QSA_ERR_INVALID, "%s: decode rows start at offset 0", who);
    if (num_rows / decode_query_len > num_requests)
      return fail(QSA_ERR_INVALID, "%s: %d decode requests but %d page-table rows", who,
                  num_rows / decode_query_len, num_requests);
  } else if (num_requests <= 0 || max_query_len <= 0) {
    return fail(QSA_ERR_INVALID, "%s: prefill needs requests and max_query_len", who);
  }
  IndexerParams p = {};
  p.q = q;
  p.q_row_stride = q_row_stride;
  p.q_head_stride = q_head_stride;
  p.heads = num_heads;
  p.dim = head_dim;
  p.k_cache = k_cache;
  p.block_stride = cache_block_stride;
  p.token_stride = cache_token_stride;
  p.num_blocks = num_blocks;
  p.page_size = page_size;
  p.page_div = FastDiv(static_cast<uint32_t>(page_size));
  p.table = page_table;
  p.table_row_stride = table_row_stride;
  p.table_width = table_width;
  p.num_requests = num_requests;
  p.visible = visible;
  p.positions = positions;
  p.seq_lens = sequence_lengths;
  p.num_sequences = num_sequences;
  p.token_to_req = token_to_req;
  p.ratio = ratio;
  p.query_start_loc = query_start_loc;
  p.decode_query_len = decode_query_len;
  p.max_query_len = max_query_len;
  p.query_offset = query_offset;
  p.num_rows = num_rows;
  p.weights = weights;
  p.w_row_stride = weight_row_stride;
  p.w_head_stride = weight_head_stride;
  p.scale = scale;
  p.logits = logits;
  p.logits_row_stride = logits_row_stride;
  p.logits_width = logits_width;
  p.err = device_error_word();
  cudaError_t e = launch_indexer(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, who);
  return QSA_OK;
}

int qsa_select_decode(const void* q, int64_t q_row_stride, int64_t q_head_stride,
                      int32_t num_heads, int32_t head_dim, const void* k_cache,
                      int64_t cache_block_stride, int64_t cache_token_stride, int32_t num_blocks,
                      int32_t page_size, const int32_t* page_table, int64_t table_row_stride,
                      int32_t table_width, int32_t num_requests, const int32_t* visible,
                      const int64_t* positions, const int32_t* sequence_lengths,
                      int32_t num_sequences, const int32_t* token_to_req, int32_t ratio,
                      int32_t decode_query_len, int32_t num_rows, const float* weights,
                      int64_t weight_row_stride, int64_t weight_head_stride, float scale,
                      int32_t score_width, const int32_t* main_table,
                      int64_t main_table_row_stride, int32_t main_table_width,
                      int32_t main_page_size, int32_t physical, int32_t* output,
                      int64_t output_row_stride, int64_t output_col_stride,
                      int32_t output_width, int32_t* counts, float* scores_out,
                      int64_t scores_row_stride, void* stream) {
  const char* who = "qsa_select_decode";
  if (num_rows < 0 || score_width < 0 || output_width < 0 || num_sequences < 0)
    return fail(QSA_ERR_INVALID, "%s: negative size", who);
  if (num_rows == 0) return QSA_OK;
  if (!q || !k_cache || !page_table || !output || !positions || !sequence_lengths ||
      !token_to_req)
    return fail(QSA_ERR_INVALID, "%s: null pointer", who);
  if (ratio <= 0) return fail(QSA_ERR_INVALID, "%s: ratio must be positive", who);
  if (physical && (!main_table || main_page_size <= 0))
    return fail(QSA_ERR_INVALID, "%s: physical output needs a block table and page size", who);
  if (head_dim != 64 && head_dim != 128)
    return fail(QSA_ERR_UNSUPPORTED, "%s: head_dim %d (supported: 64, 128)", who, head_dim);
  if (page_size <= 0 || table_width < 0 || num_blocks < 0)
    return fail(QSA_ERR_INVALID, "%s: bad page geometry", who);
  if (!aligned(q, 16) || q_row_stride % 8 || q_head_stride % 8 || !aligned(k_cache, 16) ||
      cache_block_stride % 8 || cache_token_stride % 8)
    return fail(QSA_ERR_INVALID, "%s: q / key cache need 16-byte aligned rows", who);
  if (decode_query_len <= 0 || num_rows % decode_query_len)
    return fail(QSA_ERR_INVALID, "%s: %d decode rows not a multiple of query len %d", who,
                num_rows, decode_query_len);
  if (num_rows / decode_query_len > num_requests)
    return fail(QSA_ERR_INVALID, "%s: %d decode requests but %d page-table rows", who,
                num_rows / decode_query_len, num_requests);
  if (scores_out && scores_row_stride < score_width)
    return fail(QSA_ERR_INVALID, "%s: scores row stride %lld < width %d", who,
                (long long)scores_row_stride, score_width);
  SelectParams sp = {};
  IndexerParams& p = sp.ix;
  p.q = q;
  p.q_row_stride = q_row_stride;
  p.q_head_stride = q_head_stride;
  p.heads = num_heads;
  p.dim = head_dim;
  p.k_cache = k_cache;
  p.block_stride = cache_block_stride;
  p.token_stride = cache_token_stride;
  p.num_blocks = num_blocks;
  p.page_size = page_size;
  p.page_div = FastDiv(static_cast<uint32_t>(page_size));
  p.table = page_table;
  p.table_row_stride = table_row_stride;
  p.table_width = table_width;
  p.num_requests = num_requests;
  p.visible = visible;
  p.positions = positions;
  p.seq_lens = sequence_lengths;
  p.num_sequences = num_sequences;
  p.token_to_req = token_to_req;
  p.ratio = ratio;
  p.query_start_loc = nullptr;
  p.decode_query_len = decode_query_len;
  p.max_query_len = decode_query_len;
  p.query_offset = 0;
  p.num_rows = num_rows;
  p.weights = weights;
  p.w_row_stride = weight_row_stride;
  p.w_head_stride = weight_head_stride;
  p.scale = scale;
  p.logits = nullptr;
  p.logits_row_stride = 0;
  p.logits_width = score_width;
  p.err = device_error_word();
  TopkParams& t = sp.tk;
  t.rows = num_rows;
  t.width = score_width;
  t.positions = positions;
  t.seq_lens = sequence_lengths;
  t.num_requests = num_sequences;
  t.token_to_req = token_to_req;
  t.table = main_table;
  t.table_row_stride = main_table_row_stride;
  t.table_width = physical ? main_table_width : 0;
  t.output = output;
  t.out_row_stride = output_row_stride;
  t.out_col_stride = output_col_stride;
  t.out_width = output_width;
  t.counts = counts;
  t.ratio = ratio;
  t.page_size = physical ? main_page_size : 1;
  t.page_div = FastDiv(static_cast<uint32_t>(t.page_size));
  t.physical = physical ? 1 : 0;
  t.aligned_blocks = (physical && main_page_size % ratio == 0) ? 1 : 0;
  t.expand = 1;
  t.topk = output_width / ratio;
  sp.score_width = score_width;
  sp.scores_out = scores_out;
  sp.scores_row_stride = scores_row_stride;
  const char* why = "unsupported shape";
  const cudaError_t e = launch_select_decode(sp, static_cast<cudaStream_t>(stream), &why);
  if (e == cudaErrorNotSupported)
    return fail(QSA_ERR_UNSUPPORTED,
                "%s: outside the fused kernel's range (%s); use qsa_indexer_scores + "
                "qsa_topk_expand", who, why);
  if (e != cudaSuccess) return cuda_fail(e, who);
  return QSA_OK;
}

int qsa_visible_blocks(const int64_t* positions, const int32_t* sequence_lengths,
                       int32_t num_requests, const int32_t* token_to_req, int32_t rows,
                       int32_t ratio, int32_t* visible, void* stream) {
  const char* who = "qsa_visible_blocks";
  if (rows < 0 || ratio <= 0) return fail(QSA_ERR_INVALID, "%s: bad rows / ratio", who);
  if (rows == 0) return QSA_OK;
  if (!positions || !sequence_lengths || !token_to_req || !visible)
    return fail(QSA_ERR_INVALID, "%s: null pointer", who);
  cudaError_t e = launch_visible_blocks(positions, sequence_lengths, num_requests, token_to_req,
                                        rows, ratio, visible, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, who);
  return QSA_OK;
}

// ---------------------------------------------------------------- prepare
int qsa_prepare(const void* index_qk, int64_t index_row_stride, int32_t num_tokens,
                int32_t num_index_heads, int32_t index_head_dim, const int64_t* positions,
                int64_t positions_stride, const void* q_norm_weight, const void* k_norm_weight,
                const void* cos_sin_cache, int64_t cos_sin_rows, int32_t rotary_dim, float eps,
                void* index_q_out, void* state_cache, int64_t state_block_stride,
                int64_t state_token_stride, int64_t state_blocks, int32_t state_size,
                const int64_t* state_slots, const int32_t* state_table,
                int64_t state_table_stride, const int32_t* query_start_loc,
                int32_t num_requests, const int64_t* logical_positions, void* compressed_cache,
                int64_t compressed_block_stride, int64_t compressed_token_stride,
                int64_t compressed_blocks, int32_t compressed_page_size,
                const int64_t* compressed_slots, const int32_t* k_work, int32_t num_k_work,
                int32_t compress_ratio, const void* main_key, int64_t main_key_token_stride,
                int64_t main_key_head_stride, int64_t main_key_dim_stride,
                const void* main_value, int64_t main_value_token_stride,
                int64_t main_value_head_stride, int64_t main_value_dim_stride,
                void* main_key_cache, int64_t main_key_cache_block_stride,
                int64_t main_key_cache_token_stride, int64_t main_key_cache_head_stride,
                int64_t main_key_cache_dim_stride, void* main_value_cache,
                int64_t main_value_cache_block_stride, int64_t main_value_cache_token_stride,
                int64_t main_value_cache_head_stride, int64_t main_value_cache_dim_stride,
                int64_t main_blocks, int32_t main_page_size, const int64_t* main_slots,
                int32_t num_main_kv_heads, int32_t main_head_dim, void* stream) {
  const char* who = "qsa_prepare";
  if (num_tokens < 0 || num_k_work < 0 || num_index_heads <= 0 || num_main_kv_heads < 0 ||
      num_requests < 0)
    return fail(QSA_ERR_INVALID, "%s: negative or zero sizes", who);
  if (index_head_dim != 64 && index_head_dim != 128)
    return fail(QSA_ERR_UNSUPPORTED, "%s: index head dim %d (64 or 128 supported)", who,
                index_head_dim);
  if (rotary_dim < 2 || rotary_dim % 2 || rotary_dim > index_head_dim)
    return fail(QSA_ERR_INVALID, "%s: rotary dim %d must be even and in [2, %d]", who,
                rotary_dim, index_head_dim);
  if (compress_ratio <= 0 || state_size <= 0 || compressed_page_size <= 0 ||
      (num_main_kv_heads > 0 && (main_page_size <= 0 || main_head_dim <= 0)))
    return fail(QSA_ERR_INVALID, "%s: ratio, ring size and page sizes must be positive", who);
  if (num_tokens == 0 && num_k_work == 0) return QSA_OK;
  if (!index_qk || !positions || !q_norm_weight || !k_norm_weight || !cos_sin_cache ||
      !index_q_out)
    return fail(QSA_ERR_INVALID, "%s: null index projection / weights / rotary cache", who);
  if (num_k_work > 0 && (!state_cache || !state_slots || !state_table || !query_start_loc ||
                         !logical_positions || !compressed_cache || !compressed_slots || !k_work))
    return fail(QSA_ERR_INVALID, "%s: null compression metadata or cache", who);
  if (num_main_kv_heads > 0 && num_tokens > 0 &&
      (!main_key || !main_value || !main_key_cache || !main_value_cache || !main_slots))
    return fail(QSA_ERR_INVALID, "%s: null main K/V or cache", who);
  if (index_row_stride < static_cast<int64_t>(num_index_heads + 1) * index_head_dim)
    return fail(QSA_ERR_INVALID, "%s: index row stride %lld < (heads + 1) * dim", who,
                (long long)index_row_stride);
  // rows are read and written as bf16 pairs
  if (!aligned(index_qk, 4) || index_row_stride % 2 || !aligned(index_q_out, 4) ||
      (num_k_work > 0 && (!aligned(state_cache, 4) || state_block_stride % 2 ||
                          state_token_stride % 2 || !aligned(compressed_cache, 4) ||
                          compressed_block_stride % 2 || compressed_token_stride % 2)))
    return fail(QSA_ERR_INVALID, "%s: index rows must be 4-byte aligned with even strides", who);
  PrepareParams p{};
  p.index_qk = static_cast<const __nv_bfloat16*>(index_qk);
  p.index_row_stride = index_row_stride;
  p.num_tokens = num_tokens;
  p.heads = num_index_heads;
  p.dim = index_head_dim;
  p.positions = positions;
  p.positions_stride = positions_stride;
  p.q_weight = static_cast<const __nv_bfloat16*>(q_norm_weight);
  p.k_weight = static_cast<const __nv_bfloat16*>(k_norm_weight);
  p.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin_cache);
  p.cos_sin_rows = cos_sin_rows;
  p.rotary = rotary_dim;
  p.eps = eps;
  p.index_q_out = static_cast<__nv_bfloat16*>(index_q_out);
  p.state_cache = static_cast<__nv_bfloat16*>(state_cache);
  p.state_block_stride = state_block_stride;
  p.state_token_stride = state_token_stride;
  p.state_size = state_size;
  p.state_blocks = state_blocks;
  p.state_slots = state_slots;
  p.state_table = state_table;
  p.state_table_stride = state_table_stride;
  p.query_start_loc = query_start_loc;
  p.num_requests = num_requests;
  p.logical_positions = logical_positions;
  p.compressed_cache = static_cast<__nv_bfloat16*>(compressed_cache);
  p.comp_block_stride = compressed_block_stride;
  p.comp_token_stride = compressed_token_stride;
  p.comp_page = compressed_page_size;
  p.comp_blocks = compressed_blocks;
  p.compressed_slots = compressed_slots;
  p.k_work = k_work;
  p.num_k_work = num_k_work;
  p.ratio = compress_ratio;
  p.main_key = static_cast<const __nv_bfloat16*>(main_key);
  p.main_value = static_cast<const __nv_bfloat16*>(main_value);
  p.main_key_cache = static_cast<__nv_bfloat16*>(main_key_cache);
  p.main_value_cache = static_cast<__nv_bfloat16*>(main_value_cache);
  const int64_t mk[3] = {main_key_token_stride, main_key_head_stride, main_key_dim_stride};
  const int64_t mv[3] = {main_value_token_stride, main_value_head_stride, main_value_dim_stride};
  const int64_t kc[4] = {main_key_cache_block_stride, main_key_cache_token_stride,
                         main_key_cache_head_stride, main_key_cache_dim_stride};
  const int64_t vc[4] = {main_value_cache_block_stride, main_value_cache_token_stride,
                         main_value_cache_head_stride, main_value_cache_dim_stride};
  bool vec = main_head_dim % 8 == 0 && aligned(main_key, 16) && aligned(main_value, 16) &&
             aligned(main_key_cache, 16) && aligned(main_value_cache, 16);
  for (int i = 0; i < 3; ++i) {
    p.mk_stride[i] = mk[i];
    p.mv_stride[i] = mv[i];
    vec = vec && (i == 2 ? mk[i] == 1 && mv[i] == 1 : mk[i] % 8 == 0 && mv[i] % 8 == 0);
  }
  for (int i = 0; i < 4; ++i) {
    p.kc_stride[i] = kc[i];
    p.vc_stride[i] = vc[i];
    vec = vec && (i == 3 ? kc[i] == 1 && vc[i] == 1 : kc[i] % 8 == 0 && vc[i] % 8 == 0);
  }
  p.main_slots = main_slots;
  p.kv_heads = num_main_kv_heads;
  p.main_dim = main_head_dim;
  p.main_page = main_page_size;
  p.main_blocks = main_blocks;
  p.main_vec = vec ? 1 : 0;
  p.err = device_error_word();
  cudaError_t e = launch_prepare(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, who);
  return QSA_OK;
}

// -------------------------------------------------------------- attention
size_t qsa_sparse_attention_workspace_bytes(int32_t rows, int32_t num_q_heads,
                                            int32_t num_kv_heads, int32_t head_dim,
                                            int32_t topk_width, int32_t use_decode_kernel) {
  if (rows <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads ||
      topk_width < 0)
    return 0;  // no launch for these shapes (qsa_sparse_attention rejects them)
  return plan_attention(rows, num_q_heads, num_kv_heads, head_dim, topk_width, use_decode_kernel)
      .workspace_bytes;
}

int qsa_sparse_attention(const void* q, int64_t q_row_stride, int64_t q_head_stride,
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
                         void* stream) {
  const char* who = "qsa_sparse_attention";
  if (rows < 0 || topk_width < 0) return fail(QSA_ERR_INVALID, "%s: negative size", who);
  if (rows == 0) return QSA_OK;
  if (!q || !k_cache || !v_cache || !indices || !out)
    return fail(QSA_ERR_INVALID, "%s: null pointer", who);
  if (!indices_are_physical && (!block_table || !token_to_req))
    return fail(QSA_ERR_INVALID, "%s: logical indices need block_table and token_to_req", who);
  if (head_dim != 64 && head_dim != 128)
    return fail(QSA_ERR_UNSUPPORTED, "%s: head_dim %d (supported: 64, 128)", who, head_dim);
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return fail(QSA_ERR_INVALID, "%s: %d query heads not a multiple of %d kv heads", who,
                num_q_heads, num_kv_heads);
  const int group = num_q_heads / num_kv_heads;
  if (group > 16)
    return fail(QSA_ERR_UNSUPPORTED, "%s: GQA group %d > 16", who, group);
  if (page_size <= 0 || num_blocks < 0) return fail(QSA_ERR_INVALID, "%s: bad page geometry", who);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || k_block_stride % 8 ||
      k_token_stride % 8 || k_head_stride % 8 || v_block_stride % 8 || v_token_stride % 8 ||
      v_head_stride % 8)
    return fail(QSA_ERR_INVALID, "%s: K/V cache rows must be 16-byte aligned", who);
  if (!aligned(q, 16) || q_row_stride % 8 || q_head_stride % 8)
    return fail(QSA_ERR_INVALID, "%s: q head rows must be 16-byte aligned", who);
  if (!aligned(out, 4) || out_row_stride % 2 || out_head_stride % 2)
    return fail(QSA_ERR_INVALID, "%s: out rows must be 4-byte aligned", who);
  const AttnPlan plan =
      plan_attention(rows, num_q_heads, num_kv_heads, head_dim, topk_width, use_decode_kernel);
  if (plan.workspace_bytes > 0 && (workspace == nullptr || workspace_bytes < plan.workspace_bytes))
    return fail(QSA_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", who, workspace_bytes,
                plan.workspace_bytes);
  if (plan.workspace_bytes > 0 && !aligned(workspace, 256))
    return fail(QSA_ERR_INVALID, "%s: workspace must be 256-byte aligned", who);
  AttnParams p = {};
  p.q = q;
  p.q_row_stride = q_row_stride;
  p.q_head_stride = q_head_stride;
  p.rows = rows;
  p.q_heads = num_q_heads;
  p.dim = head_dim;
  p.k_cache = k_cache;
  p.k_block_stride = k_block_stride;
  p.k_token_stride = k_token_stride;
  p.k_head_stride = k_head_stride;
  p.v_cache = v_cache;
  p.v_block_stride = v_block_stride;
  p.v_token_stride = v_token_stride;
  p.v_head_stride = v_head_stride;
  p.num_blocks = num_blocks;
  p.page_size = page_size;
  p.num_slots = static_cast<uint32_t>(
      std::min<int64_t>(static_cast<int64_t>(num_blocks) * page_size, 0xffffffffll));
  p.page_div = FastDiv(static_cast<uint32_t>(page_size));
  p.kv_heads = num_kv_heads;
  p.indices = indices;
  p.indices_row_stride = indices_row_stride;
  p.topk_width = topk_width;
  p.block_table = block_table;
  p.table_row_stride = table_row_stride;
  p.table_width = table_width;
  p.num_requests = num_requests;
  p.token_to_req = token_to_req;
  p.valid_counts = valid_counts;
  p.gate = gate;
  p.gate_row_stride = gate_row_stride;
  p.gate_head_stride = gate_head_stride;
  p.gate_dim_stride = gate_dim_stride;
  p.out = out;
  p.out_row_stride = out_row_stride;
  p.out_head_stride = out_head_stride;
  p.scale_log2 = static_cast<float>(std::pow(static_cast<double>(head_dim), -0.5) *
                                    1.4426950408889634);
  p.physical = indices_are_physical ? 1 : 0;
  // 2: each token's K||V rows of consecutive KV heads form one run (the
  //    [blocks, page, H_kv, K||V] layout); 1: K||V adjacent per head; 0: apart.
  const bool fused = (static_cast<const char*>(v_cache) ==
                      static_cast<const char*>(k_cache) + 2 * head_dim) &&
                     k_block_stride == v_block_stride && k_token_stride == v_token_stride &&
                     k_head_stride == v_head_stride;
  p.kv_fused = fused ? (k_head_stride == 2 * head_dim ? 2 : 1) : 0;
  p.slot_contig = k_block_stride == static_cast<int64_t>(page_size) * k_token_stride &&
                  k_token_stride == static_cast<int64_t>(num_kv_heads) * k_head_stride;
  p.gate_vec = gate != nullptr && gate_dim_stride == 1 && aligned(gate, 16) &&
               gate_row_stride % 8 == 0 && gate_head_stride % 8 == 0;
  p.out_vec = aligned(out, 16) && out_row_stride % 8 == 0 && out_head_stride % 8 == 0;
  p.pair_tiles = plan.pair_tiles;
  p.sk_ctas = plan.ctas;
  p.sk_units = plan.units;
  p.heads_per_unit = plan.heads_per_unit;
  p.partials = plan.partials;
  p.merge_pieces = plan.merge_pieces;
  if (plan.partials > 0) {
    p.part_o = static_cast<float*>(workspace);
    p.part_lse = reinterpret_cast<float*>(static_cast<char*>(workspace) + plan.lse_offset);
  }
  p.err = device_error_word();
  cudaError_t e = launch_attention(p, plan.split, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, who);
  return QSA_OK;
}

}  // extern "C"
