// Indexer preparation and main K/V cache writes in one launch (sm_100a).
//
// Semantics follow the reference qsa_prepare (ops/prepare.py:16-228):
//  * index queries: per (token, index head), RMSNorm of the head's row of
//    index_qk, times q_weight, then rotate-half RoPE over the first `rotary`
//    dims at the token's position, with bf16 rounding after every post-norm
//    step (ops/prepare.py:16-46, :99-118);
//  * key compression: per (request, work item) of k_work, the fp32 mean of
//    `ratio` raw keys ending at the group boundary (this chunk's key part of
//    index_qk, or the request's ring cache for positions before the chunk),
//    rounded to bf16, normed and rotated at the group's first position with
//    k_weight, stored at the boundary token's compressed slot (:120-152);
//  * ring commit: work item 0 of a request writes the chunk's last
//    min(query_len, state_size) raw keys into the ring after its own group has
//    read it (:154-166); other work items only read this chunk's keys;
//  * main K/V: each (token, KV head) key and value row to its paged slot
//    (:81-97).  Slots < 0 are skipped.
//
// Design: every item is one warp (a CTA holds four independent warps).  A row
// of the index head dim lives in registers, D/32 values per lane; the RMS sum
// is a warp reduction and the rotate-half partner is read through the warp's
// slot of shared memory.  All of it is latency-bound, small work: one launch,
// no barriers across warps.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

constexpr int kPrepWarps = 4;
constexpr int kPrepThreads = kPrepWarps * 32;
constexpr int kMaxDim = 128;

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// RMSNorm + rotate-half RoPE of one row held as DPL values per lane (dims
// lane*DPL ..), in place; `row` is this warp's shared-memory scratch.
template <int DPL>
__device__ __forceinline__ void norm_rope(float (&v)[DPL], const PrepareParams& p,
                                          const __nv_bfloat16* gamma, int64_t pos, float* row) {
  constexpr int D = DPL * 32;
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
  // squares rounded before the sum (the reference kernel runs without FMA contraction)
#pragma unroll
  for (int i = 0; i < DPL; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  const float inv_rms = rsqrtf(warp_sum(ss) / D + p.eps);
  float scaled[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const float normalized = round_bf16(__fmul_rn(v[i], inv_rms));
    scaled[i] = round_bf16(__fmul_rn(normalized, __bfloat162float(gamma[lane * DPL + i])));
    row[lane * DPL + i] = scaled[i];
  }
  __syncwarp();
  const int half = p.rotary / 2;
  const __nv_bfloat16* cs = p.cos_sin + pos * p.rotary;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int d = lane * DPL + i;
    if (d < p.rotary) {
      const int channel = d % half;
      const float partner = d < half ? row[d + half] : row[d - half];
      const float rotated = d < half ? -partner : partner;
      const float first = round_bf16(__fmul_rn(scaled[i], __bfloat162float(cs[channel])));
      const float second = round_bf16(__fmul_rn(rotated, __bfloat162float(cs[half + channel])));
      v[i] = round_bf16(__fadd_rn(first, second));
    } else {
      v[i] = scaled[i];
    }
  }
  __syncwarp();  // `row` is reused by the warp's next item
}

template <int DPL>
__device__ __forceinline__ void load_row(float (&v)[DPL], const __nv_bfloat16* src) {
  const int lane = threadIdx.x & 31;
  if constexpr (DPL == 2) {
    const float2 f = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(src)[lane]);
    v[0] = f.x;
    v[1] = f.y;
  } else {
#pragma unroll
    for (int i = 0; i < DPL; ++i) v[i] = __bfloat162float(src[lane * DPL + i]);
  }
}

template <int DPL>
__device__ __forceinline__ void store_row(__nv_bfloat16* dst, const float (&v)[DPL]) {
  const int lane = threadIdx.x & 31;
  if constexpr (DPL == 2) {
    reinterpret_cast<__nv_bfloat162*>(dst)[lane] = __floats2bfloat162_rn(v[0], v[1]);
  } else {
#pragma unroll
    for (int i = 0; i < DPL; ++i) dst[lane * DPL + i] = __float2bfloat16_rn(v[i]);
  }
}

__device__ __forceinline__ bool in_range(int64_t i, int64_t n) { return i >= 0 && i < n; }

// fp32 sum, in member order, of the R raw keys first .. first+R-1 (this
// chunk's projection rows, or the request's ring block for positions before
// the chunk).  The rows of a batch are all loaded before the first add.
constexpr int kPoolBatch = 8;

template <int DPL>
__device__ __forceinline__ void pool_group(const PrepareParams& p, float (&acc)[DPL],
                                           int64_t first, int64_t chunk_start, int q0,
                                           int64_t block, int64_t key_offset) {
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
#pragma unroll 1
  for (int m0 = 0; m0 < p.ratio; m0 += kPoolBatch) {
    float x[kPoolBatch][DPL];
#pragma unroll
    for (int b = 0; b < kPoolBatch; ++b) {
      const int64_t src_pos = first + m0 + b;
      if (m0 + b < p.ratio) {
        const __nv_bfloat16* src =
            src_pos >= chunk_start
                ? p.index_qk + (q0 + src_pos - chunk_start) * p.index_row_stride + key_offset
                : p.state_cache + block * p.state_block_stride +
                      (src_pos % p.state_size) * p.state_token_stride;
        load_row<DPL>(x[b], src);
      }
    }
#pragma unroll
    for (int b = 0; b < kPoolBatch; ++b) {
      if (m0 + b < p.ratio) {
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] = __fadd_rn(acc[i], x[b][i]);
      }
    }
  }
}

template <int DPL>
__device__ __forceinline__ void index_query_item(const PrepareParams& p, int item, float* row) {
  const int token = item / p.heads, head = item % p.heads;
  const int64_t pos = p.positions[static_cast<int64_t>(token) * p.positions_stride];
  if (!in_range(pos, p.cos_sin_rows)) {
    if ((threadIdx.x & 31) == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  float v[DPL];
  load_row<DPL>(v, p.index_qk + static_cast<int64_t>(token) * p.index_row_stride +
                       head * DPL * 32);
  norm_rope<DPL>(v, p, p.q_weight, pos, row);
  store_row<DPL>(p.index_q_out + (static_cast<int64_t>(token) * p.heads + head) * DPL * 32, v);
}

template <int DPL>
__device__ __forceinline__ void compress_item(const PrepareParams& p, int item, float* row) {
  constexpr int D = DPL * 32;
  const int lane = threadIdx.x & 31;
  const int request = p.k_work[2 * item], work = p.k_work[2 * item + 1];
  if (request < 0) return;  // padding item
  if (request >= p.num_requests || work < 0) {
    if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  const int q0 = p.query_start_loc[request], q1 = p.query_start_loc[request + 1];
  const int qlen = q1 - q0;
  if (qlen <= 0) return;
  if (q0 < 0 || q1 > p.num_tokens) {
    if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  const int64_t chunk_end = p.logical_positions[q1 - 1];
  const int64_t chunk_start = chunk_end - qlen + 1;
  if (chunk_start < 0) {
    if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  const int R = p.ratio;
  const int64_t groups = (chunk_end + 1) / R - chunk_start / R;
  const int64_t key_offset = static_cast<int64_t>(p.heads) * D;
  if (work < groups) {
    const int64_t first_boundary = ((chunk_start + R) / R) * R - 1;
    const int64_t end = first_boundary + static_cast<int64_t>(work) * R;
    const int64_t first = end - (R - 1);
    const int64_t boundary_token = q0 + end - chunk_start;
    const int64_t block = p.state_table[static_cast<int64_t>(request) * p.state_table_stride];
    const int64_t slot = p.compressed_slots[boundary_token];
    const bool ring_ok = first >= chunk_start || in_range(block, p.state_blocks);
    if (!ring_ok || !in_range(first, p.cos_sin_rows)) {
      if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    } else {
      float acc[DPL];
      pool_group<DPL>(p, acc, first, chunk_start, q0, block, key_offset);
      float v[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) v[i] = round_bf16(acc[i] / R);
      norm_rope<DPL>(v, p, p.k_weight, first, row);
      if (in_range(slot, p.comp_blocks * p.comp_page)) {
        store_row<DPL>(p.compressed_cache + (slot / p.comp_page) * p.comp_block_stride +
                           (slot % p.comp_page) * p.comp_token_stride,
                       v);
      } else if (slot >= 0 && lane == 0) {
        record_error(p.err, kDeviceErrOutOfRange);
      }
    }
  }
  if (work == 0) {
    // The ring reads above went into registers in program order, per lane
    // and column, before any of the stores below can overwrite those slots.
    const int suffix = min(qlen, p.state_size);
    for (int t = q1 - suffix; t < q1; ++t) {
      const int64_t slot = p.state_slots[t];
      if (!in_range(slot, p.state_blocks * p.state_size)) {
        if (slot >= 0 && lane == 0) record_error(p.err, kDeviceErrOutOfRange);
        continue;
      }
      const __nv_bfloat16* src =
          p.index_qk + static_cast<int64_t>(t) * p.index_row_stride + key_offset;
      __nv_bfloat16* dst = p.state_cache + (slot / p.state_size) * p.state_block_stride +
                           (slot % p.state_size) * p.state_token_stride;
      if constexpr (DPL == 2) {
        reinterpret_cast<__nv_bfloat162*>(dst)[lane] =
            reinterpret_cast<const __nv_bfloat162*>(src)[lane];
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) dst[lane * DPL + i] = src[lane * DPL + i];
      }
    }
  }
}

__device__ __forceinline__ void main_kv_item(const PrepareParams& p, int item) {
  const int lane = threadIdx.x & 31;
  const int token = item / p.kv_heads, head = item % p.kv_heads;
  const int64_t slot = p.main_slots[token];
  if (!in_range(slot, p.main_blocks * p.main_page)) {
    if (slot >= 0 && lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  const int64_t block = slot / p.main_page, off = slot % p.main_page;
  const __nv_bfloat16* ks = p.main_key + token * p.mk_stride[0] + head * p.mk_stride[1];
  const __nv_bfloat16* vs = p.main_value + token * p.mv_stride[0] + head * p.mv_stride[1];
  __nv_bfloat16* kd =
      p.main_key_cache + block * p.kc_stride[0] + off * p.kc_stride[1] + head * p.kc_stride[2];
  __nv_bfloat16* vd =
      p.main_value_cache + block * p.vc_stride[0] + off * p.vc_stride[1] + head * p.vc_stride[2];
  if (p.main_vec) {
    // 8 bf16 per lane and operand; lanes 0..15 copy the key, 16..31 the value
    // (main_dim % 8 == 0 and 16-byte aligned rows, checked on the host)
    const int chunks = p.main_dim / 8;
    const int half = lane >> 4, sub = lane & 15;
    const uint4* src = reinterpret_cast<const uint4*>(half ? vs : ks);
    uint4* dst = reinterpret_cast<uint4*>(half ? vd : kd);
    for (int c = sub; c < chunks; c += 16) dst[c] = src[c];
  } else {
    for (int d = lane; d < p.main_dim; d += 32) {
      kd[d * p.kc_stride[3]] = ks[d * p.mk_stride[2]];
      vd[d * p.vc_stride[3]] = vs[d * p.mv_stride[2]];
    }
  }
}

template <int DPL>
__global__ void __launch_bounds__(kPrepThreads) prepare_kernel(const PrepareParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float rows[kPrepWarps][kMaxDim];
  const int warp = threadIdx.x >> 5;
  const int q_items = p.num_tokens * p.heads;
  const int main_items = p.num_tokens * p.kv_heads;
  const int total = p.num_k_work + q_items + main_items;
  for (int item = blockIdx.x * kPrepWarps + warp; item < total; item += gridDim.x * kPrepWarps) {
    if (item < p.num_k_work)
      compress_item<DPL>(p, item, rows[warp]);
    else if (item < p.num_k_work + q_items)
      index_query_item<DPL>(p, item - p.num_k_work, rows[warp]);
    else
      main_kv_item(p, item - p.num_k_work - q_items);
  }
}

// ------------------------------------------------------------ token path
// One warp per token: all index heads' query rows and all main K/V rows of the
// token, in 16-byte chunks of 8 bf16.  Chunk c of the query part belongs to
// head c / (D/8); a head's D/8 lanes reduce its squared sum with shuffles, and
// the rotate-half partner of a chunk is the chunk half/8 lanes away (rotary a
// multiple of 16, so a chunk never straddles half or rotary).  Every load of
// a group of passes is issued before any arithmetic or store.

__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// x holds bf16-representable values: packing truncates nothing
__device__ __forceinline__ uint4 pack8(const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = (__float_as_uint(x[2 * i]) >> 16) | (__float_as_uint(x[2 * i + 1]) & 0xffff0000u);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr int kPassGroup = 2;  // 32-chunk passes whose loads are in flight together

template <int D>
__device__ __forceinline__ void token_queries(const PrepareParams& p, int token, int64_t pos) {
  constexpr int kLanesPerHead = D / 8;
  const int lane = threadIdx.x & 31;
  const int chunks = p.heads * kLanesPerHead;
  const int half = p.rotary / 2;
  const int shift = half / 8;
  const uint4* src = reinterpret_cast<const uint4*>(
      p.index_qk + static_cast<int64_t>(token) * p.index_row_stride);
  uint4* dst = reinterpret_cast<uint4*>(p.index_q_out + static_cast<int64_t>(token) * p.heads * D);
  const __nv_bfloat16* cs = p.cos_sin + pos * p.rotary;
  const int d0 = (lane % kLanesPerHead) * 8;   // first dim of this lane's chunk in its head
  const bool rot = d0 < p.rotary;
  const int channel = d0 % half;
  const int partner_lane = d0 < half ? lane + shift : (rot ? lane - shift : lane);
  // per-lane constants: gamma, cosines and sines of this chunk's dims
  float gamma[8], cosv[8], sinv[8];
  unpack8(reinterpret_cast<const uint4*>(p.q_weight)[d0 / 8], gamma);
  if (rot) {
    unpack8(*reinterpret_cast<const uint4*>(cs + channel), cosv);
    unpack8(*reinterpret_cast<const uint4*>(cs + half + channel), sinv);
  }
#pragma unroll 1
  for (int c0 = 0; c0 < chunks; c0 += 32 * kPassGroup) {
    uint4 raw[kPassGroup];
#pragma unroll
    for (int j = 0; j < kPassGroup; ++j) {
      const int c = c0 + j * 32 + lane;
      raw[j] = c < chunks ? src[c] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < kPassGroup; ++j) {
      if (c0 + j * 32 >= chunks) break;   // warp-uniform
      const int c = c0 + j * 32 + lane;
      float x[8];
      unpack8(raw[j], x);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
#pragma unroll
      for (int o = 1; o < kLanesPerHead; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv_rms = rsqrtf(ss / D + p.eps);
      float scaled[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        scaled[i] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[i], inv_rms)), gamma[i]));
      const uint4 mine = pack8(scaled);
      uint4 other;
      other.x = __shfl_sync(0xffffffffu, mine.x, partner_lane);
      other.y = __shfl_sync(0xffffffffu, mine.y, partner_lane);
      other.z = __shfl_sync(0xffffffffu, mine.z, partner_lane);
      other.w = __shfl_sync(0xffffffffu, mine.w, partner_lane);
      float out[8];
      if (rot) {
        float partner[8];
        unpack8(other, partner);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float rotated = d0 < half ? -partner[i] : partner[i];
          const float first = round_bf16(__fmul_rn(scaled[i], cosv[i]));
          const float second = round_bf16(__fmul_rn(rotated, sinv[i]));
          out[i] = round_bf16(__fadd_rn(first, second));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = scaled[i];
      }
      if (c < chunks) dst[c] = pack8(out);
    }
  }
}

// Main K/V rows of one token in 16-byte chunks (chunk c: head c / (dim/8)).
struct MainChunks {
  uint4 k[kPassGroup], v[kPassGroup];
};

__device__ __forceinline__ void load_main(const PrepareParams& p, int token, int c0,
                                          MainChunks& m) {
  const int lane = threadIdx.x & 31;
  const int per_head = p.main_dim / 8;
  const int chunks = p.kv_heads * per_head;
  const __nv_bfloat16* ks = p.main_key + token * p.mk_stride[0];
  const __nv_bfloat16* vs = p.main_value + token * p.mv_stride[0];
#pragma unroll
  for (int j = 0; j < kPassGroup; ++j) {
    const int c = c0 + j * 32 + lane;
    if (c < chunks) {
      const int h = c / per_head, w = (c % per_head) * 8;
      m.k[j] = *reinterpret_cast<const uint4*>(ks + h * p.mk_stride[1] + w);
      m.v[j] = *reinterpret_cast<const uint4*>(vs + h * p.mv_stride[1] + w);
    }
  }
}

__device__ __forceinline__ void store_main(const PrepareParams& p, int64_t slot, int c0,
                                           const MainChunks& m) {
  const int lane = threadIdx.x & 31;
  const int per_head = p.main_dim / 8;
  const int chunks = p.kv_heads * per_head;
  const int64_t block = slot / p.main_page, off = slot % p.main_page;
  __nv_bfloat16* kd = p.main_key_cache + block * p.kc_stride[0] + off * p.kc_stride[1];
  __nv_bfloat16* vd = p.main_value_cache + block * p.vc_stride[0] + off * p.vc_stride[1];
#pragma unroll
  for (int j = 0; j < kPassGroup; ++j) {
    const int c = c0 + j * 32 + lane;
    if (c < chunks) {
      const int h = c / per_head, w = (c % per_head) * 8;
      *reinterpret_cast<uint4*>(kd + h * p.kc_stride[2] + w) = m.k[j];
      *reinterpret_cast<uint4*>(vd + h * p.vc_stride[2] + w) = m.v[j];
    }
  }
}

// compress_item with the ring commit in 16-byte chunks spread over the warp.
// The ring block and, for work item 0, the first commit rows are loaded
// before the group's arithmetic; the commit stores follow it.
template <int D>
__device__ __forceinline__ void compress_item_fast(const PrepareParams& p, int item, float* row) {
  constexpr int DPL = D / 32;
  constexpr int kRowChunks = D / 8;
  const int lane = threadIdx.x & 31;
  const int request = p.k_work[2 * item], work = p.k_work[2 * item + 1];
  if (request < 0) return;  // padding item
  if (request >= p.num_requests || work < 0) {
    if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  const int q0 = p.query_start_loc[request], q1 = p.query_start_loc[request + 1];
  const int64_t block = p.state_table[static_cast<int64_t>(request) * p.state_table_stride];
  const int qlen = q1 - q0;
  if (qlen <= 0) return;
  if (q0 < 0 || q1 > p.num_tokens) {
    if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  const int64_t chunk_end = p.logical_positions[q1 - 1];
  const int64_t key_offset = static_cast<int64_t>(p.heads) * D;
  const int suffix = min(qlen, p.state_size);
  const int commit_chunks = work == 0 ? suffix * kRowChunks : 0;
  uint4 cdata[kPassGroup];
  int64_t cslot[kPassGroup];
  const auto load_commit = [&](int c0) {
#pragma unroll
    for (int j = 0; j < kPassGroup; ++j) {
      const int c = c0 + j * 32 + lane;
      if (c < commit_chunks) {
        const int64_t t = q1 - suffix + c / kRowChunks;
        cslot[j] = p.state_slots[t];
        cdata[j] = *reinterpret_cast<const uint4*>(p.index_qk + t * p.index_row_stride +
                                                   key_offset + (c % kRowChunks) * 8);
      }
    }
  };
  const auto store_commit = [&](int c0) {
#pragma unroll
    for (int j = 0; j < kPassGroup; ++j) {
      const int c = c0 + j * 32 + lane;
      if (c < commit_chunks) {
        const int64_t slot = cslot[j];
        if (in_range(slot, p.state_blocks * p.state_size)) {
          *reinterpret_cast<uint4*>(p.state_cache + (slot / p.state_size) * p.state_block_stride +
                                    (slot % p.state_size) * p.state_token_stride +
                                    (c % kRowChunks) * 8) = cdata[j];
        } else if (slot >= 0) {
          record_error(p.err, kDeviceErrOutOfRange);
        }
      }
    }
  };
  load_commit(0);
  const int64_t chunk_start = chunk_end - qlen + 1;
  if (chunk_start < 0) {
    if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  const int R = p.ratio;
  const int64_t groups = (chunk_end + 1) / R - chunk_start / R;
  if (work < groups) {
    const int64_t first_boundary = ((chunk_start + R) / R) * R - 1;
    const int64_t end = first_boundary + static_cast<int64_t>(work) * R;
    const int64_t first = end - (R - 1);
    const int64_t boundary_token = q0 + end - chunk_start;
    const int64_t slot = p.compressed_slots[boundary_token];
    const bool ring_ok = first >= chunk_start || in_range(block, p.state_blocks);
    if (!ring_ok || !in_range(first, p.cos_sin_rows)) {
      if (lane == 0) record_error(p.err, kDeviceErrOutOfRange);
    } else {
      float acc[DPL];
      pool_group<DPL>(p, acc, first, chunk_start, q0, block, key_offset);
      float v[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) v[i] = round_bf16(acc[i] / R);
      norm_rope<DPL>(v, p, p.k_weight, first, row);
      if (in_range(slot, p.comp_blocks * p.comp_page)) {
        store_row<DPL>(p.compressed_cache + (slot / p.comp_page) * p.comp_block_stride +
                           (slot % p.comp_page) * p.comp_token_stride,
                       v);
      } else if (slot >= 0 && lane == 0) {
        record_error(p.err, kDeviceErrOutOfRange);
      }
    }
  }
  if (commit_chunks > 0) {
    // the group's ring loads were consumed above (they fed `acc`); order them
    // before the commit stores of the other lanes
    __syncwarp();
    store_commit(0);
#pragma unroll 1
    for (int c0 = 32 * kPassGroup; c0 < commit_chunks; c0 += 32 * kPassGroup) {
      load_commit(c0);
      store_commit(c0);
    }
  }
}

// One token: the first chunk group of its main K/V rows is loaded before the
// query work and stored after it; later groups (more than 32 * kPassGroup
// chunks per operand) follow.
template <int D>
__device__ __forceinline__ void token_item(const PrepareParams& p, int token) {
  const int64_t pos = p.positions[static_cast<int64_t>(token) * p.positions_stride];
  const int64_t slot = p.kv_heads > 0 ? p.main_slots[token] : -1;
  const bool vec = p.kv_heads > 0 && p.main_vec;
  MainChunks m;
  if (vec) load_main(p, token, 0, m);
  if (in_range(pos, p.cos_sin_rows)) {
    token_queries<D>(p, token, pos);
  } else if ((threadIdx.x & 31) == 0) {
    record_error(p.err, kDeviceErrOutOfRange);
  }
  if (p.kv_heads == 0) return;
  if (!in_range(slot, p.main_blocks * p.main_page)) {
    if (slot >= 0 && (threadIdx.x & 31) == 0) record_error(p.err, kDeviceErrOutOfRange);
    return;
  }
  if (vec) {
    store_main(p, slot, 0, m);
    const int chunks = p.kv_heads * (p.main_dim / 8);
#pragma unroll 1
    for (int c0 = 32 * kPassGroup; c0 < chunks; c0 += 32 * kPassGroup) {
      load_main(p, token, c0, m);
      store_main(p, slot, c0, m);
    }
  } else {
    for (int h = 0; h < p.kv_heads; ++h) main_kv_item(p, token * p.kv_heads + h);
  }
}

// Items: [k_work items][tokens].
template <int D>
__global__ void __launch_bounds__(kPrepThreads) prepare_token_kernel(const PrepareParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float rows[kPrepWarps][kMaxDim];
  const int warp = threadIdx.x >> 5;
  const int total = p.num_k_work + p.num_tokens;
  for (int item = blockIdx.x * kPrepWarps + warp; item < total; item += gridDim.x * kPrepWarps) {
    if (item < p.num_k_work)
      compress_item_fast<D>(p, item, rows[warp]);
    else
      token_item<D>(p, item - p.num_k_work);
  }
}

}  // namespace

// The token path needs 16-byte chunks that never straddle the rotary halves.
static bool prepare_token_path(const PrepareParams& p) {
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return p.rotary % 16 == 0 && a16(p.index_qk) && p.index_row_stride % 8 == 0 &&
         a16(p.index_q_out) && a16(p.q_weight) && a16(p.cos_sin) &&
         (p.num_k_work == 0 || (a16(p.state_cache) && p.state_block_stride % 8 == 0 &&
                                p.state_token_stride % 8 == 0));
}

cudaError_t launch_prepare(const PrepareParams& p, cudaStream_t stream) {
  const bool token_path = prepare_token_path(p);
  const int64_t total =
      static_cast<int64_t>(p.num_k_work) +
      static_cast<int64_t>(p.num_tokens) * (token_path ? 1 : p.heads + p.kv_heads);
  if (total <= 0) return cudaSuccess;
  const int blocks = static_cast<int>(std::min<int64_t>((total + kPrepWarps - 1) / kPrepWarps,
                                                        num_sms() * 16));
  const dim3 grid(blocks), block(kPrepThreads);
  if (token_path) {
    if (p.dim == 64)
      return count_launches(launch_kernel(prepare_token_kernel<64>, grid, block, 0, stream, 1, p));
    if (p.dim == 128)
      return count_launches(launch_kernel(prepare_token_kernel<128>, grid, block, 0, stream, 1, p));
  } else {
    if (p.dim == 64)
      return count_launches(launch_kernel(prepare_kernel<2>, grid, block, 0, stream, 1, p));
    if (p.dim == 128)
      return count_launches(launch_kernel(prepare_kernel<4>, grid, block, 0, stream, 1, p));
  }
  return cudaErrorInvalidValue;
}

}  // namespace qsa
