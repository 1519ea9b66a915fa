// Per-row pieces of the top-k selection shared by the standalone top-k kernel
// (topk.cu) and the fused decode selection (select_decode.cu): the expansion
// of selected blocks to token or slot ids with the causal tail and counts
// (reference ops/csrc/topk.cu:107-180), and a block-wide prefix sum.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

struct RowMeta {
  int seq, complete, tail_start, tail_count;
  const int32_t* trow;
  // optional shared-memory copy of the first tcache_n entries of trow
  const int32_t* tcache;
  int tcache_n;
};

// Entry lp (< table width) of the row's block table.
__device__ __forceinline__ int table_entry(const RowMeta& m, int lp) {
  return lp < m.tcache_n ? m.tcache[lp] : __ldg(m.trow + lp);
}

// Expansion metadata of one row (topk.cu:165-180): integer division truncates
// toward zero exactly as in the reference.
__device__ __forceinline__ RowMeta row_meta(const TopkParams& p, int row) {
  RowMeta m;
  const int req = p.token_to_req[row];
  const bool mapped = req >= 0 && req < p.num_requests;
  m.seq = mapped ? p.seq_lens[req] : 0;
  const int pos = static_cast<int>(p.positions[row]);
  const int q1 = (pos + 1) / p.ratio;
  m.complete = min(min(q1, m.seq / p.ratio), p.topk);
  m.tail_start = q1 * p.ratio;
  m.tail_count = pos + 1 - m.tail_start;
  m.trow = p.physical ? p.table + static_cast<int64_t>(mapped ? req : 0) * p.table_row_stride
                      : nullptr;
  m.tcache = nullptr;
  m.tcache_n = 0;
  return m;
}

__device__ __forceinline__ int map_token(const TopkParams& p, const RowMeta& m, int token) {
  if (token < 0 || token >= m.seq) return -1;
  if (!p.physical) return token;
  int lp, off;
  p.page_div.divmod(token, lp, off);
  if (lp >= p.table_width) return -1;
  const int ph = table_entry(m, lp);
  return ph >= 0 ? ph * p.page_size + off : -1;
}

// Physical page of a selected block's first token, for the expansion fast
// path (page_size % ratio == 0: the block's tokens share one page).  -1 when
// unmapped or past the sequence.
__device__ __forceinline__ int block_page(const TopkParams& p, const RowMeta& m, int first) {
  if (first < 0 || first >= m.seq) return -1;
  int lp, off;
  p.page_div.divmod(first, lp, off);
  return lp < p.table_width ? table_entry(m, lp) : -1;
}

// Writes the expansion of `block` at rank `rank` (block -1 writes -1s).
// `ph` is block_page() when p.aligned_blocks (ignored otherwise).
__device__ __forceinline__ void store_block(const TopkParams& p, const RowMeta& m,
                                            int32_t* out_row, int rank, int block, int ph) {
  if (!p.expand) {
    out_row[rank] = block;
    return;
  }
  const int first = block * p.ratio;
  int32_t* dst = out_row + static_cast<int64_t>(rank) * p.ratio * p.out_col_stride;
  if (p.aligned_blocks) {
    int lp = 0, off = 0;
    if (ph >= 0) p.page_div.divmod(first, lp, off);
    for (int o = 0; o < p.ratio; ++o) {
      const int token = first + o;
      dst[static_cast<int64_t>(o) * p.out_col_stride] =
          (ph >= 0 && token < m.seq) ? ph * p.page_size + off + o : -1;
    }
  } else {
    for (int o = 0; o < p.ratio; ++o)
      dst[static_cast<int64_t>(o) * p.out_col_stride] = map_token(p, m, first + o);
  }
}

// Writes the selection of rank `rank` (block id or -1).
__device__ __forceinline__ void write_rank(const TopkParams& p, const RowMeta& m,
                                           int32_t* out_row, int rank, int block) {
  if (p.expand && rank >= m.complete) return;
  const int ph = (p.expand && p.aligned_blocks) ? block_page(p, m, block * p.ratio) : 0;
  store_block(p, m, out_row, rank, block, ph);
}

// Causal tail, -1 fill and valid count (topk.cu:152-162), by threads
// tid = 0..T-1 of a group.
template <int T>
__device__ __forceinline__ void finish_row(const TopkParams& p, const RowMeta& m,
                                           int32_t* out_row, int row, int tid) {
  const int expanded = m.complete * p.ratio;
  for (int col = max(expanded, 0) + tid; col < p.out_width; col += T) {
    const int off = col - expanded;
    out_row[static_cast<int64_t>(col) * p.out_col_stride] =
        (off < m.tail_count && off < p.ratio - 1) ? map_token(p, m, m.tail_start + off) : -1;
  }
  if (p.counts != nullptr && tid == 0) p.counts[row] = min(expanded + m.tail_count, m.seq);
}
template <int T>
__device__ __forceinline__ void finish_row(const TopkParams& p, const RowMeta& m,
                                           int32_t* out_row, int row) {
  finish_row<T>(p, m, out_row, row, static_cast<int>(threadIdx.x));
}

// Block-wide (W warps) exclusive prefix sum of one int per thread; also
// returns the total.
template <int W>
__device__ __forceinline__ int block_exclusive_sum(int v, int* warp_tmp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < W ? warp_tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < W) warp_tmp[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  total = warp_tmp[W - 1];
  const int before = warp == 0 ? 0 : warp_tmp[warp - 1];
  const int result = before + x - v;
  __syncthreads();
  return result;
}

}  // namespace
}  // namespace qsa
