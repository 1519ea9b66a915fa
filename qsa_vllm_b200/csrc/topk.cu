// Exact per-row top-k over fp32 scores + expansion to token / slot ids (sm_100a).
//
// Semantics follow the reference selector (ops/csrc/topk.cu:107-180 expansion,
// :182-350 selection, :410-525 launchers): keys are the raw uint32 bit patterns
// of the scores, the K largest are selected with ties going to the lowest
// column, and the selection is emitted in ascending column order; rows whose
// length is <= K emit 0..length-1.
//
// Design (B200): one thread-block CLUSTER per row.  Each CTA of the cluster
// loads its contiguous slice of the row ONCE from HBM into shared memory
// (16-byte loads), and every later pass runs out of shared memory:
//   * radix select, most-significant digit first, 11/11/10-bit digits; the
//     per-CTA histograms are summed across the cluster through distributed
//     shared memory (DSMEM), so every CTA derives the same threshold;
//   * a pass stops early once the threshold digit's bucket is taken whole;
//   * the ordered write-out is a block scan of (strictly-above, tied) flags per
//     CTA plus an exchange of per-CTA totals over DSMEM: tied keys are taken
//     in ascending column order across the cluster, exactly as the reference.
// No global scratch memory is used: a row is selected in one launch whatever
// its width (the reference needs a partition + merge pass above 32768 columns).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace qsa {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 2048;
constexpr int kMaxSliceBytes = 160 * 1024;
constexpr int kMaxCluster = 16;

struct RowMeta {
  int seq, complete, tail_start, tail_count;
  const int32_t* trow;
};

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
  return m;
}

__device__ __forceinline__ int map_token(const TopkParams& p, const RowMeta& m, int token) {
  if (token < 0 || token >= m.seq) return -1;
  if (!p.physical) return token;
  const int lp = token / p.page_size;
  if (lp >= p.table_width) return -1;
  const int ph = m.trow[lp];
  return ph >= 0 ? ph * p.page_size + token % p.page_size : -1;
}

// Writes the selection of rank `rank` (block id or -1).
__device__ __forceinline__ void write_rank(const TopkParams& p, const RowMeta& m,
                                           int32_t* out_row, int rank, int block) {
  if (!p.expand) {
    out_row[rank] = block;
    return;
  }
  if (rank >= m.complete) return;
  const int first = block * p.ratio;
  for (int o = 0; o < p.ratio; ++o)
    out_row[static_cast<int64_t>(rank * p.ratio + o) * p.out_col_stride] =
        map_token(p, m, first + o);
}

// Causal tail, -1 fill and valid count (topk.cu:152-162).
__device__ __forceinline__ void finish_row(const TopkParams& p, const RowMeta& m,
                                           int32_t* out_row, int row) {
  const int expanded = m.complete * p.ratio;
  for (int col = max(expanded, 0) + static_cast<int>(threadIdx.x); col < p.out_width;
       col += kThreads) {
    const int off = col - expanded;
    out_row[static_cast<int64_t>(col) * p.out_col_stride] =
        (off < m.tail_count && off < p.ratio - 1) ? map_token(p, m, m.tail_start + off) : -1;
  }
  if (p.counts != nullptr && threadIdx.x == 0)
    p.counts[row] = min(expanded + m.tail_count, m.seq);
}

// Warp-aggregated shared-memory histogram increment (all 32 lanes call it).
__device__ __forceinline__ void hist_add(int* hist, bool valid, uint32_t bin) {
  const uint32_t key = valid ? bin : 0xffffffffu;
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  if (valid && (threadIdx.x & 31) == static_cast<unsigned>(__ffs(peers) - 1))
    atomicAdd(hist + bin, __popc(peers));
}

// Block-wide exclusive prefix sum of one int per thread; also returns the total.
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
    int w = warp_tmp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tmp[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  total = warp_tmp[kWarps - 1];
  const int before = warp == 0 ? 0 : warp_tmp[warp - 1];
  const int result = before + x - v;
  __syncthreads();
  return result;
}

__global__ void __launch_bounds__(kThreads, 1) topk_kernel(const TopkParams p) {
  extern __shared__ __align__(16) uint32_t keys[];
  __shared__ int hist[2][kBins];
  __shared__ int warp_tmp[kWarps];
  __shared__ int s_bin, s_remaining, s_bin_count;
  __shared__ int s_counts[2];  // (strictly above, tied) in this CTA's slice

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int crank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.x / C;
  const int tid = threadIdx.x;
  const int topk = p.topk;
  int32_t* out_row = p.output + static_cast<int64_t>(row) * p.out_row_stride;
  RowMeta m{};
  if (p.expand) m = row_meta(p, row);
  const int length = min(max(p.lengths[row], 0), p.width);

  if (length <= topk) {
    // Every column is selected (topk.cu:187-191); no score is read.
    const int n = p.expand ? max(m.complete, 0) : topk;
    for (int j = crank * kThreads + tid; j < n; j += C * kThreads)
      write_rank(p, m, out_row, j, j < length ? j : -1);
    if (crank == 0 && p.expand) finish_row(p, m, out_row, row);
    return;  // uniform across the cluster: no CTA reaches a cluster barrier
  }

  // ---- slice of this CTA, loaded once; pass-0 histogram fused with the load.
  const int per = ((length + C - 1) / C + 3) & ~3;
  const int begin = min(crank * per, length);
  const int n = min(begin + per, length) - begin;
  for (int b = tid; b < 2 * kBins; b += kThreads) (&hist[0][0])[b] = 0;
  __syncthreads();
  const float* src = p.scores + static_cast<int64_t>(row) * p.score_row_stride + begin;
  if (p.vec4) {
    const int n4 = (n + 3) >> 2;
    for (int base = 0; base < n4; base += kThreads) {
      const int i = base + tid;
      uint4 v = make_uint4(0, 0, 0, 0);
      const int e = i * 4;
      if (e + 3 < n) {
        v = __ldg(reinterpret_cast<const uint4*>(src) + i);
      } else if (e < n) {
        v.x = __float_as_uint(src[e]);
        if (e + 1 < n) v.y = __float_as_uint(src[e + 1]);
        if (e + 2 < n) v.z = __float_as_uint(src[e + 2]);
      }
      if (i < n4) reinterpret_cast<uint4*>(keys)[i] = v;
      hist_add(hist[0], e < n, v.x >> 21);
      hist_add(hist[0], e + 1 < n, v.y >> 21);
      hist_add(hist[0], e + 2 < n, v.z >> 21);
      hist_add(hist[0], e + 3 < n, v.w >> 21);
    }
  } else {
    for (int base = 0; base < n; base += kThreads) {
      const int i = base + tid;
      const uint32_t k = i < n ? __float_as_uint(src[i]) : 0u;
      if (i < n) keys[i] = k;
      hist_add(hist[0], i < n, k >> 21);
    }
  }
  __syncthreads();

  // ---- radix passes: digits of 11, 11, 10 bits from the most significant.
  uint32_t prefix = 0;  // resolved high bits: selection threshold is (key >> shift) == prefix
  int shift = 32;
  int remaining = topk;  // how many of the keys matching `prefix` are still to be taken
  int buf = 0;
  for (int pass = 0;; ++pass) {
    const int dbits = pass < 2 ? 11 : 10;
    const int dshift = shift - dbits;
    const uint32_t dmask = (1u << dbits) - 1u;
    if (pass > 0) {
      for (int b = tid; b < kBins; b += kThreads) hist[buf][b] = 0;
      __syncthreads();
      const int n4 = (n + 3) >> 2;
      for (int base = 0; base < n4; base += kThreads) {
        const int i = base + tid;
        const uint4 v = i < n4 ? reinterpret_cast<const uint4*>(keys)[i] : make_uint4(0, 0, 0, 0);
        const int e = i * 4;
        hist_add(hist[buf], e < n && (v.x >> shift) == prefix, (v.x >> dshift) & dmask);
        hist_add(hist[buf], e + 1 < n && (v.y >> shift) == prefix, (v.y >> dshift) & dmask);
        hist_add(hist[buf], e + 2 < n && (v.z >> shift) == prefix, (v.z >> dshift) & dmask);
        hist_add(hist[buf], e + 3 < n && (v.w >> shift) == prefix, (v.w >> dshift) & dmask);
      }
      __syncthreads();
    }
    cluster.sync();  // every CTA's histogram of this pass is complete

    // Thread t owns the two bins just below the 2t highest (descending order).
    const int nb = 1 << dbits;
    const int per_thread = nb / kThreads;  // 2 or 1
    const int b_hi = nb - 1 - per_thread * tid;
    const int b_lo = b_hi - 1;
    int h_hi = 0, h_lo = 0;
    for (int r = 0; r < C; ++r) {
      const int* rh = cluster.map_shared_rank(&hist[buf][0], r);
      h_hi += rh[b_hi];
      if (per_thread == 2) h_lo += rh[b_lo];
    }
    int total;
    const int above = block_exclusive_sum(h_hi + h_lo, warp_tmp, total);
    if (above < remaining && remaining <= above + h_hi) {
      s_bin = b_hi;
      s_remaining = remaining - above;
      s_bin_count = h_hi;
    } else if (per_thread == 2 && above + h_hi < remaining && remaining <= above + h_hi + h_lo) {
      s_bin = b_lo;
      s_remaining = remaining - above - h_hi;
      s_bin_count = h_lo;
    }
    __syncthreads();
    prefix = (prefix << dbits) | static_cast<uint32_t>(s_bin);
    remaining = s_remaining;
    shift = dshift;
    const bool done = s_bin_count == remaining || shift == 0;
    buf ^= 1;
    __syncthreads();
    if (done) break;
  }

  // ---- ordered write-out.  strict: (key >> shift) > prefix; tie: == prefix.
  int my_strict = 0, my_tie = 0;
  const int n4 = (n + 3) >> 2;
  for (int i = tid; i < n4; i += kThreads) {
    const uint4 v = reinterpret_cast<const uint4*>(keys)[i];
    const uint32_t kk[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (i * 4 + j < n) {
        const uint32_t d = kk[j] >> shift;
        my_strict += d > prefix;
        my_tie += d == prefix;
      }
    }
  }
  int tot_strict, tot_tie;
  block_exclusive_sum(my_strict, warp_tmp, tot_strict);
  block_exclusive_sum(my_tie, warp_tmp, tot_tie);
  if (tid == 0) {
    s_counts[0] = tot_strict;
    s_counts[1] = tot_tie;
  }
  cluster.sync();  // per-CTA totals visible cluster-wide
  int base_rank = 0, ties_before = 0;
  for (int r = 0; r < crank; ++r) {
    const int* rc = cluster.map_shared_rank(&s_counts[0], r);
    const int quota_r = min(max(remaining - ties_before, 0), rc[1]);
    base_rank += rc[0] + quota_r;
    ties_before += rc[1];
  }
  const int quota = min(max(remaining - ties_before, 0), tot_tie);

  int run_strict = 0, run_tie = 0;
  for (int base = 0; base < n4; base += kThreads) {
    const int i = base + tid;
    const uint4 v = i < n4 ? reinterpret_cast<const uint4*>(keys)[i] : make_uint4(0, 0, 0, 0);
    const uint32_t kk[4] = {v.x, v.y, v.z, v.w};
    int fs = 0, ft = 0;
    uint32_t flags = 0;  // bit 2j: strict, bit 2j+1: tie
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (i < n4 && i * 4 + j < n) {
        const uint32_t d = kk[j] >> shift;
        if (d > prefix) {
          flags |= 1u << (2 * j);
          ++fs;
        } else if (d == prefix) {
          flags |= 2u << (2 * j);
          ++ft;
        }
      }
    }
    int round_total;
    const int ex = block_exclusive_sum((fs << 16) | ft, warp_tmp, round_total);
    int sb = run_strict + (ex >> 16);
    int tb = run_tie + (ex & 0xffff);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int id = begin + i * 4 + j;
      if (flags & (1u << (2 * j))) {
        write_rank(p, m, out_row, base_rank + sb + min(tb, quota), id);
        ++sb;
      } else if (flags & (2u << (2 * j))) {
        if (tb < quota) write_rank(p, m, out_row, base_rank + sb + tb, id);
        ++tb;
      }
    }
    run_strict += round_total >> 16;
    run_tie += round_total & 0xffff;
  }
  if (crank == 0 && p.expand) finish_row(p, m, out_row, row);
  cluster.sync();  // no CTA leaves while a peer may still read its shared memory
}

int pow2_ceil(int x) {
  int c = 1;
  while (c < x) c <<= 1;
  return c;
}

}  // namespace

int topk_max_width() { return kMaxCluster * (kMaxSliceBytes / 4); }

cudaError_t launch_topk(const TopkParams& p0, cudaStream_t stream, int* plan_cluster) {
  TopkParams p = p0;
  if (p.rows <= 0) return cudaSuccess;
  const int sms = num_sms();
  int C = pow2_ceil((2 * sms + p.rows - 1) / p.rows);
  C = std::min(C, 8);
  int by_width = 1;
  while (by_width * 2 * 1024 <= p.width) by_width *= 2;
  C = std::max(1, std::min(C, by_width));
  auto cap_of = [&](int c) { return (((p.width + c - 1) / c) + 3) & ~3; };
  while (cap_of(C) * 4 > kMaxSliceBytes && C < kMaxCluster) C *= 2;
  if (cap_of(C) * 4 > kMaxSliceBytes) return cudaErrorInvalidValue;
  p.slice_cap = cap_of(C);
  const size_t smem = static_cast<size_t>(p.slice_cap) * 4;
  cudaError_t e = set_attr_once(reinterpret_cast<const void*>(topk_kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kMaxSliceBytes);
  if (e != cudaSuccess) return e;
  if (C > 8) {
    e = set_attr_once(reinterpret_cast<const void*>(topk_kernel), cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(C) * static_cast<unsigned>(p.rows), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (plan_cluster) *plan_cluster = C;
  return cudaLaunchKernelEx(&cfg, topk_kernel, p);
}

}  // namespace qsa
