// Exact per-row top-k over fp32 scores + expansion to token / slot ids (sm_100a).
//
// Semantics follow the reference selector (ops/csrc/topk.cu:107-180 expansion,
// :182-350 selection, :410-525 launchers): keys are the raw uint32 bit patterns
// of the scores, the K largest are selected with ties going to the lowest
// column, and the selection is emitted in ascending column order; rows whose
// length is <= K emit 0..length-1.
//
// Design (B200), latency first (a decode step selects over only ~2-8 MB):
//   * one CTA per row slice, sized to the row: 256 or 512 threads for rows of
//     up to 2048 / 4096 keys (prefill rows; several CTAs share an SM), 1024
//     threads above; each thread keeps its keys (8, or 32 for very wide rows)
//     in REGISTERS after one coalesced 16-byte load pass from HBM, so every
//     radix pass re-reads registers, not memory;
//   * radix select, most-significant digit first, in digits of up to 11
//     bits below the high bits shared by every key of the row (found from the
//     row's min and max key first: scores of similar magnitude share sign and
//     exponent bits, which would otherwise crowd a few histogram bins), with
//     shared-memory histograms (double-buffered, so a pass needs a single
//     barrier); a pass stops early once the threshold digit's bucket is taken
//     whole;
//   * the ordered write-out ranks every selected key with ONE block scan of
//     per-chunk (above, tied) counters;
//   * rows wider than one CTA's slice run as a thread-block CLUSTER: the
//     per-CTA histograms are summed through distributed shared memory (DSMEM)
//     and every CTA derives the same threshold; tied keys are then taken in
//     ascending column order across the cluster from per-CTA totals;
//   * no global scratch memory: one launch whatever the width (the reference
//     needs a partition + merge pass above 32768 columns).
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "topk_rows.cuh"

namespace cg = cooperative_groups;

namespace qsa {
namespace {

constexpr int kThreads = 1024;  // widest CTA (rows above 4096 keys and clusters)
constexpr int kBins = 2048;
constexpr int kMaxCluster = 16;
constexpr int kMaxSelBytes = 192 * 1024;  // selected ids of one CTA: up to 49152 blocks

// Shared-memory histogram increment.  The digits lie below the row's common
// high bits, so lanes rarely collide on a bin.
__device__ __forceinline__ void hist_add(int* hist, bool valid, uint32_t bin) {
  if (valid) atomicAdd(hist + bin, 1);
}

// Block-wide exclusive prefix sums of NC counters per thread in one round
// (one barrier pair): ex[c] = sum of v[c] over lower threads, tot[c] = sum
// over the block of W warps.  `tmp` holds W * NC ints.
template <int NC, int W>
__device__ __forceinline__ void block_scan_multi(const int (&v)[NC], int (&ex)[NC],
                                                 int (&tot)[NC], int* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) x[c] = v[c];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int y = __shfl_up_sync(0xffffffffu, x[c], o);
      if (lane >= o) x[c] += y;
    }
  }
  if (lane == 31) {
#pragma unroll
    for (int c = 0; c < NC; ++c) tmp[warp * NC + c] = x[c];
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      int w = lane < W ? tmp[lane * NC + c] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      __syncwarp();
      if (lane < W) tmp[lane * NC + c] = w;  // inclusive warp prefix
    }
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    tot[c] = tmp[(W - 1) * NC + c];
    ex[c] = (warp == 0 ? 0 : tmp[(warp - 1) * NC + c]) + x[c] - v[c];
  }
  __syncthreads();
}

// T threads, V keys per thread; the slice of a CTA is T * V keys, stored as
// V/4 chunks of T float4 (thread t holds keys 4*(c*T+t)+0..3).
template <int T, int V>
__global__ void __launch_bounds__(T, 1024 / T) topk_kernel(const TopkParams p) {
  constexpr int kChunks = V / 4;
  constexpr int kWarps = T / 32;
  constexpr int kPer = kBins / T > 0 ? kBins / T : 1;  // most bins one thread ranks
  extern __shared__ int sel[];  // selected column ids of this CTA, by rank (topk entries)
  __shared__ int hist[2][kBins];
  __shared__ int warp_tmp[kWarps * kChunks * 2];
  __shared__ uint32_t s_minmax[2][kWarps];
  __shared__ uint32_t s_range[2];  // this CTA's (min, max) key
  __shared__ int s_bin, s_remaining, s_bin_count;
  __shared__ int s_counts[2];  // (strictly above, tied) in this CTA's slice

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int crank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.x / C;
  const int tid = threadIdx.x;
  const int topk = p.topk;
  int32_t* out_row = p.output + static_cast<int64_t>(row) * p.out_row_stride;
  // The row's metadata (request, sequence length, position, visible count,
  // block table) is step metadata that the preceding kernel (the indexer)
  // does not write: it is read before waiting on that kernel, so these
  // dependent loads overlap its tail.  The scores are read after the wait.
  RowMeta m{};
  if (p.expand) m = row_meta(p, row);
  const int length =
      min(max(p.lengths != nullptr ? p.lengths[row]
                                   : visible_of(p.positions, p.seq_lens, p.num_requests,
                                                p.token_to_req, p.ratio, row),
              0),
          p.width);
  pdl_wait();
  pdl_trigger();

  if (length <= topk || topk == 0) {
    // Every column is selected (topk.cu:187-191), or none is asked for; no
    // score is read.
    const int n = p.expand ? max(m.complete, 0) : topk;
    for (int j = crank * T + tid; j < n; j += C * T)
      write_rank(p, m, out_row, j, j < length ? j : -1);
    if (crank == 0 && p.expand) finish_row<T>(p, m, out_row, row);
    return;  // uniform across the cluster: no CTA reaches a cluster barrier
  }

  // ---- this CTA's slice -> registers (one pass over HBM).
  const int per = ((length + C - 1) / C + 3) & ~3;
  const int begin = min(crank * per, length);
  const int n = min(begin + per, length) - begin;
  for (int b = tid; b < 2 * kBins; b += T) (&hist[0][0])[b] = 0;
  const float* src = p.scores + static_cast<int64_t>(row) * p.score_row_stride + begin;
  uint32_t key[V];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int e = 4 * (c * T + tid);
    if (p.vec4 && e + 3 < n) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + e));
      key[4 * c] = v.x;
      key[4 * c + 1] = v.y;
      key[4 * c + 2] = v.z;
      key[4 * c + 3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) key[4 * c + j] = e + j < n ? __float_as_uint(src[e + j]) : 0u;
    }
  }
  auto valid_at = [&](int i) { return 4 * ((i / 4) * T + tid) + (i % 4) < n; };

  // ---- min and max key of the row: their common high bits are shared by
  // every key and need no radix pass.
  uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if (valid_at(i)) {
      kmin = min(kmin, key[i]);
      kmax = max(kmax, key[i]);
    }
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  if ((tid & 31) == 0) {
    s_minmax[0][tid >> 5] = kmin;
    s_minmax[1][tid >> 5] = kmax;
  }
  __syncthreads();
  if (tid < 32) {
    uint32_t a = tid < kWarps ? s_minmax[0][tid] : 0xffffffffu;
    uint32_t z = tid < kWarps ? s_minmax[1][tid] : 0u;
    a = __reduce_min_sync(0xffffffffu, a);
    z = __reduce_max_sync(0xffffffffu, z);
    if (tid == 0) {
      s_range[0] = a;
      s_range[1] = z;
    }
  }
  __syncthreads();
  kmin = s_range[0];
  kmax = s_range[1];
  if (C > 1) {
    cluster.sync();  // every CTA's (min, max) published
    for (int r = 0; r < C; ++r) {
      const uint32_t* rr = cluster.map_shared_rank(&s_range[0], r);
      kmin = min(kmin, rr[0]);
      kmax = max(kmax, rr[1]);
    }
  }
  const int common = kmin == kmax ? 32 : __clz(kmin ^ kmax);  // shared high bits

  // ---- radix passes over the bits below the common prefix, digits of <= 11.
  int shift = 32 - common;
  uint32_t prefix = common == 0 ? 0u : kmax >> shift;  // resolved high bits of the threshold
  int remaining = topk;  // how many of the keys matching `prefix` are still to be taken
  for (int pass = 0; shift > 0; ++pass) {
    const int b = pass & 1;
    const int dbits = shift < 11 ? shift : 11;
    const int dshift = shift - dbits;
    const uint32_t dmask = (1u << dbits) - 1u;
    if (pass >= 2) {  // hist[b] was last read (cluster-wide) two passes ago
      for (int i = tid; i < kBins; i += T) hist[b][i] = 0;
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const bool in = valid_at(i) && (shift >= 32 || (key[i] >> shift) == prefix);
      hist_add(hist[b], in, (key[i] >> dshift) & dmask);
    }
    __syncthreads();
    if (C > 1) cluster.sync();  // every CTA's histogram of this pass is complete

    // Thread t owns per_thread bins just below the per_thread*t highest
    // (descending order); with fewer bins than threads, one bin each.
    const int nb = 1 << dbits;
    const int per_thread = nb >= T ? nb / T : 1;  // <= kPer
    const bool owns = per_thread * tid < nb;
    const int top = nb - 1 - per_thread * tid;
    int h[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) h[j] = 0;
    if (owns) {
      if (C > 1) {
#pragma unroll
        for (int r = 0; r < kMaxCluster; ++r) {
          if (r < C) {
            const int* rh = cluster.map_shared_rank(&hist[b][0], r);
#pragma unroll
            for (int j = 0; j < kPer; ++j)
              if (j < per_thread) h[j] += rh[top - j];
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < kPer; ++j)
          if (j < per_thread) h[j] = hist[b][top - j];
      }
    }
    int total, mine_sum = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) mine_sum += h[j];
    int above = block_exclusive_sum<kWarps>(mine_sum, warp_tmp, total);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (owns && j < per_thread && above < remaining && remaining <= above + h[j]) {
        s_bin = top - j;
        s_remaining = remaining - above;
        s_bin_count = h[j];
      }
      above += h[j];
    }
    __syncthreads();
    prefix = (shift >= 32 ? 0u : (prefix << dbits)) | static_cast<uint32_t>(s_bin);
    remaining = s_remaining;
    shift = dshift;
    const bool done = s_bin_count == remaining;
    __syncthreads();  // s_* are rewritten by the next pass
    if (done) break;
  }

  // ---- ordered write-out.  strict: (key >> shift) > prefix; tie: == prefix.
  // (shift < 32 here: at least the sign bit was resolved or shared.)
  // Counters per chunk c, packed (strict << 16 | tie); one block scan ranks
  // every key of the CTA's slice in column order.
  int cnt[kChunks], ex[kChunks], tot[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    int fs = 0, ft = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t d = key[4 * c + j] >> shift;
      const bool v = valid_at(4 * c + j);
      fs += v && d > prefix;
      ft += v && d == prefix;
    }
    cnt[c] = (fs << 16) | ft;
  }
  block_scan_multi<kChunks, kWarps>(cnt, ex, tot, warp_tmp);
  int tot_strict = 0, tot_tie = 0;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    tot_strict += tot[c] >> 16;
    tot_tie += tot[c] & 0xffff;
  }
  int base_rank = 0, ties_before = 0;
  if (C > 1) {
    if (tid == 0) {
      s_counts[0] = tot_strict;
      s_counts[1] = tot_tie;
    }
    cluster.sync();  // per-CTA totals visible cluster-wide
    for (int r = 0; r < crank; ++r) {
      const int* rc = cluster.map_shared_rank(&s_counts[0], r);
      const int quota_r = min(max(remaining - ties_before, 0), rc[1]);
      base_rank += rc[0] + quota_r;
      ties_before += rc[1];
    }
  }
  const int quota = min(max(remaining - ties_before, 0), tot_tie);

  // Selection: each selected column id goes to sel[its rank - base_rank]
  // (ascending column order = rank order, ties to the lowest columns).
  int run_strict = 0, run_tie = 0;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    int sb = run_strict + (ex[c] >> 16);
    int tb = run_tie + (ex[c] & 0xffff);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t d = key[4 * c + j] >> shift;
      const bool v = valid_at(4 * c + j);
      const int id = begin + 4 * (c * T + tid) + j;
      if (v && d > prefix) {
        sel[sb + min(tb, quota)] = id;
        ++sb;
      } else if (v && d == prefix) {
        if (tb < quota) sel[sb + tb] = id;
        ++tb;
      }
    }
    run_strict += tot[c] >> 16;
    run_tie += tot[c] & 0xffff;
  }
  __syncthreads();
  // Expansion: one rank per thread and iteration, so consecutive threads
  // write consecutive output columns and issue their page lookups together.
  const int mine = tot_strict + quota;
  for (int i = tid; i < mine; i += T) {
    const int rank = base_rank + i;
    if (p.expand && rank >= m.complete) break;
    write_rank(p, m, out_row, rank, sel[i]);
  }
  if (crank == 0 && p.expand) finish_row<T>(p, m, out_row, row);
  if (C > 1) cluster.sync();  // no CTA leaves while a peer may still read its shared memory
}

// Rows of up to kWarpRowKeys keys (prefill rows): ONE WARP per row, the
// same selection and ordering as topk_kernel with no barrier and no shared
// histogram.  A lane holds 64 keys in registers (16 coalesced float4 loads:
// key 4c+e is column 4(32c + lane) + e).  The K-th largest key T is built
// one bit at a time below the row's common high bits: a bit is kept when at
// least K keys are >= the candidate (one warp reduction per bit), stopping
// early once exactly K keys are >= T.  Keys > T are selected, keys == T in
// column order up to the quota; ids go to the warp's shared-memory buffer by
// rank, then the expansion writes them out.
constexpr int kWarpRowKeys = 2048;
constexpr int kRowWarps = 8;  // rows per CTA
template <int SELCAP>
__global__ void __launch_bounds__(kRowWarps * 32, 2) topk_warp_kernel(const TopkParams p) {
  constexpr int kV = kWarpRowKeys / 32;  // keys per lane
  constexpr int kChunks = kV / 4;
  extern __shared__ int smem_w[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* sel = smem_w + warp * SELCAP;
  const int row = blockIdx.x * kRowWarps + warp;
  const bool live = row < p.rows;
  const int topk = p.topk;
  int32_t* out_row = p.output + static_cast<int64_t>(live ? row : 0) * p.out_row_stride;
  // row metadata before the wait, as in topk_kernel
  RowMeta m{};
  if (live && p.expand) m = row_meta(p, row);
  const int length =
      live ? min(max(p.lengths != nullptr ? p.lengths[row]
                                          : visible_of(p.positions, p.seq_lens, p.num_requests,
                                                       p.token_to_req, p.ratio, row),
                     0),
                 p.width)
           : 0;
  pdl_wait();
  pdl_trigger();
  if (!live) return;

  if (length <= topk || topk == 0) {  // all columns selected (topk.cu:187-191), or none asked
    const int n = p.expand ? max(m.complete, 0) : topk;
    for (int j = lane; j < n; j += 32) write_rank(p, m, out_row, j, j < length ? j : -1);
    if (p.expand) finish_row<32>(p, m, out_row, row, lane);
    return;
  }

  const float* src = p.scores + static_cast<int64_t>(row) * p.score_row_stride;
  uint32_t key[kV];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int e = 4 * (c * 32 + lane);
    if (p.vec4 && e + 3 < length) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + e));
      key[4 * c] = v.x;
      key[4 * c + 1] = v.y;
      key[4 * c + 2] = v.z;
      key[4 * c + 3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        key[4 * c + j] = e + j < length ? __float_as_uint(src[e + j]) : 0u;
    }
  }
  // Slots past the row's length hold key 0 and come last in column order.
  // They are never >= a candidate (candidates are >= 1) nor > T; as keys
  // == T (only when T = 0) they follow every valid tie, so the quota never
  // reaches them, and they are subtracted from the tie count.
  uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
  for (int i = 0; i < kV; ++i) {
    const bool v = 4 * ((i / 4) * 32 + lane) + (i % 4) < length;
    kmin = min(kmin, v ? key[i] : 0xffffffffu);
    kmax = max(kmax, key[i]);
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  // T starts as the common high bits with zeros below: every valid key is
  // >= T, so at least K are (length > K).  Each bit below is kept when at
  // least K keys are >= the candidate; T ends as the K-th largest key.
  const int common = kmin == kmax ? 32 : __clz(kmin ^ kmax);
  uint32_t T = common == 0 ? 0u : (kmax >> (32 - common)) << (32 - common);
  for (int b = 31 - common; b >= 0; --b) {
    const uint32_t cand = T | (1u << b);
    int c4[4] = {0, 0, 0, 0};  // independent sums: a short dependency chain
#pragma unroll
    for (int i = 0; i < kV; ++i) c4[i & 3] += key[i] >= cand ? 1 : 0;
    const int c = __reduce_add_sync(0xffffffffu, (c4[0] + c4[1]) + (c4[2] + c4[3]));
    if (c >= topk) {
      T = cand;
      if (c == topk) break;  // exactly K keys >= T: they are the selection
    }
  }

  // ---- ordered write-out: keys > T are taken, keys == T in column order up
  // to the quota.
  int above = 0, ties = 0;
#pragma unroll
  for (int i = 0; i < kV; ++i) {
    above += key[i] > T ? 1 : 0;
    ties += key[i] == T ? 1 : 0;
  }
  above = __reduce_add_sync(0xffffffffu, above);
  ties = __reduce_add_sync(0xffffffffu, ties) - (T == 0u ? kWarpRowKeys - length : 0);
  const int quota = min(topk - above, ties);
  const unsigned lt = (1u << lane) - 1u;  // lanes below this one
  int run = 0;
  if (quota == ties) {
    // every valid key >= T is taken (invalid slots, key 0, only when T > 0):
    // a key's rank is the number of taken keys before it in column order
    // (chunk, lane, j), from one ballot per (chunk, j)
    const bool t0 = T != 0u;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      bool tk[4];
      unsigned mk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tk[j] = key[4 * c + j] > T || (key[4 * c + j] == T && (t0 || 4 * (c * 32 + lane) + j < length));
        mk[j] = __ballot_sync(0xffffffffu, tk[j]);
      }
      int r = run;
#pragma unroll
      for (int j = 0; j < 4; ++j) r += __popc(mk[j] & lt);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (tk[j]) sel[r] = 4 * (c * 32 + lane) + j;
        r += tk[j] ? 1 : 0;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) run += __popc(mk[j]);
    }
  } else {
    // ties straddle the threshold: the first `quota` of them in column order
    int run_tie = 0;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      unsigned ms[4], mt[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ms[j] = __ballot_sync(0xffffffffu, key[4 * c + j] > T);
        mt[j] = __ballot_sync(0xffffffffu, key[4 * c + j] == T);
      }
      int sb = run, tb = run_tie;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sb += __popc(ms[j] & lt);
        tb += __popc(mt[j] & lt);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int id = 4 * (c * 32 + lane) + j;
        if (key[4 * c + j] > T) {
          sel[sb + min(tb, quota)] = id;
          ++sb;
        } else if (key[4 * c + j] == T) {
          if (tb < quota) sel[sb + tb] = id;
          ++tb;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        run += __popc(ms[j]);
        run_tie += __popc(mt[j]);
      }
    }
    run += quota;
  }
  __syncwarp();
  const int chosen = run;  // = topk
  for (int i = lane; i < chosen; i += 32) {
    if (p.expand && i >= m.complete) break;
    write_rank(p, m, out_row, i, sel[i]);
  }
  if (p.expand) finish_row<32>(p, m, out_row, row, lane);
}

template <int SELCAP>
cudaError_t launch_warp_rows(const TopkParams& p, cudaStream_t stream) {
  const int smem = kRowWarps * SELCAP * static_cast<int>(sizeof(int));
  cudaError_t e = set_attr_once(reinterpret_cast<const void*>(topk_warp_kernel<SELCAP>),
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const unsigned blocks = static_cast<unsigned>((p.rows + kRowWarps - 1) / kRowWarps);
  return count_launches(launch_kernel(topk_warp_kernel<SELCAP>, dim3(blocks),
                                      dim3(kRowWarps * 32), static_cast<size_t>(smem), stream,
                                      1, p));
}

int pow2_ceil(int x) {
  int c = 1;
  while (c < x) c <<= 1;
  return c;
}

template <int T, int V>
cudaError_t launch_v(TopkParams p, int C, cudaStream_t stream) {
  const int smem = std::max(p.topk, 1) * static_cast<int>(sizeof(int));
  if (smem > kMaxSelBytes) return cudaErrorInvalidValue;
  cudaError_t e0 = set_attr_once(reinterpret_cast<const void*>(topk_kernel<T, V>),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSelBytes);
  if (e0 != cudaSuccess) return e0;
  if (C > 8) {
    cudaError_t e = set_attr_once(reinterpret_cast<const void*>(topk_kernel<T, V>),
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  return count_launches(launch_kernel(
      topk_kernel<T, V>, dim3(static_cast<unsigned>(C) * static_cast<unsigned>(p.rows)),
      dim3(T), static_cast<size_t>(std::max(p.topk, 1)) * sizeof(int), stream,
      static_cast<unsigned>(C), p));
}

}  // namespace

int topk_max_width() { return kMaxCluster * kThreads * 32; }

int topk_max_blocks() { return kMaxSelBytes / static_cast<int>(sizeof(int)); }

cudaError_t launch_topk(const TopkParams& p0, cudaStream_t stream, int* plan_cluster) {
  TopkParams p = p0;
  if (p.rows <= 0) return cudaSuccess;
  // Rows of one CTA at 8 keys per thread: the narrowest CTA that covers them.
  const int w = std::max(p.width, 1);
  // One warp per row has a longer per-row latency than a 256-thread CTA but
  // runs four times as many rows per SM: it pays off from about three waves
  // of the CTA form (4 CTAs per SM) on.
  if (w <= kWarpRowKeys && p.topk <= 1024 && p.rows >= 12 * num_sms()) {
    p.slice_cap = kWarpRowKeys;
    if (plan_cluster) *plan_cluster = 1;
    return p.topk <= 256 ? launch_warp_rows<256>(p, stream) : launch_warp_rows<1024>(p, stream);
  }
  if (w <= 256 * 8) {
    p.slice_cap = 256 * 8;
    if (plan_cluster) *plan_cluster = 1;
    return launch_v<256, 8>(p, 1, stream);
  }
  if (w <= 512 * 8) {
    p.slice_cap = 512 * 8;
    if (plan_cluster) *plan_cluster = 1;
    return launch_v<512, 8>(p, 1, stream);
  }
  // Smallest (keys per thread, cluster width) whose slices cover the row.
  int V = 8;
  int C = pow2_ceil((w + kThreads * V - 1) / (kThreads * V));
  if (C > kMaxCluster) {
    V = 32;
    C = pow2_ceil((w + kThreads * V - 1) / (kThreads * V));
  }
  if (C > kMaxCluster) return cudaErrorInvalidValue;
  p.slice_cap = kThreads * V;
  if (plan_cluster) *plan_cluster = C;
  return V == 8 ? launch_v<kThreads, 8>(p, C, stream) : launch_v<kThreads, 32>(p, C, stream);
}

}  // namespace qsa
