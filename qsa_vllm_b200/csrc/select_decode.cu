// Fused decode selection on sm_100a: indexer scores -> exact top-k ->
// expansion to physical slots in ONE launch, the scores kept in shared memory.
//
// Replaces, for decode rows, the two launches per workspace chunk of the
// reference's qsa_select_paged_decode (ops/indexer.py:227-279): the scoring
// kernel (ops/indexer.py:24-114) writing an fp32 logits chunk, then
// topk_expand (ops/csrc/topk.cu:182-350 selection, :107-180 expansion)
// reading it back.  The results are those of qsa_indexer_scores followed by
// qsa_topk_expand on the same inputs, bit for bit: the score arithmetic is
// the scoring kernel's (rounded step by step, one summation order) and the
// selection is exact.
//
// Decomposition.  One thread-block cluster of C CTAs per decode request (its
// decode_query_len rows share one page-table row and one MMA B operand).  CTA
// c of the cluster owns the request's key columns [c*kpc, (c+1)*kpc).
//  * Phase 1, scores: the tcgen05 pipeline of indexer_tc.cu for one segment.
//    Warp 0 loads the query rows and the CTA's key stages with TMA (3-D
//    tensor copies per page, 128-byte swizzled) into a ring of stages; warp 1
//    issues tcgen05.mma (M = 128 keys, N = query columns) into a ring of TMEM
//    accumulators; 8 epilogue warps read them back with tcgen05.ld, apply
//    ReLU, head weight, head sum and scale, and store each row's scores into
//    this CTA's shared-memory slice.
//    The epilogue also counts each row's scores by their top 11 bits (a
//    2048-bin histogram of the uint32 key order) while the keys stream in.
//  * Phase 2, selection (K = the row's block budget).  After one cluster
//    barrier every CTA sums the cluster's histograms (distributed shared
//    memory loads, all in flight at once) and finds the same threshold bin:
//    the keys above it are selected, and R more come from the bin itself.
//    Each CTA stores into CTA 0's shared memory its selected columns and its
//    threshold-bin candidates (key and column, in column order; a CTA with
//    more candidates than slots first keeps its R best).  After a second
//    cluster barrier the other CTAs leave; CTA 0 takes the R best candidates
//    (uint32 key order, ties to the lower column, as the reference), merges
//    them with the selected columns in ascending column order, and expands
//    them to physical slots through the block table, plus the causal tail
//    and the count.
// No global scratch and no flags between CTAs or kernels: only CTA barriers,
// mbarriers (bounded waits) and cluster barriers that every CTA takes the
// same number of times.  Remote loads of a CTA's shared memory happen only
// between two cluster barriers it takes part in, so no CTA leaves while
// another still reads it.  A bounded wait that gives up in phase 1 sets the
// device error word and that request's selection is not written.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"
#include "topk_rows.cuh"

namespace qsa {
namespace {

constexpr int kSelThreads = 320;  // producer, MMA issuer, 8 epilogue warps; all 10 select
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelMaxStages = 8;
constexpr int kSelAcc = 4;         // TMEM accumulator ring (even: one epilogue group each)
constexpr int kSelBins = 2048;     // radix digits of up to 11 bits
constexpr int kSelMaxRows = 4;     // decode rows per request
constexpr int kSelDigitShift = 21; // coarse histogram digit: key bits 31..21
constexpr int kSelFineShift = 16;  // fine histogram digit: key bits 26..16
constexpr int kSelTableCap = 2048; // block-table entries CTA 0 keeps in shared memory
constexpr int kSelMaxCluster = 16;
constexpr int kSelMaxTopk = 8192;  // selected blocks per row
constexpr int kSelMaxScoreBytes = 64 * 1024;  // one CTA's score slices

template <int D, int NQ>
struct SelCfg {
  static constexpr int kSub = D / 64;                  // 128-byte sub-rows per key / query row
  static constexpr int MT = D == 64 ? 2 : 1;           // 128-key MMA tiles per stage
  static constexpr int kStageKeys = MT * kTileKeys;    // 256 keys (D=64) / 128 keys (D=128)
  static constexpr int kSubBytes = kTileKeys * 128;    // one MMA tile, one sub-row: 16 KB
  static constexpr int kStageBytes = MT * kSub * kSubBytes;  // 32 KB
  static constexpr int kQBytes = kSub * NQ * 128;
  static constexpr int kAccCols = MT * NQ;             // TMEM columns of one stage's scores
  static constexpr int kCols = kSelAcc * kAccCols < 32 ? 32 : kSelAcc * kAccCols;
  static_assert(kAccCols <= 64, "a stage's scores are read in one round of TMEM loads");
};

// Per-CTA control block.
struct SelCtl {
  uint64_t full[kSelMaxStages], empty[kSelMaxStages], tfull[kSelAcc], tempty[kSelAcc];
  uint64_t qfull;     // query rows landed; nstages published (MMA issuer)
  uint64_t metafull;  // weights, limits and visible counts published (epilogue)
  uint32_t tmem_base;
  int abort_flag;
  int nstages;            // key stages this CTA scores
  int vis[kSelMaxRows];   // per row: columns with a score (visible count, clipped)
  float w[128];           // per query column: head weight (0 for padding columns)
  int limit[128];         // per query column: its row's scored columns (0: padding)
  // CTA 0 of a cluster: per row and CTA, (selected columns, candidates)
  // stored there by every CTA before the second cluster barrier
  int cnt[kSelMaxRows][kSelMaxCluster][2];
  int any_abort;       // CTAs of the cluster whose scoring gave up (added by each)
  int b1[kSelMaxRows];    // per row: threshold bin of the top-11-bit histogram
  int need[kSelMaxRows];  // per row: keys still to take from the threshold bin
  int sbefore[kSelMaxCluster + 1];  // CTA 0: selected columns of the regions before r
  RowMeta meta[kSelMaxRows];        // CTA 0: expansion metadata of each row
  int tcache_n;                     // CTA 0: block-table entries copied to shared memory
  int tcache_req;                   // CTA 0: their request (-1: none)
  int dshift[kSelMaxRows];          // per row: digit shift of the threshold (16 or 21)
  // selection scratch
  uint32_t wmin[kSelWarps], wmax[kSelWarps];
  int wsum[2][kSelWarps];  // per pass parity: warp totals of the bin scan
  int found[2][3];         // per pass parity: threshold bin, remaining, its count
  int warp_tmp[32];
};

struct SelGeom {
  int C;        // CTAs per cluster (one cluster per decode request)
  int kpc;      // key columns per CTA (a multiple of the stage)
  int stages;   // depth of the stage ring
  int cap;      // columns that can hold a score: min(score width, table capacity)
  int box_rows; // key rows per TMA box (divides the page and 128)
  int hshift;   // log2(heads)
  int kp;       // candidate slots per (CTA, row): the block budget rounded up to 4
};

// Dynamic shared memory, from a 1024-byte aligned base: [ring: stages x
// stage][query rows][scores: rows x kpc fp32][histograms: rows x 2 x
// kSelBins ints][landing: rows x C x 3 x kp ints][block-table cache:
// kSelTableCap ints][control block].  The landing area and the table cache
// are used in CTA 0 only; a landing region (row, CTA) holds selected
// columns [kp], then candidate keys [kp] and candidate columns [kp].  The
// selection's scratch reuses the ring once scoring is done.
template <int D, int NQ>
__host__ __device__ constexpr size_t sel_scores_offset(int stages) {
  return static_cast<size_t>(stages) * SelCfg<D, NQ>::kStageBytes + SelCfg<D, NQ>::kQBytes;
}
template <int D, int NQ>
__host__ __device__ constexpr size_t sel_hist_offset(int stages, int rows, int kpc) {
  return sel_scores_offset<D, NQ>(stages) + static_cast<size_t>(rows) * kpc * sizeof(float);
}
template <int D, int NQ>
__host__ __device__ constexpr size_t sel_landing_offset(int stages, int rows, int kpc) {
  return sel_hist_offset<D, NQ>(stages, rows, kpc) +
         static_cast<size_t>(rows) * 2 * kSelBins * sizeof(int);
}
template <int D, int NQ>
__host__ __device__ constexpr size_t sel_ctl_offset(int stages, int rows, int kpc, int C, int kp) {
  return sel_landing_offset<D, NQ>(stages, rows, kpc) +
         (static_cast<size_t>(rows) * C * 3 * kp + kSelTableCap) * sizeof(int);
}

// ReLU(score) x head weight for the N columns of one key, then the sum of
// each row's H adjacent columns by a log-depth tree: r[x] with x % H == 0
// holds row x / H's sum.  Rounded step by step, in the scoring kernel's order.
template <int N>
__device__ __forceinline__ void head_sums(const uint32_t* v, const float* wr, int H, float* r) {
#pragma unroll
  for (int x = 0; x < N; ++x) r[x] = __fmul_rn(fmaxf(__uint_as_float(v[x]), 0.f), wr[x]);
#pragma unroll
  for (int step = 1; step < N; step <<= 1) {
    if (step < H) {
#pragma unroll
      for (int x = 0; x + step < N; x += 2 * step) r[x] = __fadd_rn(r[x], r[x + step]);
    }
  }
}

__device__ __forceinline__ float ld_once_f32(const float* ptr) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(ptr));
  return v;
}

// ------------------------------------------------ cluster communication
// Results travel to CTA 0 as remote stores / reductions into its shared
// memory (fire and forget), which the next cluster barrier (release /
// acquire) makes visible; histograms are read remotely, all loads of a
// thread in flight together, between two barriers.
__device__ __forceinline__ uint32_t peer_addr(const void* p, int rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void peer_store(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t peer_load(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void peer_add(uint32_t a, uint32_t v) {
  asm volatile("red.relaxed.cluster.shared::cluster.add.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------- block-wide select
// Keys of a selection, as an index range [0, n) with a validity test.
// This CTA's scores of a row in the threshold bin: key >> dshift == bin.
struct BinSrc {
  const float* sc;
  int col0;
  int dshift;
  uint32_t bin;
  __device__ __forceinline__ uint32_t key(int i) const { return __float_as_uint(sc[i]); }
  __device__ __forceinline__ bool valid(int i) const { return (key(i) >> dshift) == bin; }
  __device__ __forceinline__ int col(int i) const { return col0 + i; }
};
// CTA 0's candidate slots of a row: slot s of region r = s / kp holds a key
// at region + kp + s % kp and its column at region + 2 kp + s % kp, valid
// below the region's candidate count counts[2 r + 1].
struct CandSrc {
  const int* land;  // the row's region 0; region r at land + 3 r kp
  const int* counts;
  int kp;
  __device__ __forceinline__ bool valid(int s) const { return s % kp < counts[2 * (s / kp) + 1]; }
  __device__ __forceinline__ uint32_t key(int s) const {
    return static_cast<uint32_t>(land[(s / kp) * 3 * kp + kp + s % kp]);
  }
  __device__ __forceinline__ int col(int s) const {
    return land[(s / kp) * 3 * kp + 2 * kp + s % kp];
  }
};

// Number of entries of the ascending array a[0, n) below v.
__device__ __forceinline__ int lower_bound(const int* a, int n, int v) {
  int lo = 0;
  while (n > 0) {
    const int half = n >> 1;
    if (a[lo + half] < v) {
      lo += half + 1;
      n -= half + 1;
    } else {
      n = half;
    }
  }
  return lo;
}

// Threshold of the `want` largest valid keys of [0, n) (uint32 order, ties
// to the lower index; fewer than all valid keys are wanted): selected are
// the keys with (key >> shift) > prefix and, in index order, the first
// `quota` keys with (key >> shift) == prefix.  A most-significant-digit
// radix select below the high bits that every key shares, with digits of up
// to 11 bits; hist (2 x kSelBins ints, double-buffered by the pass parity
// gp & 1) is zero on entry and on return.
template <class Src>
__device__ __forceinline__ void block_threshold(const Src& src, int n, int want, int* hist,
                                                SelCtl& ctl, int& gp, uint32_t& prefix,
                                                int& shift, int& quota) {
  constexpr int T = kSelThreads, W = kSelWarps;
  constexpr int kPer = (kSelBins + T - 1) / T;  // most bins one thread ranks
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t kmin = 0xffffffffu, kmax = 0u;
  for (int i = tid; i < n; i += T) {
    if (src.valid(i)) {
      const uint32_t k = src.key(i);
      kmin = min(kmin, k);
      kmax = max(kmax, k);
    }
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  if (lane == 0) {
    ctl.wmin[warp] = kmin;
    ctl.wmax[warp] = kmax;
  }
  __syncthreads();
#pragma unroll
  for (int w = 0; w < W; ++w) {
    kmin = min(kmin, ctl.wmin[w]);
    kmax = max(kmax, ctl.wmax[w]);
  }
  const int common = kmin == kmax ? 32 : __clz(kmin ^ kmax);  // high bits every key shares
  shift = 32 - common;
  prefix = common == 0 ? 0u : kmax >> shift;  // resolved high bits of the threshold
  int remaining = want;  // keys matching `prefix` still to be taken
  for (; shift > 0; ++gp) {
    const int par = gp & 1;
    int* hb = hist + par * kSelBins;
    const int dbits = shift < 11 ? shift : 11;
    const int dshift = shift - dbits;
    const uint32_t dmask = (1u << dbits) - 1u;
    for (int i = tid; i < n; i += T) {
      if (src.valid(i)) {
        const uint32_t k = src.key(i);
        if (shift >= 32 || (k >> shift) == prefix) atomicAdd(hb + ((k >> dshift) & dmask), 1);
      }
    }
    // the other buffer, last read a pass ago, is cleared for the next pass
    for (int i = tid; i < kSelBins; i += T) hist[(par ^ 1) * kSelBins + i] = 0;
    __syncthreads();
    // thread t ranks `per` bins downwards from bin nb-1-per*t (descending
    // order): a warp scan, then the totals of the warps before it
    const int nb = 1 << dbits;
    const int per = (nb + T - 1) / T;
    const int top = nb - 1 - per * tid;
    int h[kPer];
    int mine = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      h[i] = (i < per && top - i >= 0) ? hb[top - i] : 0;
      mine += h[i];
    }
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) ctl.wsum[par][warp] = incl;
    __syncthreads();
    int above = incl - mine;
    for (int w = 0; w < warp; ++w) above += ctl.wsum[par][w];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (i < per && top - i >= 0 && above < remaining && remaining <= above + h[i]) {
        ctl.found[par][0] = top - i;
        ctl.found[par][1] = remaining - above;
        ctl.found[par][2] = h[i];
      }
      above += h[i];
    }
    __syncthreads();
    prefix = (shift >= 32 ? 0u : (prefix << dbits)) | static_cast<uint32_t>(ctl.found[par][0]);
    remaining = ctl.found[par][1];
    shift = dshift;
    if (ctl.found[par][2] == remaining) {  // the threshold bin is taken whole
      ++gp;
      break;
    }
  }
  // the last pass cleared the buffer of parity gp & 1: both are zero again
  // once this one is (its counts are not needed any more)
  for (int i = tid; i < kSelBins; i += T) hist[((gp & 1) ^ 1) * kSelBins + i] = 0;
  quota = remaining;
  __syncthreads();
}

// Hands the selected entries of [0, n) to sink(rank, index) in index order
// (rank 0, 1, ...; ties to the lower index) and returns how many there are.
// Each thread takes a contiguous run of indexes, so one block scan of its
// packed (strict << 16 | tie) counts ranks them (n < 65536).
template <class Src, class Sink>
__device__ __forceinline__ int block_compact(const Src& src, int n, uint32_t prefix, int shift,
                                             int quota, SelCtl& ctl, Sink sink) {
  constexpr int T = kSelThreads, W = kSelWarps;
  const int tid = threadIdx.x;
  const int run = (n + T - 1) / T;
  const int lo = min(tid * run, n), hi = min(lo + run, n);
  int fs = 0, ft = 0;
  for (int i = lo; i < hi; ++i) {
    if (src.valid(i)) {
      const uint32_t d = src.key(i) >> shift;
      fs += d > prefix;
      ft += d == prefix;
    }
  }
  int total = 0;
  const int ex = block_exclusive_sum<W>((fs << 16) | ft, ctl.warp_tmp, total);
  int sb = ex >> 16, tb = ex & 0xffff;
  for (int i = lo; i < hi; ++i) {
    if (!src.valid(i)) continue;
    const uint32_t d = src.key(i) >> shift;
    if (d > prefix) {
      sink(sb + min(tb, quota), i);
      ++sb;
    } else if (d == prefix) {
      if (tb < quota) sink(sb + tb, i);
      ++tb;
    }
  }
  return (total >> 16) + min(quota, total & 0xffff);
}

// Writes row `row`'s selection: `count` block ids sel[0..count) (ascending),
// expanded through the block table, then the causal tail, -1 fill and count.
__device__ __forceinline__ void expand_row(const TopkParams& tk, const RowMeta& m, int row,
                                           const int* sel, int count) {
  int32_t* out_row = tk.output + static_cast<int64_t>(row) * tk.out_row_stride;
  const int n = min(count, m.complete);
  // two ranks per thread and round: their block-table loads are in flight together
  for (int i = threadIdx.x; i < n; i += 2 * kSelThreads) {
    const int i2 = i + kSelThreads;
    const int b0 = sel[i], b1 = i2 < n ? sel[i2] : -1;
    const int ph0 = tk.aligned_blocks ? block_page(tk, m, b0 * tk.ratio) : 0;
    const int ph1 = (tk.aligned_blocks && i2 < n) ? block_page(tk, m, b1 * tk.ratio) : 0;
    store_block(tk, m, out_row, i, b0, ph0);
    if (i2 < n) store_block(tk, m, out_row, i2, b1, ph1);
  }
  finish_row<kSelThreads>(tk, m, out_row, row);
}

// Writes a row whose length is at most the budget: every column is selected
// (reference topk.cu:187-191), no score is read.
__device__ __forceinline__ void expand_whole_row(const TopkParams& tk, const RowMeta& m, int row,
                                                 int length) {
  int32_t* out_row = tk.output + static_cast<int64_t>(row) * tk.out_row_stride;
  const int nsel = max(m.complete, 0);
  for (int i = threadIdx.x; i < nsel; i += kSelThreads)
    write_rank(tk, m, out_row, i, i < length ? i : -1);
  finish_row<kSelThreads>(tk, m, out_row, row);
}

template <int D, int NQ>
__global__ void __launch_bounds__(kSelThreads, 1) select_decode_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap qmap,
    const SelectParams p, const SelGeom g) {
  using Cf = SelCfg<D, NQ>;
  constexpr int SK = Cf::kStageKeys, A = kSelAcc, MT = Cf::MT;
  constexpr uint32_t kIdesc = instr_desc<kTileKeys, NQ>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the 128-byte swizzle pattern is taken from address bits: 1024-byte base
  uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const IndexerParams& ix = p.ix;
  const TopkParams& tk = p.tk;
  const int dql = ix.decode_query_len;
  const int S = g.stages;
  const int C = g.C;
  uint8_t* qs = ring + static_cast<size_t>(S) * Cf::kStageBytes;
  float* scores = reinterpret_cast<float*>(ring + sel_scores_offset<D, NQ>(S));
  int* h1 = reinterpret_cast<int*>(ring + sel_hist_offset<D, NQ>(S, dql, g.kpc));
  int* land = reinterpret_cast<int*>(ring + sel_landing_offset<D, NQ>(S, dql, g.kpc));
  int* tcache = land + static_cast<size_t>(dql) * C * 3 * g.kp;
  SelCtl& ctl = *reinterpret_cast<SelCtl*>(ring + sel_ctl_offset<D, NQ>(S, dql, g.kpc, C, g.kp));

  const int crank = static_cast<int>(blockIdx.x) % C;  // rank in the cluster (1-D clusters)
  const int seg = static_cast<int>(blockIdx.x) / C;    // decode request
  const int r0 = seg * dql;
  const int k_begin = crank * g.kpc;                   // a multiple of SK
  const int k_end = min(k_begin + g.kpc, g.cap);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = ix.heads, hshift = g.hshift;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctl.full[s], 1);
      mbar_init(&ctl.empty[s], 1);
    }
    for (int a = 0; a < A; ++a) {
      mbar_init(&ctl.tfull[a], 1);
      mbar_init(&ctl.tempty[a], 4);  // the four warps of the group that owns the buffer
    }
    mbar_init(&ctl.qfull, 1);
    mbar_init(&ctl.metafull, 1);
    ctl.abort_flag = 0;
    ctl.nstages = 0;
    ctl.any_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&qmap);
  }
  for (int i = tid; i < dql * 2 * kSelBins; i += kSelThreads) h1[i] = 0;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&ctl.tmem_base)),
                 "r"(Cf::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  // Every CTA of the cluster is resident before any stores into another's
  // shared memory: this CTA arrives on the cluster barrier now and waits on
  // it after scoring.
  if (C > 1) cluster_arrive();
  const uint32_t tmem = ctl.tmem_base;

  // Step metadata that no kernel of this library writes after triggering its
  // dependents (the page table, and the visible counts or the positions,
  // sequence lengths and request ids they derive from) is read before waiting
  // on the preceding kernel: the latency overlaps that wait.  Page ids come
  // from a 32-page window of the table row in registers (cur), with the next
  // window (nxt) already loaded; a stage spans at most 32 pages.
  const int ta = k_begin / SK;
  const int32_t* trow = ix.table + static_cast<int64_t>(seg) * ix.table_row_stride;
  auto page_of = [&](int lp) { return lp < ix.table_width ? ld_once(trow + lp) : -1; };
  int wbase = 0, cur = -1, nxt = -1, vis_row = 0;
  if (warp == 0) {
    wbase = static_cast<int>(ix.page_div.div(ta * SK));
    cur = page_of(wbase + lane);
    nxt = page_of(wbase + 32 + lane);
    if (lane < dql) vis_row = min(max(row_visible(ix, r0 + lane), 0), g.cap);
  }
  pdl_wait();
  pdl_trigger();

  // ====================================================== phase 1: scores
  if (warp == 0) {
    // ---------------------------------------------------------- producer
    int maxvis = vis_row;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) maxvis = max(maxvis, __shfl_xor_sync(0xffffffffu, maxvis, o));
    const int tb = max(ta, (min(k_end, maxvis) + SK - 1) / SK);
    const int nst = tb - ta;
    // head weights (loads issued now, published once the first stages are
    // on their way) and the query columns' store limits
    float w_lane[(NQ + 31) / 32];
    int lim_lane[(NQ + 31) / 32];
#pragma unroll
    for (int i = 0; i < (NQ + 31) / 32; ++i) {
      const int n = lane + 32 * i;
      const int ri = n >> hshift, h = n & (H - 1);
      const int rv = __shfl_sync(0xffffffffu, vis_row, ri & 31);
      const bool valid = n < NQ && ri < dql;
      w_lane[i] = !valid ? 0.f
                  : ix.weights != nullptr
                      ? ld_once_f32(ix.weights + static_cast<int64_t>(r0 + ri) * ix.w_row_stride +
                                    static_cast<int64_t>(h) * ix.w_head_stride)
                      : 1.f;
      lim_lane[i] = valid ? rv : 0;
    }
    if (lane == 0) {
      ctl.nstages = nst;
      if (nst > 0) {
        mbar_expect_tx(&ctl.qfull, static_cast<uint32_t>(Cf::kSub * H * dql * 128));
#pragma unroll
        for (int sub = 0; sub < Cf::kSub; ++sub)
          tma_load_3d(qs + sub * NQ * 128, &qmap, sub * 64, 0, r0, &ctl.qfull);
      }
      mbar_arrive(&ctl.qfull);  // publishes nstages to the MMA issuer
    }
    bool published = false;
    auto publish = [&]() {
#pragma unroll
      for (int i = 0; i < (NQ + 31) / 32; ++i) {
        const int n = lane + 32 * i;
        if (n < NQ) {
          ctl.w[n] = w_lane[i];
          ctl.limit[n] = lim_lane[i];
        }
      }
      if (lane < dql) ctl.vis[lane] = vis_row;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl.metafull);
      published = true;
    };
    const int first_batch = min(S, nst);
    const int boxes = SK / g.box_rows;  // <= 32: one lane per box
    const int box_key = lane * g.box_rows;
    const int box_m = box_key / kTileKeys, box_row = box_key % kTileKeys;
    bool ok = true;
    int it = 0;
    for (int t = ta; t < tb; ++t, ++it) {
      const int s = it % S;
      if (aborted(&ctl.abort_flag) || (it >= S && !warp_wait(&ctl.empty[s], ((it / S) - 1) & 1))) {
        ok = false;
        break;
      }
      const int key0 = t * SK;
      if (static_cast<int>(ix.page_div.div(key0)) >= wbase + 32) {
        wbase += 32;
        cur = nxt;
        nxt = page_of(wbase + 32 + lane);
      }
      int lp, off;
      ix.page_div.divmod(key0 + box_key, lp, off);
      const int d = lp - wbase;  // < 64
      const int pc = __shfl_sync(0xffffffffu, cur, d & 31);
      const int pn = __shfl_sync(0xffffffffu, nxt, d & 31);
      int page = d < 32 ? pc : pn;
      if (page < 0 || page >= ix.num_blocks) page = ix.num_blocks;  // out of range: zero-filled
      if (lane == 0) mbar_expect_tx(&ctl.full[s], Cf::kStageBytes);
      __syncwarp();
      if (lane < boxes) {
        uint8_t* dst = ring + static_cast<size_t>(s) * Cf::kStageBytes +
                       box_m * (Cf::kSub * Cf::kSubBytes) + box_row * 128;
#pragma unroll
        for (int sub = 0; sub < Cf::kSub; ++sub)
          tma_load_3d(dst + sub * Cf::kSubBytes, &kmap, sub * 64, off, page, &ctl.full[s]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl.full[s]);
      if (!published && it + 1 == first_batch) publish();
    }
    if (!published) publish();
    if (!ok && lane == 0) {
      record_error(ix.err, kDeviceErrWaitTimeout);
      ctl.abort_flag = 1;
    }
    // drain: every copy this CTA issued has landed before its memory is reused
    for (int x = max(0, it - S); x < it; ++x)
      if (!warp_wait(&ctl.full[x % S], (x / S) & 1) && lane == 0)
        record_error(ix.err, kDeviceErrWaitTimeout);
    if (!warp_wait(&ctl.qfull, 0) && lane == 0) record_error(ix.err, kDeviceErrWaitTimeout);
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    bool ok = !aborted(&ctl.abort_flag) && warp_wait(&ctl.qfull, 0);
    const int nst = ok ? ctl.nstages : 0;
    const uint32_t qbase = smem_u32(qs);
    int it = 0;
    for (; ok && it < nst; ++it) {
      const int s = it % S, a = it % A;
      if (aborted(&ctl.abort_flag) || !warp_wait(&ctl.full[s], (it / S) & 1) ||
          (it >= A && !warp_wait(&ctl.tempty[a], ((it / A) - 1) & 1))) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (lane == 0) {
        const uint32_t kbase = smem_u32(ring + static_cast<size_t>(s) * Cf::kStageBytes);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int sub = kk >> 2, part = kk & 3;
            const uint64_t ad =
                sw128_desc(kbase + (mt * Cf::kSub + sub) * Cf::kSubBytes + part * 32);
            const uint64_t bd = sw128_desc(qbase + sub * NQ * 128 + part * 32);
            umma_bf16(tmem + a * Cf::kAccCols + mt * NQ, ad, bd, kIdesc, kk > 0);
          }
        }
        umma_commit(&ctl.empty[s]);  // stage reusable once these MMAs have read it
        umma_commit(&ctl.tfull[a]);  // accumulator a ready for the epilogue
      }
      __syncwarp();
    }
    if (!ok && lane == 0) {
      record_error(ix.err, kDeviceErrWaitTimeout);
      ctl.abort_flag = 1;
    }
    // drain: the last MMAs have completed before TMEM is released
    if (it > 0 && !warp_wait(&ctl.tfull[(it - 1) % A], ((it - 1) / A) & 1) && lane == 0)
      record_error(ix.err, kDeviceErrWaitTimeout);
  } else {
    // ---------------------------------------------------------- epilogue
    const int grp = (warp - 2) >> 2;  // stages grp, grp + 2, ...
    const int quad = warp & 3;        // TMEM lanes 32*quad .. +31: keys of this warp
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    if (crank == 0) {
      // CTA 0 expands the selection: while the first keys are on their way,
      // it fetches each row's expansion metadata and the request's block-table
      // row (step metadata) into shared memory
      const int etid = tid - 64;  // 0 .. 255
      if (etid < dql) {
        RowMeta m = row_meta(tk, r0 + etid);
        ctl.meta[etid] = m;
      }
      if (tk.physical) {
        const RowMeta m0 = row_meta(tk, r0);
        const int pages = static_cast<int>(tk.page_div.div(static_cast<uint32_t>(max(m0.seq, 0)) +
                                                          tk.page_size - 1));
        const int n_tbl = min(min(pages, tk.table_width), kSelTableCap);
        for (int i = etid; i < n_tbl; i += 256) tcache[i] = __ldg(m0.trow + i);
        if (etid == 0) {
          ctl.tcache_n = n_tbl;
          ctl.tcache_req = tk.token_to_req[r0];
        }
      } else if (etid == 0) {
        ctl.tcache_n = 0;
        ctl.tcache_req = -1;
      }
    }
    bool ok = !aborted(&ctl.abort_flag) && warp_wait(&ctl.metafull, 0);
    const int nst = ok ? ctl.nstages : 0;
    float wr[NQ];
    int lim_col[NQ];
#pragma unroll
    for (int x = 0; x < NQ; ++x) {
      wr[x] = ctl.w[x];
      lim_col[x] = (x & (H - 1)) == 0 ? ctl.limit[x] : 0;
    }
    const float scale = ix.scale;
    for (int t = 0; ok && t < nst; ++t) {
      if ((t & 1) != grp) continue;
      const int a = t % A;
      if (aborted(&ctl.abort_flag) || !warp_wait(&ctl.tfull[a], (t / A) & 1)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t v[Cf::kAccCols];
#pragma unroll
      for (int c = 0; c < Cf::kAccCols; c += 16)
        tmem_ld16(tmem + lane_base + a * Cf::kAccCols + c, v + c);
      tmem_wait_ld();
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        float r[NQ];
        head_sums<NQ>(v + mt * NQ, wr, H, r);
        const int local = t * SK + mt * kTileKeys + quad * 32 + lane;  // column - k_begin
        const int key = k_begin + local;
#pragma unroll
        for (int x = 0; x < NQ; ++x) {
          if ((x & (H - 1)) == 0 && key < lim_col[x]) {
            const int ri = x >> hshift;
            const float val = r[x] * scale;
            scores[ri * g.kpc + local] = val;
            const uint32_t kb = __float_as_uint(val);
            atomicAdd(h1 + ri * 2 * kSelBins + (kb >> kSelDigitShift), 1);
            atomicAdd(h1 + ri * 2 * kSelBins + kSelBins + ((kb >> kSelFineShift) & (kSelBins - 1)),
                      1);
            if (p.scores_out != nullptr)
              p.scores_out[static_cast<int64_t>(r0 + ri) * p.scores_row_stride + key] = val;
          }
        }
      }
      // the scores are in registers: hand the accumulator back
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&ctl.tempty[a]);
    }
    if (!ok && lane == 0) {
      record_error(ix.err, kDeviceErrWaitTimeout);
      ctl.abort_flag = 1;
    }
  }
  // every role loop is warp-uniform, so each warp arrives here converged
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(Cf::kCols)
                 : "memory");
  }
  // the ring, last written by TMA and read by the tensor cores, is reused by
  // ordinary loads and stores below
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  // ==================================================== phase 2: selection
  const int K = tk.topk;
  int* sel = reinterpret_cast<int*>(ring);  // [kp] CTA 0: selected block ids, by rank
  int* tsel = sel + g.kp;                   // [kp] CTA 0: selected candidates' columns
  int* hist = tsel + g.kp;                  // [2][kSelBins] radix scratch, zero between uses
  int* tot = hist + 2 * kSelBins;           // [2][kSelBins] the cluster's two histograms
  for (int i = tid; i < 2 * kSelBins; i += kSelThreads) hist[i] = 0;
  // Barrier A: every CTA's scores and histograms are complete, and every CTA
  // knows how many CTAs of the cluster gave up (each adds itself everywhere).
  if (C > 1) {
    cluster_wait();  // every CTA resident and initialised (arrived before scoring)
    if (ctl.abort_flag != 0 && tid < C) peer_add(peer_addr(&ctl.any_abort, tid), 1u);
    cluster_arrive();
    cluster_wait();
  } else {
    if (tid == 0 && ctl.abort_flag != 0) ctl.any_abort = 1;
    __syncthreads();
  }
  if (ctl.any_abort != 0) return;  // the same decision in every CTA of the cluster
  int gp = 0;  // radix passes so far (scratch parity)
  constexpr int kPer = (kSelBins + kSelThreads - 1) / kSelThreads;  // bins per thread
  constexpr int kRun = 16;  // keys a thread classifies from registers
  for (int j = 0; j < dql; ++j) {
    const int length = ctl.vis[j];
    if (length <= K) continue;  // CTA 0 writes the whole row
    // ---- the cluster's two histograms of the row: consecutive threads read
    // consecutive bins of every CTA (coalesced), four CTAs' loads in flight;
    // plus the lowest and highest non-empty coarse bin
    const int* hj = h1 + j * 2 * kSelBins;
    int lo_bin = kSelBins, hi_bin = -1;
    for (int i = 0; i < kPer; ++i) {
      const int b = tid + i * kSelThreads;
      if (b >= kSelBins) break;
      int sa = 0, sf = 0;
      if (C == 1) {
        sa = hj[b];
        sf = hj[kSelBins + b];
      } else {
        for (int r0c = 0; r0c < C; r0c += 4) {
          uint32_t va[4], vf[4];
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            const bool live = r0c + rr < C;
            const uint32_t base = live ? peer_addr(hj + b, r0c + rr) : 0u;
            va[rr] = live ? peer_load(base) : 0u;
            vf[rr] = live ? peer_load(base + 4u * kSelBins) : 0u;
          }
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            sa += static_cast<int>(va[rr]);
            sf += static_cast<int>(vf[rr]);
          }
        }
      }
      tot[b] = sa;
      tot[kSelBins + b] = sf;
      if (sa != 0) {
        lo_bin = min(lo_bin, b);
        hi_bin = max(hi_bin, b);
      }
    }
    lo_bin = __reduce_min_sync(0xffffffffu, lo_bin);
    hi_bin = __reduce_max_sync(0xffffffffu, hi_bin);
    if (lane == 0) {
      ctl.wmin[warp] = static_cast<uint32_t>(lo_bin);
      ctl.wmax[warp] = static_cast<uint32_t>(hi_bin + 1);
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kSelWarps; ++w) {
      lo_bin = min(lo_bin, static_cast<int>(ctl.wmin[w]));
      hi_bin = max(hi_bin, static_cast<int>(ctl.wmax[w]) - 1);
    }
    // The fine histogram (key bits 26..16) resolves five more bits when
    // every key of the row has the same top five bits (31..27); otherwise
    // the coarse one (bits 31..21) is used.
    const int prefix5 = lo_bin >> 6;
    const bool fine = prefix5 == (hi_bin >> 6);
    const int* cnt = tot + (fine ? kSelBins : 0);
    // ---- threshold bin: where the running count from the top reaches K
    const int top = kSelBins - 1 - kPer * tid;
    int h[kPer];
    int mine = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      h[i] = top - i >= 0 ? cnt[top - i] : 0;
      mine += h[i];
    }
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) ctl.wsum[0][warp] = incl;
    __syncthreads();
    int above = incl - mine;
    for (int w = 0; w < warp; ++w) above += ctl.wsum[0][w];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (top - i >= 0 && above < K && K <= above + h[i]) {
        ctl.b1[j] = fine ? ((prefix5 << 11) | (top - i)) : top - i;
        ctl.need[j] = K - above;
        ctl.dshift[j] = fine ? kSelFineShift : kSelDigitShift;
      }
      above += h[i];
    }
    __syncthreads();
    const uint32_t b1 = static_cast<uint32_t>(ctl.b1[j]);
    const int need = ctl.need[j];  // 1..K
    const int dshift = ctl.dshift[j];
    // ---- this CTA's columns above the bin, and its candidates in the bin,
    // into its region of CTA 0's landing area, in column order
    const int n = min(max(min(k_end, length) - k_begin, 0), g.kpc);
    const float* sc = scores + j * g.kpc;
    int* region = land + (j * C + crank) * 3 * g.kp;  // this CTA's region (used in CTA 0)
    const uint32_t rb = C > 1 ? peer_addr(region, 0) : 0u;
    auto put = [&](int idx, uint32_t v) {
      if (C > 1)
        peer_store(rb + 4u * idx, v);
      else
        region[idx] = static_cast<int>(v);
    };
    const int run = (n + kSelThreads - 1) / kSelThreads;
    const int lo = min(tid * run, n), hi = min(lo + run, n);
    const bool in_regs = run <= kRun;
    uint32_t kk[kRun];
#pragma unroll
    for (int i = 0; i < kRun; ++i) kk[i] = in_regs && lo + i < hi ? __float_as_uint(sc[lo + i]) : 0u;
    int fs = 0, fc = 0;
    if (in_regs) {
#pragma unroll
      for (int i = 0; i < kRun; ++i) {
        if (lo + i < hi) {
          const uint32_t d = kk[i] >> dshift;
          fs += d > b1;
          fc += d == b1;
        }
      }
    } else {
      for (int i = lo; i < hi; ++i) {
        const uint32_t d = __float_as_uint(sc[i]) >> dshift;
        fs += d > b1;
        fc += d == b1;
      }
    }
    int total = 0;
    const int ex = block_exclusive_sum<kSelWarps>((fs << 16) | fc, ctl.warp_tmp, total);
    const int n_strict = total >> 16, n_cand = total & 0xffff;
    const bool keep_all = n_cand <= g.kp;  // all candidates fit their slots
    int sb = ex >> 16, cb = ex & 0xffff;
    auto emit = [&](int i, uint32_t k) {
      const uint32_t d = k >> dshift;
      if (d > b1) {
        put(sb++, static_cast<uint32_t>(k_begin + i));
      } else if (d == b1 && keep_all) {
        put(g.kp + cb, k);
        put(2 * g.kp + cb, static_cast<uint32_t>(k_begin + i));
        ++cb;
      }
    };
    if (in_regs) {
#pragma unroll
      for (int i = 0; i < kRun; ++i)
        if (lo + i < hi) emit(lo + i, kk[i]);
    } else {
      for (int i = lo; i < hi; ++i) emit(i, __float_as_uint(sc[i]));
    }
    int n_kept = n_cand;
    if (!keep_all) {
      // more candidates than slots: only this CTA's `need` best of them can
      // be selected, so those are kept
      const BinSrc src{sc, k_begin, dshift, b1};
      uint32_t prefix;
      int shift, quota;
      block_threshold(src, n, need, hist, ctl, gp, prefix, shift, quota);
      n_kept = block_compact(src, n, prefix, shift, quota, ctl, [&](int rank, int i) {
        put(g.kp + rank, src.key(i));
        put(2 * g.kp + rank, static_cast<uint32_t>(src.col(i)));
      });
    }
    if (tid == 0) {
      int* c = &ctl.cnt[j][crank][0];
      if (C > 1) {
        peer_store(peer_addr(c, 0), static_cast<uint32_t>(n_strict));
        peer_store(peer_addr(c + 1, 0), static_cast<uint32_t>(n_kept));
      } else {
        c[0] = n_strict;
        c[1] = n_kept;
      }
    }
    __syncthreads();  // ctl.wsum / wmin / b1 / need and tot are rewritten by the next row
  }
  // Barrier B: CTA 0 holds every CTA's columns and candidates; no CTA reads
  // another's shared memory after it, so the others leave.
  if (C > 1) {
    cluster_arrive();
    cluster_wait();
  } else {
    __syncthreads();
  }
  if (crank != 0) return;

  // CTA 0: per row, the `need` best candidates, merged with the columns
  // above the threshold bin in ascending column order, then expanded.
  for (int j = 0; j < dql; ++j) {
    RowMeta m = ctl.meta[j];
    if (tk.physical && ctl.tcache_n > 0 && tk.token_to_req[r0 + j] == ctl.tcache_req) {
      m.tcache = tcache;
      m.tcache_n = ctl.tcache_n;
    }
    const int length = ctl.vis[j];
    if (length <= K) {
      expand_whole_row(tk, m, r0 + j, length);
      continue;
    }
    const int need = ctl.need[j];
    const int* counts = &ctl.cnt[j][0][0];
    const int* land_j = land + j * C * 3 * g.kp;
    if (tid == 0) {
      ctl.sbefore[0] = 0;
      int nc = 0;
      for (int r = 0; r < C; ++r) {
        ctl.sbefore[r + 1] = ctl.sbefore[r] + counts[2 * r];
        nc += counts[2 * r + 1];
      }
      ctl.b1[j] = nc;  // the row's candidates (b1 is not needed any more)
    }
    __syncthreads();
    const int n_cand = ctl.b1[j];
    const CandSrc src{land_j, counts, g.kp};
    const int slots = C * g.kp;
    if (n_cand <= need) {
      // every candidate is selected: with shift 0 and prefix 0, keys above 0
      // count as strict and keys equal to 0 as ties, and all ties are taken
      block_compact(src, slots, 0u, 0, n_cand, ctl,
                    [&](int rank, int s) { tsel[rank] = src.col(s); });
    } else {
      uint32_t prefix;
      int shift, quota;
      block_threshold(src, slots, need, hist, ctl, gp, prefix, shift, quota);
      block_compact(src, slots, prefix, shift, quota, ctl,
                    [&](int rank, int s) { tsel[rank] = src.col(s); });
    }
    __syncthreads();
    // merge: regions are in column order, each region's columns ascending;
    // a column's rank = its index in its own list + the entries of the other
    // list below it
    const int* sbefore = ctl.sbefore;
    const int n_strict = sbefore[C];
    for (int f = tid; f < n_strict; f += kSelThreads) {
      int r = 0;
      while (f >= sbefore[r + 1]) ++r;
      const int c = land_j[r * 3 * g.kp + (f - sbefore[r])];
      sel[f + lower_bound(tsel, need, c)] = c;
    }
    for (int k = tid; k < need; k += kSelThreads) {
      const int c = tsel[k];
      const int r = c / g.kpc;
      sel[k + sbefore[r] + lower_bound(land_j + r * 3 * g.kp, counts[2 * r], c)] = c;
    }
    __syncthreads();
    expand_row(tk, m, r0 + j, sel, n_strict + need);
    __syncthreads();  // sel, tsel and sbefore are rewritten by the next row
  }
}

// Clusters of this kernel, width and shared-memory size that can be resident
// at once on the current device (cached per kernel, width, size and device;
// 0 when none fits).
int active_clusters(const void* fn, int C, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t, int>, int> seen;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(fn, C, smem, dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto f = seen.find(key);
    if (f != seen.end()) return f->second;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(C));
  cfg.blockDim = dim3(kSelThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    clusters = 0;
  }
  std::lock_guard<std::mutex> lk(mu);
  seen[key] = clusters;
  return clusters;
}

// Picks the cluster width and launches.  Every request's cluster must be
// resident at once (one wave): the widest power-of-two width, at most 16 and
// at most one CTA per SM overall, whose clusters all fit the device together,
// with each CTA's score slices within kSelMaxScoreBytes, at least two stages
// in its ring, and room for the selection's buffers.
template <int D, int NQ>
cudaError_t plan_and_launch(const SelectParams& p, int segments, int stages_total, int optin,
                            int box_rows, int hshift, const CUtensorMap& kmap,
                            const CUtensorMap& qmap, cudaStream_t stream, const char** why) {
  using Cf = SelCfg<D, NQ>;
  const void* fn = reinterpret_cast<const void*>(select_decode_kernel<D, NQ>);
  // the shared-memory size varies from call to call: the function's limit is
  // raised once to the device maximum, so every size below it can launch
  cudaError_t e = set_attr_once(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
  if (e != cudaSuccess) return e;
  if (set_attr_once(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    cudaGetLastError();  // portable widths (<= 8) only
  const int dql = p.ix.decode_query_len;
  const int kp = (p.tk.topk + 3) & ~3;
  const int sms = num_sms();
  int c_hi = 1;
  while (c_hi * 2 <= kSelMaxCluster && static_cast<int64_t>(segments) * c_hi * 2 <= sms &&
         c_hi * 2 <= stages_total)
    c_hi *= 2;
  for (int C = c_hi; C >= 1; C /= 2) {
    const int kpc = (stages_total + C - 1) / C * Cf::kStageKeys;
    if (static_cast<int64_t>(dql) * kpc * 4 > kSelMaxScoreBytes) break;  // narrower: larger
    // candidate slots of one row: their counts are packed in 16 bits, and
    // strict counts shifted left by 16 must stay positive
    if (static_cast<int64_t>(C) * kp >= 32768) continue;
    if (kpc >= 65536) continue;                            // packed per-CTA counts
    const int64_t fixed =
        1024 + static_cast<int64_t>(sel_ctl_offset<D, NQ>(0, dql, kpc, C, kp)) + sizeof(SelCtl);
    const int stages =
        static_cast<int>(std::min<int64_t>(kSelMaxStages, (optin - fixed) / Cf::kStageBytes));
    // the selection's scratch (two id lists, four histograms) lives in the ring
    if (stages < 2 || static_cast<int64_t>(stages) * Cf::kStageBytes <
                          static_cast<int64_t>(4 * kSelBins + 2 * kp) * 4)
      continue;
    const size_t smem = static_cast<size_t>(fixed) + static_cast<size_t>(stages) * Cf::kStageBytes;
    if (active_clusters(fn, C, smem) < segments) continue;
    SelGeom g{};
    g.C = C;
    g.kpc = kpc;
    g.stages = stages;
    g.cap = std::min(p.score_width, p.ix.table_width * p.ix.page_size);
    g.box_rows = box_rows;
    g.hshift = hshift;
    g.kp = kp;
    return count_launches(launch_kernel(select_decode_kernel<D, NQ>,
                                        dim3(static_cast<unsigned>(segments * C)),
                                        dim3(kSelThreads), smem, stream,
                                        static_cast<unsigned>(C), kmap, qmap, p, g));
  }
  if (why != nullptr) *why = "the requests' thread-block clusters do not fit the GPU at once";
  return cudaErrorNotSupported;
}

}  // namespace

cudaError_t launch_select_decode(const SelectParams& p, cudaStream_t stream, const char** why) {
  const IndexerParams& ix = p.ix;
  auto decline = [why](const char* reason) {
    if (why != nullptr) *why = reason;
    return cudaErrorNotSupported;
  };
  if (ix.num_rows <= 0) return cudaSuccess;
  if (ix.query_start_loc != nullptr || !indexer_tc_eligible(ix))
    return decline("key pages or strides a TMA box cannot address");
  const int H = ix.heads;
  const int dql = ix.decode_query_len;
  if (H <= 0 || (H & (H - 1)) != 0) return decline("head count not a power of two");
  if (dql < 1 || dql > kSelMaxRows) return decline("more than 4 decode rows per request");
  const int n = dql * H;
  if (n > 32) return decline("decode_query_len * heads above 32");
  const int nq = n <= 16 ? 16 : 32;
  if (!p.tk.expand || p.tk.topk < 1 || p.tk.topk > kSelMaxTopk)
    return decline("top-k blocks outside 1..8192");
  const int segments = ix.num_rows / dql;
  if (segments > num_sms()) return decline("more requests than SMs");
  const int sk = ix.dim == 64 ? SelCfg<64, 16>::kStageKeys : SelCfg<128, 16>::kStageKeys;
  const int cap = std::max(0, std::min(p.score_width, ix.table_width * ix.page_size));
  const int stages_total = std::max(1, (cap + sk - 1) / sk);
  int dev = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return decline("device attributes unavailable");
  const int box_rows = gcd_int(ix.page_size, kTileKeys);
  const int hshift = __builtin_ctz(static_cast<unsigned>(H));
  CUtensorMap kmap, qmap;
  if (!encode_indexer_maps(ix, box_rows, dql, ix.num_rows, &kmap, &qmap))
    return decline("tensor map refused");
  if (ix.dim == 64)
    return nq == 16 ? plan_and_launch<64, 16>(p, segments, stages_total, optin, box_rows, hshift,
                                              kmap, qmap, stream, why)
                    : plan_and_launch<64, 32>(p, segments, stages_total, optin, box_rows, hshift,
                                              kmap, qmap, stream, why);
  return nq == 16 ? plan_and_launch<128, 16>(p, segments, stages_total, optin, box_rows, hshift,
                                             kmap, qmap, stream, why)
                  : plan_and_launch<128, 32>(p, segments, stages_total, optin, box_rows, hshift,
                                             kmap, qmap, stream, why);
}

}  // namespace qsa
