// Indexer scores on the 5th-generation tensor cores (tcgen05 + TMA), sm_100a.
//
// logits[r, c] = scale * sum_h w[r,h] * relu(q[r,h] . key(c)) for c < visible[r]
// (reference ops/indexer.py:24-114 decode, :117-223 prefill: bf16 inputs, fp32
// products, ReLU per head, head sum, head_dim^-0.5).
//
// Work decomposition.  A "segment" is the group of query rows that share one
// page-table row and one B operand: a decode request (its decode_query_len
// rows) or, in prefill, up to 128/H consecutive rows of one request.  Every
// segment has at most T = ceil(capacity / 128) key tiles of 128 keys; the
// (segment, tile) units are split into contiguous ranges, one per persistent
// CTA (grid = resident CTAs of the whole GPU), so each CTA pays its set-up
// once and streams keys through one continuous pipeline across segments.
//
// Roles (every role loop runs on the whole warp; one lane issues):
//  * warp 0, producer: per segment, reads the rows' visible counts, writes
//    the segment descriptor, head weights and column limits into one of two
//    segment slots and loads the segment's query rows with a TMA tensor copy
//    (128-byte swizzled, column n = row n/H, head n%H).  Then it loads the
//    key tiles page by page with 3-D TMA copies (head dim, slot in page,
//    physical page) into a ring of shared-memory stages.  Page ids come
//    from a 32-page window of the table row held in registers, with the next
//    window already in flight.  An unmapped page is read through an
//    out-of-range page coordinate, which the TMA unit fills with zeros.
//  * warp 1: allocates TMEM and issues tcgen05.mma (M = 128 keys, N = the
//    segment's query columns padded to 16, K = 16 per instruction) into a
//    double-buffered fp32 accumulator; tcgen05.commit releases the stage and
//    publishes the accumulator.
//  * warps 2-5, epilogue: each thread owns one key (one TMEM lane) and,
//    per tile, loads its scores with tcgen05.ld, applies ReLU, the head
//    weights, the head sum and the scale, and stores one fp32 per query row
//    (a warp writes 32 consecutive columns).
// Every wait is bounded: on expiry the error word is set, the CTA stops
// issuing work, waits (bounded) for its own copies and MMAs, releases TMEM
// and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace qsa {
namespace {

constexpr int kEpiGroups = 2;   // epilogue warpgroups; group g takes stages g, g+2, ...
constexpr int kTcThreads = (2 + 4 * kEpiGroups) * 32;  // producer, MMA, 8 epilogue warps

struct SegMeta {
  int r0;       // first absolute query row of the segment
  int nrows;    // rows in the segment
  int k_first;  // first key of this CTA's part of the segment
  int nstages;  // key stages of this CTA's part; < 0 marks the end of the work
};

// Compile-time shape of one instantiation: head dim D, padded query columns NQ.
template <int D, int NQ>
struct TcCfg {
  static constexpr int kSub = D / 64;                  // 128-byte sub-rows per key / query row
  static constexpr int MT = D == 64 ? 2 : 1;           // 128-key MMA tiles per stage
  static constexpr int kStageKeys = MT * kTileKeys;    // 256 keys (D=64) / 128 keys (D=128)
  static constexpr int kSubBytes = kTileKeys * 128;    // one MMA tile, one sub-row: 16 KB
  static constexpr int kStageBytes = MT * kSub * kSubBytes;  // 32 KB
  static constexpr int kQSubBytes = NQ * 128;
  static constexpr int kAccCols = MT * NQ;             // TMEM columns of one stage's scores
  static constexpr int A = kAccCols <= 64 ? 4 : 2;     // accumulator ring (even: one group each)
  static constexpr int kCols = A * kAccCols < 32 ? 32 : A * kAccCols;
  // stages in flight: the 32 KB stages that fit beside the two query slots in
  // half of an SM's shared memory when two CTAs share an SM (two independent
  // pipelines per SM, half-size work ranges), or in all of it when the CTA's
  // TMEM columns (more than half of the SM's 512) leave it alone on the SM;
  // at least two stages
  static constexpr int kSmemBudget = kCols > 256 ? 220 * 1024 : 110 * 1024;
  // wide epilogue (rounds of 64 columns): a 16-row x 32-key fp32 tile per
  // epilogue warp to turn a round's row sums into row-contiguous 16-byte stores
  static constexpr int kTrFloats = kAccCols > 64 ? 16 * 32 : 1;
  static constexpr int kTrBytes = kAccCols > 64 ? 4 * kEpiGroups * kTrFloats * 4 : 0;
  static constexpr int kFit =
      (kSmemBudget - 2 * kSub * kQSubBytes - kTrBytes) / (MT * kSub * kTileKeys * 128);
  static constexpr int S = kFit > 8 ? 8 : (kFit < 2 ? 2 : kFit);
  static_assert(S >= 2, "stage ring too small");
};

template <int D, int NQ>
struct TcSmem {
  using C = TcCfg<D, NQ>;
  // stage layout: [mma tile m][sub][key row][128 B], each 128-key sub-tile 128B-swizzled
  alignas(1024) uint8_t k[C::S][C::kStageBytes];
  alignas(1024) uint8_t q[2][C::kSub][C::kQSubBytes];  // [slot][sub][column][128 B], swizzled
  float tr[4 * kEpiGroups][C::kTrFloats];  // per epilogue warp (wide epilogue only)
  SegMeta meta[2];
  float w[2][NQ];
  int limit[2][NQ];  // per row of the segment: columns below this are stored
  uint64_t full[C::S], empty[C::S], tfull[C::A], tempty[C::A], segfull[2], segempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct TcGeometry {
  int segments;       // segment slots (prefill: requests x row tiles, some empty)
  int row_tiles;      // prefill row tiles per request (1 for decode)
  int rows_per_seg;   // rows of a full segment
  int stages_per_seg; // key-stage upper bound per segment
  int box_rows;       // key rows per TMA box (divides the page and 128)
  int64_t units;      // segments x stages_per_seg
};

// Rows [r0, r1) of segment `seg` (absolute packed rows); r0 >= r1 if empty.
__device__ __forceinline__ void segment_rows(const IndexerParams& p, const TcGeometry& g, int seg,
                                             int& r0, int& r1) {
  if (p.query_start_loc == nullptr) {
    r0 = seg * p.decode_query_len;
    r1 = r0 + p.decode_query_len;
    return;
  }
  const int req = seg / g.row_tiles, rt = seg % g.row_tiles;
  const int base = p.query_start_loc[0];
  const int qend = p.query_offset + p.num_rows;
  const int rs = max(p.query_start_loc[req] - base, p.query_offset);
  const int re = min(p.query_start_loc[req + 1] - base, qend);
  r0 = rs + rt * g.rows_per_seg;
  r1 = min(r0 + g.rows_per_seg, re);
}

// Epilogue arithmetic.  Every product and sum is rounded on its own
// (__fmul_rn / __fadd_rn: no FMA contraction), and for a given head count the
// heads of a row are added in one fixed order (a log-depth tree over adjacent
// columns for a power-of-two count), so every formulation below, and the
// fused decode selection (select_decode.cu), give the same fp32 bits.
//
// Sequential form (any head count): ReLU, head weight,
// sum of the H heads of each row, scaled store.  (acc, h, ri) carry a row
// across calls.
template <int N>
__device__ __forceinline__ void score_columns_seq(const uint32_t* v, const float* wv, int c0,
                                                  int H, float& acc, int& h, int& ri,
                                                  int rows_here, const int* lim, float* out,
                                                  int64_t row_stride, int key, float scale) {
  float r[N];
#pragma unroll
  for (int x = 0; x < N; ++x) r[x] = __fmul_rn(fmaxf(__uint_as_float(v[x]), 0.f), wv[c0 + x]);
#pragma unroll
  for (int x = 0; x < N; ++x) {
    acc = __fadd_rn(acc, r[x]);
    if (++h == H) {
      if (ri < rows_here && key < lim[ri]) out[static_cast<int64_t>(ri) * row_stride + key] = acc * scale;
      acc = 0.f;
      h = 0;
      ++ri;
    }
  }
}

// Power-of-two head count, all of a key's columns in one chunk, with the
// segment's head weights and per-column store limits held in registers
// (lim_col[n]: columns of key index below it are stored for column n's row;
// 0 for padding rows).
template <int N>
__device__ __forceinline__ void score_columns_pow2_reg(const uint32_t* v, const float* wr,
                                                       const int* lim_col, int H, int hshift,
                                                       float* out, int64_t row_stride, int key,
                                                       float scale) {
  float r[N];
#pragma unroll
  for (int x = 0; x < N; ++x) r[x] = __fmul_rn(fmaxf(__uint_as_float(v[x]), 0.f), wr[x]);
#pragma unroll
  for (int step = 1; step < N; step <<= 1) {
    if (step < H) {
#pragma unroll
      for (int x = 0; x + step < N; x += 2 * step) r[x] = __fadd_rn(r[x], r[x + step]);
    }
  }
#pragma unroll
  for (int x = 0; x < N; ++x)
    if ((x & (H - 1)) == 0 && key < lim_col[x])
      out[static_cast<int64_t>(x >> hshift) * row_stride + key] = r[x] * scale;
}

// Epilogue arithmetic for a power-of-two head count H, fixed at compile time:
// the heads of a row are summed by a log-depth tree over the chunk's columns,
// then the chunk's N/H row sums are stored (one limit load and one store per
// row).  A row wider than the chunk (H > N) is carried in `carry` and stored
// by its last chunk.
template <int N, int H>
__device__ __forceinline__ void score_columns_h(const uint32_t* v, const float* wv, int c0,
                                                float& carry, int rows_here, const int* lim,
                                                float* out, int64_t row_stride, int key,
                                                float scale) {
  // The rows' store limits are read before the first store: the compiler
  // cannot move a (generic-pointer) limit load above an earlier logits store,
  // so loads interleaved with the stores would serialise on their latency.
  constexpr int kRows = H <= N ? N / H : 1;
  int lm[kRows];
#pragma unroll
  for (int j = 0; j < kRows; ++j) {
    const int ri = H <= N ? c0 / H + j : c0 / H;
    lm[j] = ri < rows_here ? lim[ri] : 0;
  }
  float r[N];
#pragma unroll
  for (int x = 0; x < N; ++x) r[x] = __fmul_rn(fmaxf(__uint_as_float(v[x]), 0.f), wv[c0 + x]);
  constexpr int kSpan = H < N ? H : N;  // columns summed per tree
#pragma unroll
  for (int step = 1; step < kSpan; step <<= 1) {
#pragma unroll
    for (int x = 0; x + step < N; x += 2 * step) r[x] = __fadd_rn(r[x], r[x + step]);
  }
  if constexpr (H <= N) {
#pragma unroll
    for (int j = 0; j < N / H; ++j) {
      const int ri = c0 / H + j;
      if (key < lm[j]) out[static_cast<int64_t>(ri) * row_stride + key] = r[j * H] * scale;
    }
  } else {
    carry = __fadd_rn(carry, r[0]);
    if ((c0 + N) % H == 0) {
      const int ri = c0 / H;
      if (key < lm[0]) out[static_cast<int64_t>(ri) * row_stride + key] = carry * scale;
      carry = 0.f;
    }
  }
}

// Power-of-two head count H = 1 << hshift (warp-uniform dispatch).
template <int N>
__device__ __forceinline__ void score_columns_pow2(const uint32_t* v, const float* wv, int c0,
                                                   int hshift, float& carry, int rows_here,
                                                   const int* lim, float* out,
                                                   int64_t row_stride, int key, float scale) {
  switch (hshift) {
    case 0: score_columns_h<N, 1>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
    case 1: score_columns_h<N, 2>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
    case 2: score_columns_h<N, 4>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
    case 3: score_columns_h<N, 8>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
    case 4: score_columns_h<N, 16>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
    case 5: score_columns_h<N, 32>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
    case 6: score_columns_h<N, 64>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
    default: score_columns_h<N, 128>(v, wv, c0, carry, rows_here, lim, out, row_stride, key, scale); break;
  }
}

// Wide-epilogue arithmetic for a power-of-two head count 4 <= H <= 32: the
// R = N/H row sums of each key go through the warp's shared tile (row r, key
// lane) and leave as 16-byte stores of 4 consecutive keys of one row; a chunk
// that straddles its row's store limit is written element by element.  The
// rows' limits are read before the first store (see score_columns_h).
// Requires 16-byte aligned logits rows.
template <int N, int H>
__device__ __forceinline__ void score_columns_tr(const uint32_t* v, const float* wv, int c0,
                                                 int rows_here, const int* lim, float* out,
                                                 int64_t row_stride, int key_base, float scale,
                                                 float* tile) {
  constexpr int R = N / H;                      // rows of this chunk
  constexpr int kChunks = R * 8;                // 16-byte chunks: 8 per row of 32 keys
  constexpr int kPer = (kChunks + 31) / 32;     // chunks per lane
  const int lane = threadIdx.x & 31;
  const int row0 = c0 / H;
  int lm[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int ri = row0 + (lane + 32 * i) / 8;
    lm[i] = (lane + 32 * i < kChunks && ri < rows_here) ? lim[ri] : 0;
  }
  float r[N];
#pragma unroll
  for (int x = 0; x < N; ++x) r[x] = __fmul_rn(fmaxf(__uint_as_float(v[x]), 0.f), wv[c0 + x]);
#pragma unroll
  for (int step = 1; step < H; step <<= 1) {
#pragma unroll
    for (int x = 0; x + step < N; x += 2 * step) r[x] = __fadd_rn(r[x], r[x + step]);
  }
#pragma unroll
  for (int j = 0; j < R; ++j) tile[j * 32 + lane] = r[j * H] * scale;
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int q = lane + 32 * i;
    if (q < kChunks) {
      const int row = q / 8, k4 = (q % 8) * 4;
      const float4 val = *reinterpret_cast<const float4*>(tile + row * 32 + k4);
      const int key = key_base + k4;
      float* dst = out + static_cast<int64_t>(row0 + row) * row_stride + key;
      if (key + 3 < lm[i]) {
        *reinterpret_cast<float4*>(dst) = val;
      } else {
        if (key < lm[i]) dst[0] = val.x;
        if (key + 1 < lm[i]) dst[1] = val.y;
        if (key + 2 < lm[i]) dst[2] = val.z;
      }
    }
  }
  __syncwarp();  // the tile is rewritten by the next round
}

// H = 1 << hshift with 2 <= hshift <= 5 (warp-uniform dispatch).
template <int N>
__device__ __forceinline__ void score_columns_tr_pow2(const uint32_t* v, const float* wv, int c0,
                                                      int hshift, int rows_here, const int* lim,
                                                      float* out, int64_t row_stride,
                                                      int key_base, float scale, float* tile) {
  switch (hshift) {
    case 2: score_columns_tr<N, 4>(v, wv, c0, rows_here, lim, out, row_stride, key_base, scale, tile); break;
    case 3: score_columns_tr<N, 8>(v, wv, c0, rows_here, lim, out, row_stride, key_base, scale, tile); break;
    case 4: score_columns_tr<N, 16>(v, wv, c0, rows_here, lim, out, row_stride, key_base, scale, tile); break;
    default: score_columns_tr<N, 32>(v, wv, c0, rows_here, lim, out, row_stride, key_base, scale, tile); break;
  }
}

template <int D, int NQ>
__global__ void __launch_bounds__(kTcThreads) indexer_tc_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap qmap,
    const IndexerParams p, const TcGeometry g) {
  using C = TcCfg<D, NQ>;
  using Sm = TcSmem<D, NQ>;
  constexpr int S = C::S, A = C::A, MT = C::MT;
  constexpr uint32_t kIdesc = instr_desc<kTileKeys, NQ>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the 128-byte swizzle pattern is taken from address bits: 1024-byte align
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = p.heads;
  const int cap = min(p.table_width * p.page_size, p.logits_width);

  // this CTA's contiguous range of (segment, key stage) units
  const int64_t ua = g.units * blockIdx.x / gridDim.x;
  const int64_t ub = g.units * (blockIdx.x + 1) / gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < A; ++a) {
      mbar_init(&sm.tfull[a], 1);
      mbar_init(&sm.tempty[a], 4);  // the four warps of the group that owns the buffer
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.segfull[b], 1);
      mbar_init(&sm.segempty[b], 4 * kEpiGroups);
    }
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&qmap);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(C::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ================================================================ producer
    const int boxes = C::kStageKeys / g.box_rows;  // <= 32: one lane per box
    const uint32_t qbytes = static_cast<uint32_t>(C::kSub * H * g.rows_per_seg * 128);
    int it = 0;  // key stages issued (stage ring position)
    int j = 0;   // segments published (slot ring position)
    bool ok = true;
    int64_t u = ua;
    while (u < ub && ok) {
      const int seg = static_cast<int>(u / g.stages_per_seg);
      const int64_t seg_first = static_cast<int64_t>(seg) * g.stages_per_seg;
      const int ta = static_cast<int>(u - seg_first);
      const int64_t u_next = min(ub, seg_first + g.stages_per_seg);
      const int tb0 = static_cast<int>(u_next - seg_first);
      u = u_next;
      int r0, r1;
      segment_rows(p, g, seg, r0, r1);
      if (r0 >= r1) continue;
      const int nrows = r1 - r0;
      const int table_row = p.query_start_loc == nullptr ? seg : seg / g.row_tiles;
      const int32_t* trow = p.table + static_cast<int64_t>(table_row) * p.table_row_stride;
      // All of the segment's metadata loads are issued before any is used:
      // visible counts, head weights and a 64-page window of the table row
      // (cur: pages wbase.., nxt: wbase+32..).  Pages past the visible keys
      // may be read; their scores are never stored.
      auto page_of = [&](int lp) { return lp < p.table_width ? ld_once(trow + lp) : -1; };
      int wbase = static_cast<int>(p.page_div.div(ta * C::kStageKeys));
      int cur = page_of(wbase + lane);
      int nxt = page_of(wbase + 32 + lane);
      int vis_lane[(NQ + 31) / 32];
      float w_lane[(NQ + 31) / 32];
#pragma unroll
      for (int i = 0; i < (NQ + 31) / 32; ++i) {
        const int n = lane + 32 * i;
        const int ri = n / H, h = n - ri * H;
        vis_lane[i] = n < nrows ? min(row_visible(p, r0 + n), cap) : 0;
        w_lane[i] = 0.f;
        if (n < NQ && ri < nrows)
          w_lane[i] = p.weights ? p.weights[static_cast<int64_t>(r0 + ri) * p.w_row_stride +
                                            static_cast<int64_t>(h) * p.w_head_stride]
                                : 1.f;
      }
      int maxvis = 0;
#pragma unroll
      for (int i = 0; i < (NQ + 31) / 32; ++i) maxvis = max(maxvis, vis_lane[i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        maxvis = max(maxvis, __shfl_xor_sync(0xffffffffu, maxvis, o));
      const int tb = min(tb0, (maxvis + C::kStageKeys - 1) / C::kStageKeys);
      if (ta >= tb) continue;

      // ---- publish the segment: descriptor, weights, limits, query rows
      const int slot = j & 1;
      if (aborted(&sm.abort_flag) ||
          (j >= 2 && !warp_wait(&sm.segempty[slot], ((j >> 1) - 1) & 1))) {
        ok = false;
        break;
      }
#pragma unroll
      for (int i = 0; i < (NQ + 31) / 32; ++i) {
        const int n = lane + 32 * i;
        if (n < NQ) {
          sm.w[slot][n] = w_lane[i];
          sm.limit[slot][n] = vis_lane[i];
        }
      }
      if (lane == 0) sm.meta[slot] = SegMeta{r0, nrows, ta * C::kStageKeys, tb - ta};
      __syncwarp();
      if (lane == 0) {
        mbar_expect_tx(&sm.segfull[slot], qbytes);
#pragma unroll
        for (int sub = 0; sub < C::kSub; ++sub)
          tma_load_3d(sm.q[slot][sub], &qmap, sub * 64, 0, r0, &sm.segfull[slot]);
        mbar_arrive(&sm.segfull[slot]);
      }
      ++j;

      // ---- key stages [ta, tb): lane b loads box b of each stage
      const int box_key = lane * g.box_rows;  // this lane's box, relative to the stage
      const int box_m = box_key / kTileKeys, box_row = box_key % kTileKeys;
      for (int t = ta; t < tb; ++t) {
        const int s = it % S;
        if (aborted(&sm.abort_flag) ||
            (it >= S && !warp_wait(&sm.empty[s], ((it / S) - 1) & 1))) {
          ok = false;
          break;
        }
        const int key0 = t * C::kStageKeys;
        if (static_cast<int>(p.page_div.div(key0)) >= wbase + 32) {  // at most one page in 32
          wbase += 32;
          cur = nxt;
          nxt = page_of(wbase + 32 + lane);
        }
        int lp, off;
        p.page_div.divmod(key0 + box_key, lp, off);
        const int d = lp - wbase;  // < 64: a stage spans at most 32 pages
        const int pc = __shfl_sync(0xffffffffu, cur, d & 31);
        const int pn = __shfl_sync(0xffffffffu, nxt, d & 31);
        int page = d < 32 ? pc : pn;
        if (page < 0 || page >= p.num_blocks) page = p.num_blocks;  // zero-filled
        if (lane == 0) mbar_expect_tx(&sm.full[s], C::kStageBytes);
        __syncwarp();
        if (lane < boxes) {
          uint8_t* dst = sm.k[s] + box_m * (C::kSub * C::kSubBytes) + box_row * 128;
#pragma unroll
          for (int sub = 0; sub < C::kSub; ++sub)
            tma_load_3d(dst + sub * C::kSubBytes, &kmap, sub * 64, off, page, &sm.full[s]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.full[s]);
        ++it;
      }
    }
    if (ok) {  // end marker in the next slot
      const int slot = j & 1;
      if (j >= 2 && !warp_wait(&sm.segempty[slot], ((j >> 1) - 1) & 1)) {
        ok = false;
      } else if (lane == 0) {
        sm.meta[slot] = SegMeta{0, 0, 0, -1};
        mbar_arrive(&sm.segfull[slot]);
      }
    }
    if (!ok && lane == 0) {
      record_error(p.err, kDeviceErrWaitTimeout);
      sm.abort_flag = 1;
    }
    // drain: every copy this CTA issued has landed before it may retire
    for (int x = max(0, it - S); x < it; ++x)
      if (!warp_wait(&sm.full[x % S], (x / S) & 1) && lane == 0)
        record_error(p.err, kDeviceErrWaitTimeout);
    // query rows: with the end marker published, segment j-2's rows have
    // landed (its slot was released by the epilogue) and its slot has moved
    // on to the marker's phase, so only segment j-1 is waited for.
    for (int x = max(0, ok ? j - 1 : j - 2); x < j; ++x)
      if (!warp_wait(&sm.segfull[x & 1], (x >> 1) & 1) && lane == 0)
        record_error(p.err, kDeviceErrWaitTimeout);
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    int it = 0, j = 0;
    bool ok = true;
    while (ok) {
      const int slot = j & 1;
      if (aborted(&sm.abort_flag) || !warp_wait(&sm.segfull[slot], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      const SegMeta m = sm.meta[slot];
      if (m.nstages < 0) break;
      const uint32_t qbase = smem_u32(sm.q[slot][0]);
      for (int t = 0; t < m.nstages; ++t) {
        const int s = it % S, a = it % A;
        if (aborted(&sm.abort_flag) || !warp_wait(&sm.full[s], (it / S) & 1) ||
            (it >= A && !warp_wait(&sm.tempty[a], ((it / A) - 1) & 1))) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (lane == 0) {
          const uint32_t kbase = smem_u32(sm.k[s]);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int sub = kk >> 2, part = kk & 3;
              const uint64_t ad = sw128_desc(kbase + (mt * C::kSub + sub) * C::kSubBytes + part * 32);
              const uint64_t bd = sw128_desc(qbase + sub * C::kQSubBytes + part * 32);
              umma_bf16(tmem + a * C::kAccCols + mt * NQ, ad, bd, kIdesc, kk > 0);
            }
          }
          umma_commit(&sm.empty[s]);  // stage reusable once these MMAs have read it
          umma_commit(&sm.tfull[a]);  // accumulator a ready for the epilogue
        }
        __syncwarp();
        ++it;
      }
      ++j;
    }
    if (!ok && lane == 0) {
      record_error(p.err, kDeviceErrWaitTimeout);
      sm.abort_flag = 1;
    }
    // drain: the last MMAs have completed before TMEM is released
    if (it > 0 && !warp_wait(&sm.tfull[(it - 1) % A], ((it - 1) / A) & 1) && lane == 0)
      record_error(p.err, kDeviceErrWaitTimeout);
  } else {
    // ================================================================ epilogue
    const int grp = (warp - 2) >> 2;  // stages grp, grp + 2, ...
    const int quad = warp & 3;        // TMEM lanes 32*quad .. +31 = keys of this warp
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const float scale = p.scale;
    const int hshift = (H & (H - 1)) == 0 ? __ffs(H) - 1 : -1;  // log2(H), or -1
    // wide epilogue through the shared tile: 4 <= H <= 32, 16-byte aligned rows
    const bool tr_path = C::kAccCols > 64 && hshift >= 2 && hshift <= 5 &&
                         (p.logits_row_stride & 3) == 0 &&
                         (reinterpret_cast<uintptr_t>(p.logits) & 15) == 0;
    float* tile = sm.tr[warp - 2];
    int it = 0, j = 0;
    bool ok = true;
    while (ok) {
      const int slot = j & 1;
      if (aborted(&sm.abort_flag) || !warp_wait(&sm.segfull[slot], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      const SegMeta m = sm.meta[slot];
      if (m.nstages < 0) break;
      const float* wv = sm.w[slot];
      const int* lim = sm.limit[slot];
      const int rows_here = min(NQ / H, m.nrows);
      float* out = p.logits + static_cast<int64_t>(m.r0 - p.query_offset) * p.logits_row_stride;
      // small shapes: the segment's weights and column limits in registers
      constexpr bool kRegPath = C::kAccCols <= 32;
      constexpr int kRegCols = kRegPath ? NQ : 1;
      float wr[kRegCols];
      int lim_col[kRegCols];
      if constexpr (kRegPath) {
#pragma unroll
        for (int x = 0; x < NQ; ++x) {
          wr[x] = wv[x];
          const int ri = hshift >= 0 ? x >> hshift : x / H;
          lim_col[x] = ri < rows_here ? lim[ri] : 0;
        }
      }
      for (int t = 0; t < m.nstages; ++t, ++it) {
        if ((it & 1) != grp) continue;
        const int a = it % A;
        if (aborted(&sm.abort_flag) || !warp_wait(&sm.tfull[a], (it / A) & 1)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int key0 = m.k_first + t * C::kStageKeys + quad * 32 + lane;
        const uint32_t acc_base = tmem + lane_base + a * C::kAccCols;
        constexpr int CH = C::kAccCols <= 64 ? NQ : 64;  // columns per arithmetic chunk
        if constexpr (C::kAccCols <= 64) {
          // all of this stage's columns in one round of loads
          uint32_t v[C::kAccCols];
#pragma unroll
          for (int c = 0; c < C::kAccCols; c += 16) tmem_ld16(acc_base + c, v + c);
          tmem_wait_ld();
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int key = key0 + mt * kTileKeys;
            if (kRegPath && hshift >= 0) {
              score_columns_pow2_reg<CH>(v + mt * NQ, wr, lim_col, H, hshift, out,
                                         p.logits_row_stride, key, scale);
            } else if (hshift >= 0) {
              float carry = 0.f;
              score_columns_pow2<CH>(v + mt * NQ, wv, 0, hshift, carry, rows_here, lim, out,
                                     p.logits_row_stride, key, scale);
            } else {
              float acc = 0.f;
              int h = 0, ri = 0;
              score_columns_seq<CH>(v + mt * NQ, wv, 0, H, acc, h, ri, rows_here, lim, out,
                                    p.logits_row_stride, key, scale);
            }
          }
        } else {
          // 64 columns per round of loads; a row may span rounds.  The
          // rounds share one copy of the (unrolled) 64-column body: unrolled
          // rounds would outgrow the instruction cache.
#pragma unroll 1
          for (int mt = 0; mt < MT; ++mt) {
            const int key = key0 + mt * kTileKeys;
            float acc = 0.f;
            int h = 0, ri = 0;
#pragma unroll 1
            for (int c0 = 0; c0 < NQ; c0 += CH) {
              uint32_t v[CH];
#pragma unroll
              for (int c = 0; c < CH; c += 16) tmem_ld16(acc_base + mt * NQ + c0 + c, v + c);
              tmem_wait_ld();
              if (tr_path)
                score_columns_tr_pow2<CH>(v, wv, c0, hshift, rows_here, lim, out,
                                          p.logits_row_stride, key - lane, scale, tile);
              else if (hshift >= 0)
                score_columns_pow2<CH>(v, wv, c0, hshift, acc, rows_here, lim, out,
                                       p.logits_row_stride, key, scale);
              else
                score_columns_seq<CH>(v, wv, c0, H, acc, h, ri, rows_here, lim, out,
                                      p.logits_row_stride, key, scale);
            }
          }
        }
        // the scores are in registers (tcgen05.wait::ld above): hand the
        // accumulator back without waiting for this warp's logits stores
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_relaxed(&sm.tempty[a]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.segempty[slot]);  // slot's rows, weights, limits done
      ++j;
    }
    if (!ok && lane == 0) {
      record_error(p.err, kDeviceErrWaitTimeout);
      sm.abort_flag = 1;
    }
  }
  // every role loop is warp-uniform, so each warp arrives here converged
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------- host side
template <int D, int NQ>
cudaError_t launch_tc(const IndexerParams& p, const CUtensorMap& kmap, const CUtensorMap& qmap,
                      const TcGeometry& g, cudaStream_t stream) {
  using C = TcCfg<D, NQ>;
  const void* fn = reinterpret_cast<const void*>(indexer_tc_kernel<D, NQ>);
  const size_t smem = sizeof(TcSmem<D, NQ>) + 1024;  // + slack for 1024-byte alignment
  cudaError_t e = set_attr_once(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // all of the SM's unified L1/shared storage as shared memory, so that two
  // CTAs' stage rings fit on one SM
  e = set_attr_once(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                    cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  // Resident CTAs per SM from the SM's shared memory and registers (each CTA
  // also reserves 1 KB of shared memory), capped by the 512 TMEM columns.
  int dev = 0, sm_smem = 0, sm_regs = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&sm_regs, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
  cudaFuncAttributes fa{};
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, fn);
  if (e != cudaSuccess) return e;
  const int by_smem = sm_smem / static_cast<int>(smem + 1024);
  const int by_regs = sm_regs / std::max(1, fa.numRegs * kTcThreads);
  const int per_sm = std::max(1, std::min({by_smem, by_regs, 512 / C::kCols}));
  const int64_t ctas = std::min<int64_t>(g.units, static_cast<int64_t>(num_sms()) * per_sm);
  return count_launches(launch_kernel(indexer_tc_kernel<D, NQ>, dim3(static_cast<int>(ctas)),
                                      dim3(kTcThreads), smem, stream, 1, kmap, qmap, p, g));
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int gcd_int(int a, int b) {
  while (b) {
    const int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

// Tensor maps of the indexer's operands.  Key cache: (head dim, slot in
// page, page) with boxes of 64 dims x box_rows slots; query rows: (head dim,
// head, row) with boxes of 64 dims x all heads x rows_per_seg rows.  Both
// 128-byte swizzled.  False when the driver refuses the layout.
bool encode_indexer_maps(const IndexerParams& p, int box_rows, int rows_per_seg, int q_rows,
                         CUtensorMap* kmap, CUtensorMap* qmap) {
  const int H = p.heads;
  const cuuint32_t estr[3] = {1, 1, 1};
  {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.dim),
                                static_cast<cuuint64_t>(p.page_size),
                                static_cast<cuuint64_t>(p.num_blocks)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.token_stride) * 2,
                                   static_cast<cuuint64_t>(p.block_stride) * 2};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
    if (tensor_map_encoder()(kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                             const_cast<void*>(p.k_cache), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  {
    const int64_t hs = H == 1 ? p.dim : p.q_head_stride;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.dim), static_cast<cuuint64_t>(H),
                                static_cast<cuuint64_t>(q_rows)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(hs) * 2,
                                   static_cast<cuuint64_t>(p.q_row_stride) * 2};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(H),
                               static_cast<cuuint32_t>(rows_per_seg)};
    if (tensor_map_encoder()(qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p.q),
                             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  return true;
}

// Whether the tensor-core indexer takes these shapes (else the mma.sync path):
// head dim 64 / 128, page size a multiple of 8 (whole 8-row swizzle atoms per
// TMA box), 16-byte aligned rows and strides, <= 128 query columns per segment.
bool indexer_tc_eligible(const IndexerParams& p) {
  if (p.dim != 64 && p.dim != 128) return false;
  if (p.heads <= 0 || p.heads > 128) return false;
  if (p.page_size % 8 != 0) return false;
  if ((p.token_stride * 2) % 16 != 0 || (p.block_stride * 2) % 16 != 0) return false;
  if (reinterpret_cast<uintptr_t>(p.k_cache) % 16 != 0) return false;
  if (reinterpret_cast<uintptr_t>(p.q) % 16 != 0) return false;
  if ((p.q_row_stride * 2) % 16 != 0) return false;
  if (p.heads > 1 && (p.q_head_stride * 2) % 16 != 0) return false;
  if (p.num_blocks <= 0) return false;
  if (p.query_start_loc == nullptr && p.decode_query_len * p.heads > 128) return false;
  return tensor_map_encoder() != nullptr;
}

cudaError_t launch_indexer_tc(const IndexerParams& p, cudaStream_t stream) {
  const bool decode = p.query_start_loc == nullptr;
  const int H = p.heads;
  TcGeometry g{};
  int q_rows;  // rows addressable through the query tensor map
  if (decode) {
    g.rows_per_seg = p.decode_query_len;
    g.row_tiles = 1;
    g.segments = p.num_rows / p.decode_query_len;
    q_rows = p.num_rows;
  } else {
    g.rows_per_seg = std::max(1, 128 / H);
    g.row_tiles = (std::min(p.num_rows, p.max_query_len) + g.rows_per_seg - 1) / g.rows_per_seg;
    g.segments = p.num_requests * g.row_tiles;
    q_rows = p.query_offset + p.num_rows;
  }
  const int cap = std::min(p.logits_width, p.table_width * p.page_size);
  if (g.segments <= 0 || cap <= 0) return cudaSuccess;
  const int stage_keys = p.dim == 64 ? TcCfg<64, 16>::kStageKeys : TcCfg<128, 16>::kStageKeys;
  g.stages_per_seg = (cap + stage_keys - 1) / stage_keys;
  g.units = static_cast<int64_t>(g.segments) * g.stages_per_seg;
  g.box_rows = gcd_int(p.page_size, kTileKeys);
  const int n = g.rows_per_seg * H;
  const int nq = n <= 16 ? 16 : n <= 32 ? 32 : n <= 64 ? 64 : 128;

  CUtensorMap kmap, qmap;
  if (!encode_indexer_maps(p, g.box_rows, g.rows_per_seg, q_rows, &kmap, &qmap))
    return cudaErrorNotSupported;
  if (p.dim == 64) {
    switch (nq) {
      case 16: return launch_tc<64, 16>(p, kmap, qmap, g, stream);
      case 32: return launch_tc<64, 32>(p, kmap, qmap, g, stream);
      case 64: return launch_tc<64, 64>(p, kmap, qmap, g, stream);
      default: return launch_tc<64, 128>(p, kmap, qmap, g, stream);
    }
  }
  switch (nq) {
    case 16: return launch_tc<128, 16>(p, kmap, qmap, g, stream);
    case 32: return launch_tc<128, 32>(p, kmap, qmap, g, stream);
    case 64: return launch_tc<128, 64>(p, kmap, qmap, g, stream);
    default: return launch_tc<128, 128>(p, kmap, qmap, g, stream);
  }
}

}  // namespace qsa
