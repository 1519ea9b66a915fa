// Paged sparse GQA attention over selected tokens (sm_100a).
//
// Semantics follow the reference split-K kernel and merge (ops/qsa.py:109-303,
// :306-362): s = (q . k) * d^-0.5 in fp32 with base-2 online softmax, P rounded
// to bf16 before P.V with fp32 accumulation, out = acc / max(l, 1e-20) (0 when
// no token is valid), optional bf16 rounding then * sigmoid(gate).  Decode
// indices are physical slots bounded by the per-row valid count; prefill
// indices are logical tokens mapped through the request's block table.
//
// Design (B200).  The work is a gather at 8 flop/byte, so the kernel is built
// around keeping HBM busy:
//  * Persistent CTAs (one per SM) take contiguous ranges of the (row,
//    kv-head group, token tile) work (stream-K), so a row is met by only a
//    few CTAs, each writing one partial of it.  A pair covers HB = up to 4
//    KV heads of one row: a selected token's K||V
//    rows of those heads are one contiguous run (2 KB at head_dim 128), moved
//    by ONE bulk copy (cp.async.bulk on the TMA engine) into a 6-stage
//    shared-memory ring guarded by mbarriers.  Token rows are padded by 16 B
//    so ldmatrix reads are bank-conflict free.  Invalid tokens are zero-filled.
//  * Three producer warps issue the copies, each for every third tile (two
//    stages each: the copy issue itself bounds L2-resident gathers).  The
//    token ids a producer needs are
//    streamed into a small shared-memory ring by cp.async several tiles
//    ahead, and the unit's query rows are bulk-copied into a double buffer,
//    so no global-load latency sits on the issue path.
//  * Eight consumer warps in two groups that take alternate stages (two
//    warps per scheduler hide each other's MMA / shuffle latency).  In a
//    group, each warp owns one (kv head, 16-token sub-tile) of the stage:
//    S^T = K.Q^T on mma.sync with tokens as M and the query heads of the GQA
//    group as N (no padding lanes at group 8), in two independent
//    accumulator chains; P^T is transposed in registers (movmatrix) into the
//    B operand of O^T = V^T.P^T.
//  * A pair met by one CTA only (the common case at prefill) is finished
//    there: the softmax states of the warps that share a KV head are folded
//    in shared memory, normalised, rounded to bf16, gated and stored.  A
//    range boundary inside a pair splits it: each consumer warp writes its
//    piece's normalised fp32 partial + LSE (the reference's split-K format)
//    straight from registers, and a small merge kernel combines the at most
//    sk_ctas - 1 split pairs.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

constexpr int kStages = 6;
constexpr int kGroups = 2;                        // consumer groups take alternate stages
constexpr int kGroupWarps = 4;                    // warps per group: one (head, sub-tile) each
constexpr int kConsumerWarps = kGroups * kGroupWarps;
// Stage s is always consumed by group s % kGroups; with a stage count that is
// not a multiple of kGroups, consecutive uses of a stage would alternate groups
// and a group running two barrier phases ahead would alias the parity wait.
static_assert(kStages % kGroups == 0, "each stage must belong to one consumer group");
// Producer warp p fills the tiles it % kProducers == p: issuing a tile's bulk
// copies costs a warp ~0.6 us, which bounds L2-resident (prefill) gathers, so
// three warps share the issue.  Stage s is always filled by producer
// s % kProducers, which takes its stages in order: its empty-barrier waits
// are never more than one phase ahead (no parity aliasing).
constexpr int kProducers = 3;
static_assert(kStages % kProducers == 0, "each stage must belong to one producer");
constexpr int kThreads = (kConsumerWarps + kProducers) * 32;
constexpr int kRing = 8;       // token-id ring slots per producer (one per own tile)
constexpr int kLookahead = 4;  // own tiles of token ids in flight ahead of the copies
static_assert(kLookahead < kRing, "ring / lookahead sizes");
constexpr float kNegBig = -1.0e20f;

template <int D, int NT, int HB>
struct Smem {
  static constexpr int kTT = 64 / HB;            // tokens per stage
  static constexpr int kRow = HB * 4 * D;        // K||V of HB heads of one token (bytes)
  static constexpr int kBlk = 4 * kRow + 16;     // 4-token block + pad (bytes)
  static constexpr int kQRows = HB * 8 * NT;     // staged query head rows per unit
  // byte offset of token j of a stage: tokens are grouped in blocks of 4 that
  // are copied whole when their slots are consecutive in the cache
  static __device__ __forceinline__ int tok_off(int j) { return (j >> 2) * kBlk + (j & 3) * kRow; }
  alignas(128) uint8_t stage[kStages][(kTT / 4) * kBlk];
  alignas(128) uint8_t q[2][kQRows * 2 * D];
  int32_t ring[kProducers][kRing][kTT];
  // unit-end fold of the warps' softmax states (4 writer slots of one
  // m16n8 column block: (D/16) float4 per lane), reused as the pair's
  // [head][dim] fp32 result (at most 32 heads)
  alignas(16) float comb[32 * D];
  float cm[4][8], cl[4][8];  // writer slot: m and l of its 8 head columns
  uint64_t mask[kStages];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t qfull[2];
  uint64_t qempty[2];
  int abort_flag;
};

struct Unit {
  int row, hg, t0, t1, n_cols;
  bool split;  // another CTA's range meets the pair too
};

// Stream-K split: CTA c owns units [U*c/C, U*(c+1)/C) of the U = pairs x
// pair_tiles work units (pair = (row, kv-head group), pairs in row-major order).
__device__ __forceinline__ int64_t sk_begin(const AttnParams& p, int c) {
  return p.sk_units * c / p.sk_ctas;
}
// The CTA whose range holds unit x: the largest c with U*c/C <= x.
__device__ __forceinline__ int sk_owner(const AttnParams& p, int64_t x) {
  return static_cast<int>(((x + 1) * p.sk_ctas + p.sk_units - 1) / p.sk_units - 1);
}

// The k-th pair this CTA meets (g0 = ua / pair_tiles: the first), its tile
// range inside the pair (clipped to the row's valid tiles; may be empty) and
// whether a range boundary splits it.  Called once per pair by every warp:
// no 64-bit division except where a pair spans several KV-head groups.
template <int TT>
__device__ __forceinline__ Unit unit_of(const AttnParams& p, int groups, int64_t g0, int64_t ua,
                                        int64_t ub, int k) {
  Unit x;
  const int T = p.pair_tiles;
  const int64_t g = g0 + k;
  if (groups == 1) {
    x.hg = 0;
    x.row = static_cast<int>(g);
  } else {
    x.hg = static_cast<int>(g % groups);
    x.row = static_cast<int>(g / groups);
  }
  int n = p.topk_width;
  if (p.valid_counts != nullptr) n = min(max(p.valid_counts[x.row], 0), p.topk_width);
  x.n_cols = n;
  const int tiles = (n + TT - 1) / TT;
  const int64_t first = g * T;
  const int t0 = static_cast<int>(max(ua, first) - first);
  const int t1 = static_cast<int>(min(ub, first + T) - first);
  x.t1 = min(t1, tiles);
  x.t0 = min(t0, x.t1);
  // The CTA ranges partition the units, and this one meets the pair: it is
  // the only one to do so exactly when the pair lies inside its range.
  x.split = first < ua || first + T > ub;
  return x;
}

// Pairs met by this CTA's range [ua, ub).
__device__ __forceinline__ int units_met(const AttnParams& p, int64_t ua, int64_t ub) {
  if (ub <= ua) return 0;
  return static_cast<int>((ub - 1) / p.pair_tiles - ua / p.pair_tiles + 1);
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}

// Per KV head of a finished pair, its GQA group's output in 8-dim chunks
// spread over the 8 / HB consumer warps that share the head.
template <int D, int HB, int NT>
constexpr int kOutItems = (8 * NT * (D / 8) + (8 / HB) * 32 - 1) / ((8 / HB) * 32);

// Gate values of dims d0..d0+7 of one (row, head), packed bf16 pairs.  The
// loads are volatile asm so they stay where they are issued (a unit's start)
// instead of being moved next to their use at the unit's end.
__device__ __forceinline__ uint4 load_gate8(const AttnParams& p, int row, int head, int d0) {
  const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(p.gate) +
                            static_cast<int64_t>(row) * p.gate_row_stride +
                            static_cast<int64_t>(head) * p.gate_head_stride;
  uint4 r;
  if (p.gate_vec) {
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(gp + d0));
    return r;
  }
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];"
                 : "=h"(v)
                 : "l"(gp + static_cast<int64_t>(d0 + i) * p.gate_dim_stride));
    w[i] = v;
  }
  r.x = w[0] | (w[1] << 16);
  r.y = w[2] | (w[3] << 16);
  r.z = w[4] | (w[5] << 16);
  r.w = w[6] | (w[7] << 16);
  return r;
}

// 1 / (1 + e^-x) with the fast exponential and division: a few ulp of fp32,
// far below the bf16 rounding of the gated output.
__device__ __forceinline__ float sigmoid(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// Output dims d0..d0+7 of one (row, head): bf16 rounding; with a gate,
// bf16(o) * sigmoid(gate) rounded again (ops/qsa.py:250-275, :348-358).
__device__ __forceinline__ void store_out8(const AttnParams& p, int row, int head, int d0,
                                           float4 a, float4 b, uint4 gate8) {
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  if (p.gate != nullptr) {
    const uint32_t gw[4] = {gate8.x, gate8.y, gate8.z, gate8.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float g0 = __uint_as_float(gw[i] << 16), g1 = __uint_as_float(gw[i] & 0xffff0000u);
      v[2 * i] = __bfloat162float(__float2bfloat16_rn(v[2 * i])) * sigmoid(g0);
      v[2 * i + 1] = __bfloat162float(__float2bfloat16_rn(v[2 * i + 1])) * sigmoid(g1);
    }
  }
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.out) +
                      static_cast<int64_t>(row) * p.out_row_stride +
                      static_cast<int64_t>(head) * p.out_head_stride + d0;
  if (p.out_vec) {
    *reinterpret_cast<uint4*>(op) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<uint32_t*>(op)[i] = w[i];
  }
}

// Iterator over this CTA's (unit, tile) positions: the producer uses one to
// prefetch token ids ahead of the copies.
template <int TT>
struct Cursor {
  int k, t, units, groups;
  int64_t g0, ua, ub;
  Unit x;
  bool live;
  __device__ void init(const AttnParams& p, int units_, int groups_, int64_t ua_, int64_t ub_) {
    units = units_;
    groups = groups_;
    ua = ua_;
    ub = ub_;
    g0 = ua / p.pair_tiles;
    k = 0;
    t = 0;
    live = k < units;
    if (live) {
      x = unit_of<TT>(p, groups, g0, ua, ub, k);
      t = x.t0;
      advance(p, 0);
    }
  }
  // Moves n positions on (tiles of later units count on from their t0).
  __device__ void advance(const AttnParams& p, int n) {
    t += n;
    while (live && t >= x.t1) {
      const int over = t - x.t1;
      ++k;
      live = k < units;
      if (live) {
        x = unit_of<TT>(p, groups, g0, ua, ub, k);
        t = x.t0 + over;
      }
    }
  }
};

template <int D, int NT, int HB>
__device__ void producer(const AttnParams& p, Smem<D, NT, HB>& sm, int units, int groups,
                         int64_t ua, int64_t ub) {
  const int64_t g0 = ua / p.pair_tiles;  // first pair met
  using S = Smem<D, NT, HB>;
  constexpr int kRow = S::kRow;
  constexpr int TT = S::kTT;
  const int lane = threadIdx.x & 31;
  const int group = p.q_heads / p.kv_heads;
  const uint8_t* kbase = static_cast<const uint8_t*>(p.k_cache);
  const uint8_t* vbase = static_cast<const uint8_t*>(p.v_cache);
  const uint8_t* qbase = static_cast<const uint8_t*>(p.q);
  const int pw = (threadIdx.x >> 5) - kConsumerWarps;  // this producer fills it % kProducers == pw
  int32_t (*ring)[TT] = sm.ring[pw];

  Cursor<TT> ahead;  // this producer's own tiles: positions pw, pw + kProducers, ...
  ahead.init(p, units, groups, ua, ub);
  ahead.advance(p, pw);
  auto prefetch = [&](int slot) {
    if (ahead.live) {
      const int32_t* idx_row = p.indices + static_cast<int64_t>(ahead.x.row) * p.indices_row_stride;
      for (int j = lane; j < TT; j += 32) {
        const int col = ahead.t * TT + j;
        const bool v = col < ahead.x.n_cols;
        cp_async4(&ring[slot][j], v ? idx_row + col : idx_row, v);
      }
      ahead.advance(p, kProducers);
    }
    cp_async_commit();
  };
#pragma unroll 1
  for (int i = 0; i < kLookahead; ++i) prefetch(i % kRing);

  int it = 0, k = 0, own = 0;
  int next_own = pw;  // position of this producer's next own tile
  constexpr int kOwnStages = kStages / kProducers;  // own tile n uses stage pw + kProducers * (n % kOwnStages)

  bool ok = true;
  for (; k < units && ok; ++k) {
    const Unit x = unit_of<TT>(p, groups, g0, ua, ub, k);
    // ---- the unit's query rows -> q[k & 1] (producer 0 only)
    const int qb = k & 1;
    if (pw == 0 && k >= 2 && !mbar_wait(&sm.qempty[qb], ((k >> 1) - 1) & 1)) {
      record_error(p.err, kDeviceErrWaitTimeout);
      sm.abort_flag = 1;
      ok = false;
      break;
    }
    const int nq = HB * group;  // query head rows of this unit
    const uint8_t* qsrc = qbase + 2 * (static_cast<int64_t>(x.row) * p.q_row_stride +
                                       static_cast<int64_t>(x.hg * HB * group) * p.q_head_stride);
    if (pw == 0 && lane == 0) {
      mbar_expect_tx(&sm.qfull[qb], static_cast<uint32_t>(nq * 2 * D));
      if (p.q_head_stride == D) {
        bulk_g2s(sm.q[qb], qsrc, static_cast<uint32_t>(nq * 2 * D), &sm.qfull[qb]);
      } else {
        for (int h = 0; h < nq; ++h)
          bulk_g2s(sm.q[qb] + h * 2 * D, qsrc + 2 * static_cast<int64_t>(h) * p.q_head_stride,
                   2u * D, &sm.qfull[qb]);
      }
      mbar_arrive(&sm.qfull[qb]);
    }
    int req = 0;
    bool req_ok = true;
    if (!p.physical) {
      req = p.token_to_req[x.row];
      req_ok = req >= 0 && req < p.num_requests;
    }
    const int32_t* trow =
        p.block_table + static_cast<int64_t>(req_ok ? req : 0) * p.table_row_stride;
    const int64_t head0 = static_cast<int64_t>(x.hg) * HB;
    const int64_t head_k = head0 * p.k_head_stride, head_v = head0 * p.v_head_stride;
    // this producer's tiles of the unit: positions next_own, next_own + kProducers, ...
    const int it0 = it;  // position of tile x.t0
    for (int t = x.t0 + (next_own - it0); t < x.t1; t += kProducers) {
      it = it0 + (t - x.t0);
      next_own = it + kProducers;
      const int s = pw + kProducers * (own % kOwnStages);  // = it % kStages
      if (own >= kOwnStages && !mbar_wait(&sm.empty[s], ((own / kOwnStages) - 1) & 1)) {
        record_error(p.err, kDeviceErrWaitTimeout);
        sm.abort_flag = 1;
        ok = false;
        break;
      }
      // token ids of this tile: this lane's own cp.async writes (same lane
      // mapping as the prefetch), complete once all but the newest
      // kLookahead-1 groups are.
      cp_async_wait<kLookahead - 1>();

      uint8_t* stage = sm.stage[s];
      const int slot = own % kRing;
      // Lane l handles tokens l and l + 32 of the tile; the second half
      // exists only for one-head pairs (TT = 64).  Every instruction here
      // is on the issue path that bounds L2-resident gathers.
      constexpr int kHalves = TT > 32 ? 2 : 1;
      int64_t off_k[kHalves];
      int slot_id[kHalves];  // physical slot (page * page_size + offset), -1 when masked
#pragma unroll
      for (int h = 0; h < kHalves; ++h) {
        const int j = lane + 32 * h;
        const int col = t * TT + j;
        int sl = -1, page = 0, off = 0;
        if (j < TT && col < x.n_cols) {
          const int tok = ring[slot][j];
          if (p.physical) {
            if (tok >= 0 && static_cast<uint32_t>(tok) < p.num_slots) sl = tok;
          } else {
            int lp;
            p.page_div.divmod(max(tok, 0), lp, off);
            page = req_ok && tok >= 0 && lp < p.table_width ? trow[lp] : -1;
            if (page >= 0 && page < p.num_blocks) sl = page * p.page_size + off;
          }
        }
        slot_id[h] = sl;
        if (p.slot_contig) {  // block stride = page_size x token stride
          off_k[h] = static_cast<int64_t>(max(sl, 0)) * p.k_token_stride + head_k;
        } else {
          if (p.physical) p.page_div.divmod(max(sl, 0), page, off);
          off_k[h] = static_cast<int64_t>(page) * p.k_block_stride +
                     static_cast<int64_t>(off) * p.k_token_stride + head_k;
        }
        if (sl < 0 && j < TT) {  // masked token: zeros, as the reference's masked loads
          uint4* z = reinterpret_cast<uint4*>(stage + S::tok_off(j));
#pragma unroll 4
          for (int c = 0; c < kRow / 16; ++c) z[c] = make_uint4(0, 0, 0, 0);
        }
      }
      // Zero fills (generic proxy) are ordered before this stage's next bulk
      // copies (async proxy), issued after the full -> empty barrier chain;
      // without fills there is nothing to order.
      const unsigned lo = __ballot_sync(0xffffffffu, slot_id[0] >= 0);
      const unsigned hi = kHalves > 1 ? __ballot_sync(0xffffffffu, slot_id[kHalves - 1] >= 0) : 0u;
      constexpr unsigned kLoLanes = TT >= 32 ? 0xffffffffu : (1u << (TT & 31)) - 1u;  // tokens 0..31
      if ((~lo & kLoLanes) != 0u || (kHalves > 1 && ~hi != 0u))  // some token was zero-filled
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      // A 4-token block whose slots are consecutive in a slot-contiguous cache
      // is one run of 4*kRow bytes (4 selected tokens of one compressed block):
      // copy it whole.  cont bit j: token j+1 is the slot after token j.
      unsigned cont[kHalves];
#pragma unroll
      for (int h = 0; h < kHalves; ++h) {
        const int nxt = __shfl_down_sync(0xffffffffu, slot_id[h], 1);
        cont[h] = __ballot_sync(0xffffffffu, slot_id[h] >= 0 && nxt == slot_id[h] + 1);
      }
      if (lane == 0) {
        sm.mask[s] = static_cast<uint64_t>(lo) | (static_cast<uint64_t>(hi) << 32);
        mbar_expect_tx(&sm.full[s], static_cast<uint32_t>(__popc(lo) + __popc(hi)) * kRow);
      }
      __syncwarp();
#pragma unroll
      for (int h = 0; h < kHalves; ++h) {
        if (slot_id[h] < 0) continue;
        const int j = lane + 32 * h;
        uint8_t* dst = stage + S::tok_off(j);
        const bool whole = p.kv_fused == 2 && p.slot_contig && p.kv_heads == HB &&
                           ((cont[h] >> (lane & ~3)) & 7u) == 7u;
        if (whole) {
          if ((lane & 3) == 0) bulk_g2s(dst, kbase + 2 * off_k[h], 4u * kRow, &sm.full[s]);
        } else if (p.kv_fused == 2) {  // all HB heads' K||V rows of the token contiguous
          bulk_g2s(dst, kbase + 2 * off_k[h], kRow, &sm.full[s]);
        } else if (p.kv_fused == 1) {  // K||V adjacent per head
#pragma unroll 1
          for (int hh = 0; hh < HB; ++hh)
            bulk_g2s(dst + hh * 4 * D, kbase + 2 * (off_k[h] + hh * p.k_head_stride), 4u * D,
                     &sm.full[s]);
        } else {  // K and V apart: V's own strides
          int page, off;
          p.page_div.divmod(slot_id[h], page, off);
          const int64_t off_v = static_cast<int64_t>(page) * p.v_block_stride +
                                static_cast<int64_t>(off) * p.v_token_stride + head_v;
#pragma unroll 1
          for (int hh = 0; hh < HB; ++hh) {
            bulk_g2s(dst + hh * 4 * D, kbase + 2 * (off_k[h] + hh * p.k_head_stride), 2u * D,
                     &sm.full[s]);
            bulk_g2s(dst + hh * 4 * D + 2 * D, vbase + 2 * (off_v + hh * p.v_head_stride), 2u * D,
                     &sm.full[s]);
          }
        }
      }
      mbar_arrive(&sm.full[s]);
      prefetch((own + kLookahead) % kRing);
      ++own;
    }
    if (ok) it = it0 + (x.t1 - x.t0);
  }
  // Drain: never leave while a copy into this CTA's shared memory may be in
  // flight.  Wait (bounded) for the last issued phase of every barrier.
  cp_async_wait<0>();
  for (int j = std::max(0, it - kStages); j < it; ++j) {
    if (j % kProducers != pw) continue;
    if (!mbar_wait(&sm.full[j % kStages], (j / kStages) & 1))
      record_error(p.err, kDeviceErrWaitTimeout);
  }
  for (int j = std::max(0, k - 2); j < k && pw == 0; ++j) {
    if (!mbar_wait(&sm.qfull[j & 1], (j >> 1) & 1)) record_error(p.err, kDeviceErrWaitTimeout);
  }
}

template <int D, int NT, int HB>
__device__ void consumer(const AttnParams& p, Smem<D, NT, HB>& sm, int units, int groups,
                         int64_t ua, int64_t ub) {
  const int64_t g0 = ua / p.pair_tiles;  // first pair met
  using S = Smem<D, NT, HB>;
  constexpr int TT = S::kTT;
  constexpr int SUB = kGroupWarps / HB;  // 16-token sub-tiles per stage per head
  constexpr int KS = D / 16;             // k-steps of S^T, m-tiles of O^T
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int cg = warp / kGroupWarps;  // consumer group: takes stages it % kGroups == cg
  const int w4 = warp % kGroupWarps;
  const int hh = w4 % HB, sub = w4 / HB;
  const int group = p.q_heads / p.kv_heads;
  const float scale_log2 = p.scale_log2;
  const uint32_t stage0 = smem_u32(&sm.stage[0][0]);
  constexpr uint32_t kStageBytes = (TT / 4) * S::kBlk;
  // MMA row r (0..15) of this warp's sub-tile is token (r>>2) of block
  // 4*sub + (r&3): the 8 rows of one ldmatrix span 4 blocks (2-way bank
  // conflict at most; tokens of a block are contiguous, unpadded).
  auto row_tok = [&](int r) { return (4 * sub + (r & 3)) * 4 + (r >> 2); };
  //   K (A operand of S^T, non-transposed): row = token, 16-byte chunk = dim/8
  const uint32_t a_off =
      static_cast<uint32_t>(S::tok_off(row_tok(lane & 15)) + hh * 4 * D + (lane >> 4) * 16);
  //   V (A operand of O^T, transposed): {rows0-7,d0-7},{rows0-7,d8-15},{rows8-15,d0-7},{rows8-15,d8-15}
  const int mi = lane >> 3;
  const uint32_t v_off = static_cast<uint32_t>(
      S::tok_off(row_tok((lane & 7) + ((mi >> 1) << 3))) + hh * 4 * D + 2 * D + (mi & 1) * 16);

  // After a bounded wait expires (error recorded, abort flag raised) a warp
  // neither waits nor computes any more, but it still walks every unit and
  // reaches every named barrier, so no warp of the CTA is left waiting at one.
  bool aborted = false;
  int it = 0, k = 0;
  // this group's next stage: cg + kGroups * gslot, barrier phase parity gphase
  int gslot = 0;
  uint32_t gphase = 0;
  const int hqp = HB * group;  // query heads of a pair
  // The R = 8 / HB warps sharing KV head hh.
  constexpr int R = kGroups * SUB;
  constexpr int kItems = kOutItems<D, HB, NT>;
  const int head0 = hh * group;  // first query head of hh within the pair
  for (; k < units; ++k) {
    const Unit x = unit_of<TT>(p, groups, g0, ua, ub, k);
    const int qb = k & 1;
    // Rank j of this warp among the head's R warps for the unit-end fold:
    // the group that takes the unit's last tile (and so finishes last) ranks
    // above the other, so in the first folding round it only stores its
    // state and the warps that finished earlier do the folding.  tr: thread
    // rank.
    const int lastg = (it + max(x.t1 - x.t0, 1) - 1) % kGroups;
    const int j = (cg == lastg ? SUB : 0) + sub;
    const int tr = j * 32 + lane;
    // The gate chunks this thread stores at the unit's end, loaded now so
    // their latency hides behind the unit's tiles.
    uint4 gpre[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i) gpre[i] = make_uint4(0, 0, 0, 0);
    if (p.gate != nullptr && !x.split) {
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int item = tr + i * R * 32;
        if (item < group * (D / 8))
          gpre[i] = load_gate8(p, x.row, x.hg * hqp + head0 + item / (D / 8),
                               (item % (D / 8)) * 8);
      }
    }
    aborted = aborted || *reinterpret_cast<volatile int*>(&sm.abort_flag);
    if (!aborted && !mbar_wait(&sm.qfull[qb], (k >> 1) & 1)) {
      record_error(p.err, kDeviceErrWaitTimeout);
      sm.abort_flag = 1;
      aborted = true;
    }
    // Q^T fragments (B operand of S^T): b0 = Q[head g][dims 2t4..], b1 = +8 dims.
    uint32_t qf[KS][NT][2];
    const uint8_t* qs = sm.q[qb];
#pragma unroll
    for (int nt = 0; nt < NT && !aborted; ++nt) {
      const int hl = g + 8 * nt;
      const bool hv = hl < group;
      const uint32_t* qrow =
          reinterpret_cast<const uint32_t*>(qs + (hh * group + (hv ? hl : 0)) * 2 * D);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[ks][nt][0] = hv ? qrow[ks * 8 + t4] : 0u;
        qf[ks][nt][1] = hv ? qrow[ks * 8 + 4 + t4] : 0u;
      }
    }
    __syncwarp();
    if (lane == 0 && !aborted) mbar_arrive(&sm.qempty[qb]);

    float m[NT][2], l[NT][2];
    float o[KS][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = kNegBig;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
    }

    // this group's tiles of the unit: positions it0 + t - x.t0 = cg (mod kGroups)
    const int it0 = it;
    static_assert((kGroups & (kGroups - 1)) == 0, "kGroups is a power of two");
    for (int t = x.t0 + ((cg - it0) & (kGroups - 1)); t < x.t1; t += kGroups) {
      const int s = cg + kGroups * gslot;  // = position % kStages
      const uint32_t parity = gphase;
      if (++gslot == kStages / kGroups) {
        gslot = 0;
        gphase ^= 1;
      }
      // Another role's abort shows here as a stage that never fills: the
      // bounded wait below then ends this warp's work too.
      if (aborted) continue;
      if (!mbar_wait(&sm.full[s], parity)) {
        record_error(p.err, kDeviceErrWaitTimeout);
        sm.abort_flag = 1;
        aborted = true;
        continue;
      }
      bool v_lo, v_hi;
      if constexpr (TT <= 32) {  // the stage's tokens fit the mask's low word
        const uint32_t mask = static_cast<uint32_t>(sm.mask[s]);
        v_lo = (mask >> row_tok(g)) & 1u;
        v_hi = (mask >> row_tok(g + 8)) & 1u;
      } else {
        const uint64_t mask = sm.mask[s];
        v_lo = (mask >> row_tok(g)) & 1ull;
        v_hi = (mask >> row_tok(g + 8)) & 1ull;
      }
      const uint32_t sbase = stage0 + static_cast<uint32_t>(s) * kStageBytes;
      // Pull this warp's K and V fragments into registers and hand the stage
      // back to the producer at once: the stage is held only for the
      // shared-memory reads, not for the math, so it is refilled sooner.
      uint32_t ka[KS][4], va[KS][4];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) ldsm_x4(ka[ks], sbase + a_off + ks * 32);
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) ldsm_x4_trans(va[mt], sbase + v_off + mt * 32);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);
      // two independent accumulator chains (even / odd k-steps) halve the
      // dependent MMA latency of S^T
      float acc[NT][4], acc2[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = acc2[nt][i] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_bf16(acc[nt], ka[ks], qf[ks][nt][0], qf[ks][nt][1]);
          mma_bf16(acc2[nt], ka[ks + 1], qf[ks + 1][nt][0], qf[ks + 1][nt][1]);
        }
      }
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float pr[4];
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const float s_lo = v_lo ? (acc[nt][hc] + acc2[nt][hc]) * scale_log2 : kNegBig;
          const float s_hi = v_hi ? (acc[nt][2 + hc] + acc2[nt][2 + hc]) * scale_log2 : kNegBig;
          float tmax = fmaxf(s_lo, s_hi);
          tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
          tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
          tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
          const float m_new = fmaxf(m[nt][hc], tmax);
          const float alpha = fast_exp2(m[nt][hc] - m_new);
          m[nt][hc] = m_new;
          const float p_lo = v_lo ? fast_exp2(s_lo - m_new) : 0.f;
          const float p_hi = v_hi ? fast_exp2(s_hi - m_new) : 0.f;
          l[nt][hc] = l[nt][hc] * alpha + p_lo + p_hi;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            o[mt][nt][hc] *= alpha;
            o[mt][nt][2 + hc] *= alpha;
          }
          pr[hc] = p_lo;
          pr[2 + hc] = p_hi;
        }
        pb[nt][0] = movmatrix_trans(pack_bf16x2(pr[0], pr[1]));
        pb[nt][1] = movmatrix_trans(pack_bf16x2(pr[2], pr[3]));
      }
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16(o[mt][nt], va[mt], pb[nt][0], pb[nt][1]);
      }
    }
    it = it0 + (x.t1 - x.t0);

    // ---- unit end.  An aborted warp goes on with an empty state (l = 0,
    // O = 0), so its partial or its share of the fold carries no weight.
    aborted = __any_sync(0xffffffffu, aborted);
    if (aborted) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
          o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {  // l over the warp's 16 token rows
        l[nt][hc] += __shfl_xor_sync(0xffffffffu, l[nt][hc], 4);
        l[nt][hc] += __shfl_xor_sync(0xffffffffu, l[nt][hc], 8);
        l[nt][hc] += __shfl_xor_sync(0xffffffffu, l[nt][hc], 16);
      }
    if (x.split) {
      // ---- a piece of a split pair: this warp's normalised partial and its
      // base-2 LSE (the reference's split-K format), written straight from
      // registers with no fold and no barrier, in slot
      // (2 * cta + (first pair met ? 0 : 1)) * R + rank of the warp.
      const int slot =
          (2 * static_cast<int>(blockIdx.x) + (k == 0 ? 0 : 1)) * R + cg * SUB + sub;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const int hl = 8 * nt + 2 * t4 + hc;
          if (hl >= group) continue;
          const float lv = l[nt][hc];
          const float inv = lv > 0.f ? 1.f / fmaxf(lv, 1.0e-20f) : 0.f;
          const int64_t base = static_cast<int64_t>(slot) * hqp + head0 + hl;
          float* po = p.part_o + base * D;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            po[mt * 16 + g] = o[mt][nt][hc] * inv;
            po[mt * 16 + g + 8] = o[mt][nt][2 + hc] * inv;
          }
          if (g == 0) p.part_lse[base] = lv > 0.f ? m[nt][hc] + log2f(fmaxf(lv, 1.0e-20f)) : -INFINITY;
        }
      }
      continue;
    }
    // ---- a pair this CTA met whole: fold the softmax states of the R warps
    // sharing a KV head by halving.  Each head has its own shared-memory
    // region (32 D / HB floats: R / 2 exchange slots of (D / 16) float4 per
    // lane, later its GQA group's [head][dim] result) and its own named
    // barrier, so heads do not wait for each other.  Round 1: warp j >= R/2
    // stores its (O, m, l) in slot j - R/2 and warp j - R/2 folds it in;
    // later rounds: warp j in [half, 2 half) stores in its own slot j, the
    // one it read last round (no one else reads it), and warp j - half folds
    // it in.  All warps of a head meet every barrier.
    float* region = sm.comb + hh * (32 * D / HB);
    float4* slots4 = reinterpret_cast<float4*>(region);
    const int bar_id = 1 + hh, bar_n = R * 32;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      // region free: the head's warps are done with its previous contents
      named_barrier(bar_id, bar_n);
#pragma unroll
      for (int half = R / 2; half >= 1; half >>= 1) {
        if (j >= half && j < 2 * half) {
          const int slot = half == R / 2 ? j - half : j;
          const int cs = hh * (R / 2) + slot;  // the pair's m/l slot
          __syncwarp();
#pragma unroll
          for (int mt = 0; mt < KS; ++mt)
            slots4[(slot * KS + mt) * 32 + lane] =
                make_float4(o[mt][nt][0], o[mt][nt][1], o[mt][nt][2], o[mt][nt][3]);
          if (g == 0) {
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              sm.cm[cs][2 * t4 + hc] = m[nt][hc];
              sm.cl[cs][2 * t4 + hc] = l[nt][hc];
            }
          }
        }
        named_barrier(bar_id, bar_n);
        if (j < half) {
          const int slot = half == R / 2 ? j : j + half;
          const int cs = hh * (R / 2) + slot;
          float sa[2], sb[2];
#pragma unroll
          for (int hc = 0; hc < 2; ++hc) {
            const float m2 = sm.cm[cs][2 * t4 + hc];
            const float mx = fmaxf(m[nt][hc], m2);
            sa[hc] = fast_exp2(m[nt][hc] - mx);
            sb[hc] = fast_exp2(m2 - mx);
            l[nt][hc] = l[nt][hc] * sa[hc] + sm.cl[cs][2 * t4 + hc] * sb[hc];
            m[nt][hc] = mx;
          }
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            const float4 t = slots4[(slot * KS + mt) * 32 + lane];
            o[mt][nt][0] = o[mt][nt][0] * sa[0] + t.x * sb[0];
            o[mt][nt][1] = o[mt][nt][1] * sa[1] + t.y * sb[1];
            o[mt][nt][2] = o[mt][nt][2] * sa[0] + t.z * sb[0];
            o[mt][nt][3] = o[mt][nt][3] * sa[1] + t.w * sb[1];
          }
        }
      }
    }
    // ---- the pair's result (this CTA met it whole), staged in the head's
    // region as [q head][dim] fp32 (8-float chunks XOR-swizzled by head:
    // conflict-free fragment stores, 16-byte reads), then stored as bf16
    // output with the gate (ops/qsa.py:250-275).
    named_barrier(bar_id, bar_n);
    if (j == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const int hl = 8 * nt + 2 * t4 + hc;
          if (hl >= group) continue;
          const float lv = l[nt][hc];
          const float inv = lv > 0.f ? 1.f / fmaxf(lv, 1.0e-20f) : 0.f;
          float* srow = region + hl * D;
          const int sw = (hl >> 1) & 3;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            srow[(((2 * mt) ^ sw) << 3) + g] = o[mt][nt][hc] * inv;
            srow[(((2 * mt + 1) ^ sw) << 3) + g] = o[mt][nt][2 + hc] * inv;
          }
        }
      }
    }
    named_barrier(bar_id, bar_n);
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int item = tr + i * R * 32;
      if (item >= group * (D / 8)) continue;
      const int hl = item / (D / 8), c = item % (D / 8);
      const float4* src =
          reinterpret_cast<const float4*>(region + hl * D + ((c ^ ((hl >> 1) & 3)) << 3));
      store_out8(p, x.row, x.hg * hqp + head0 + hl, c * 8, src[0], src[1], gpre[i]);
    }
  }
}

template <int D, int NT, int HB>
__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<D, NT, HB>& sm = *reinterpret_cast<Smem<D, NT, HB>*>(smem_raw);
  const int groups = p.kv_heads / HB;
  const int64_t ua = sk_begin(p, blockIdx.x), ub = sk_begin(p, blockIdx.x + 1);
  const int units = units_met(p, ua, ub);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 32);
      mbar_init(&sm.empty[s], kGroupWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.qfull[b], 1);
      mbar_init(&sm.qempty[b], kConsumerWarps);
    }
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x >= kConsumerWarps * 32)
    producer<D, NT, HB>(p, sm, units, groups, ua, ub);
  else
    consumer<D, NT, HB>(p, sm, units, groups, ua, ub);
}

// Merge of the split pairs: the reference's split-K merge (ops/qsa.py:306-362)
// over the pieces of each pair that a range boundary cuts.  Block column x
// takes the pair that CTA b = split.cta[x]'s range ends in (b holds the pair's
// first tile and a later CTA its last), so each split pair has one block
// column (grid.y blocks cover its heads).  Each CTA o1..o2 meeting the pair
// left R = 8 / heads_per_unit per-warp partials in its slot group:
// 2*o1 + 1 (2*o1 when o1's range starts at the pair), then 2*c for the later
// CTAs, for which it is the first pair met; partial slot = group * R + warp.
// Weights 2^(lse - max lse); bf16 rounding and the optional sigmoid gate
// follow.  A block of 8 warps serves 8 / W heads of the pair, W warps per
// head (from the plan's most partials of a split pair, so that each warp
// loads one batch of 8 in the common case); a lane holds 4 dims.  The W
// states of a head are combined in shared memory.
constexpr int kMergeThreads = 256;
constexpr int kMergeBatch = 8;  // partials a warp loads before using any
template <int D, int W>
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(const AttnParams p,
                                                              const SplitList split) {
  constexpr int kHeads = 8 / W;  // heads per block
  __shared__ float4 st_o[W > 1 ? 8 : 1][32];
  __shared__ float st_m[8], st_d[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hl = warp / W, w = warp % W;
  const int b = split.cta[blockIdx.x];
  const int64_t T = p.pair_tiles;
  const int64_t pair = (sk_begin(p, b + 1) - 1) / T;
  const int64_t first = pair * T;
  const int o1 = b, o2 = sk_owner(p, first + T - 1);
  const int group = p.q_heads / p.kv_heads;
  const int hqp = p.heads_per_unit * group;
  const int h = static_cast<int>(blockIdx.y) * kHeads + hl;  // head within the pair
  const bool live = h < hqp && lane < D / 4;
  const int groups = p.kv_heads / p.heads_per_unit;
  const int row = static_cast<int>(pair / groups), hg = static_cast<int>(pair % groups);
  const int d0 = lane * 4;
  // the gate is a step input the attention kernel does not write: its loads
  // go out before waiting on that kernel
  float gv[4] = {0.f, 0.f, 0.f, 0.f};
  if (live && w == 0 && p.gate != nullptr) {
    const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(p.gate) +
                              static_cast<int64_t>(row) * p.gate_row_stride +
                              static_cast<int64_t>(hg * hqp + h) * p.gate_head_stride;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      gv[i] = __bfloat162float(gp[static_cast<int64_t>(d0 + i) * p.gate_dim_stride]);
  }
  pdl_wait();
  pdl_trigger();
  const int R = 8 / p.heads_per_unit;  // partials per piece
  const int P = (o2 - o1 + 1) * R;     // partials of the pair
  const int e1 = sk_begin(p, o1) == first ? 0 : 1;
  float M = -INFINITY, den = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i0 = kMergeBatch * w; live && i0 < P; i0 += kMergeBatch * W) {
    float lse[kMergeBatch];
    float4 v[kMergeBatch];
#pragma unroll
    for (int jj = 0; jj < kMergeBatch; ++jj) {
      const int i = i0 + jj, piece = i / R;
      const int64_t grp = piece == 0 ? 2 * o1 + e1 : 2 * static_cast<int64_t>(o1 + piece);
      const int64_t base = i < P ? (grp * R + i % R) * hqp + h : 0;
      lse[jj] = i < P ? __ldg(p.part_lse + base) : -INFINITY;
      v[jj] = i < P ? __ldg(reinterpret_cast<const float4*>(p.part_o + base * D + d0))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m_new = M;
#pragma unroll
    for (int jj = 0; jj < kMergeBatch; ++jj) m_new = fmaxf(m_new, lse[jj]);
    if (m_new == -INFINITY) continue;  // no valid piece yet
    const float r = M == -INFINITY ? 0.f : exp2f(M - m_new);
    den *= r;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[c] *= r;
    M = m_new;
#pragma unroll
    for (int jj = 0; jj < kMergeBatch; ++jj) {
      const float wt = exp2f(lse[jj] - M);  // 0 for empty pieces
      den += wt;
      acc[0] += v[jj].x * wt;
      acc[1] += v[jj].y * wt;
      acc[2] += v[jj].z * wt;
      acc[3] += v[jj].w * wt;
    }
  }
  if constexpr (W > 1) {
    st_o[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    if (lane == 0) {
      st_m[warp] = M;
      st_d[warp] = den;
    }
    __syncthreads();
    if (w == 0) {
      float Mt = -INFINITY;
#pragma unroll
      for (int k = 0; k < W; ++k) Mt = fmaxf(Mt, st_m[warp + k]);
      den = 0.f;
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      if (Mt != -INFINITY) {
#pragma unroll
        for (int k = 0; k < W; ++k) {
          const float mk = st_m[warp + k];
          const float sc = mk == -INFINITY ? 0.f : exp2f(mk - Mt);
          const float4 t = st_o[warp + k][lane];
          den += st_d[warp + k] * sc;
          acc[0] += t.x * sc;
          acc[1] += t.y * sc;
          acc[2] += t.z * sc;
          acc[3] += t.w * sc;
        }
      }
    }
  }
  if (!live || w != 0) return;
  const float inv = den > 0.f ? 1.f / den : 0.f;
  float o[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    o[c] = acc[c] * inv;
    if (p.gate != nullptr)
      o[c] = __bfloat162float(__float2bfloat16_rn(o[c])) * sigmoid(gv[c]);
  }
  uint32_t* op = reinterpret_cast<uint32_t*>(
      static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.out_row_stride +
      static_cast<int64_t>(hg * hqp + h) * p.out_head_stride + d0);
  op[0] = pack_bf16x2(o[0], o[1]);
  op[1] = pack_bf16x2(o[2], o[3]);
}

// W warps per head: enough batches of kMergeBatch partials for the plan's
// most partials of a split pair (pieces x R), at most 8.
template <int D>
cudaError_t launch_merge(const AttnParams& p, const SplitList& split, cudaStream_t stream) {
  const int batches =
      (p.merge_pieces * (8 / p.heads_per_unit) + kMergeBatch - 1) / kMergeBatch;
  const int W = batches <= 1 ? 1 : batches <= 2 ? 2 : batches <= 4 ? 4 : 8;
  const int hqp = p.heads_per_unit * (p.q_heads / p.kv_heads);
  const int heads_per_block = 8 / W;
  const dim3 grid(split.n, (hqp + heads_per_block - 1) / heads_per_block);
  const dim3 block(kMergeThreads);
  switch (W) {
    case 1: return count_launches(launch_kernel(merge_kernel<D, 1>, grid, block, 0, stream, 1, p, split));
    case 2: return count_launches(launch_kernel(merge_kernel<D, 2>, grid, block, 0, stream, 1, p, split));
    case 4: return count_launches(launch_kernel(merge_kernel<D, 4>, grid, block, 0, stream, 1, p, split));
    default: return count_launches(launch_kernel(merge_kernel<D, 8>, grid, block, 0, stream, 1, p, split));
  }
}

template <int D, int NT, int HB>
cudaError_t launch_dnh(const AttnParams& p, const SplitList& split, cudaStream_t stream) {
  static_assert(sizeof(Smem<D, NT, HB>) <= 227 * 1024, "shared memory above the opt-in limit");
  static_assert(HB * 8 * NT <= 32, "a pair's heads exceed the unit-end buffer");
  const size_t smem = sizeof(Smem<D, NT, HB>);
  cudaError_t e = set_attr_once(reinterpret_cast<const void*>(attention_kernel<D, NT, HB>),
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int grid = p.sk_ctas;
  record_attention_event(0, stream);
  e = count_launches(
      launch_kernel(attention_kernel<D, NT, HB>, dim3(grid), dim3(kThreads), smem, stream, 1, p));
  if (e != cudaSuccess) return e;
  record_attention_event(1, stream);
  if (p.partials == 0) return cudaSuccess;  // no pair is split
  return launch_merge<D>(p, split, stream);
}

template <int D, int NT>
cudaError_t launch_dn(const AttnParams& p, const SplitList& split, int hb, cudaStream_t stream) {
  switch (hb) {
    case 4:
      if constexpr (NT == 1) return launch_dnh<D, NT, 4>(p, split, stream);
      break;
    case 2:
      if constexpr (NT == 1) return launch_dnh<D, NT, 2>(p, split, stream);
      break;
    case 1: return launch_dnh<D, NT, 1>(p, split, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

// KV heads handled together by one unit: the largest of 4, 2, 1 dividing the
// KV head count (1 for GQA groups above 8: a pair then holds at most 16
// query heads, and the unit-end buffers fit shared memory).
int attention_heads_per_unit(int q_heads, int kv_heads) {
  const int group = q_heads / kv_heads;
  const int cap = group <= 8 ? 4 : 1;
  for (int hb = cap; hb > 1; hb >>= 1)
    if (kv_heads % hb == 0) return hb;
  return 1;
}

// Stream-K plan: U = pairs x pair_tiles units cut into one contiguous range
// per CTA (one CTA per SM, or one per unit when there are fewer).  A pair is
// split where a range boundary falls inside it; when any is, the workspace
// holds two slot groups per CTA (the first and the last pair its range
// meets), each one partial per consumer warp sharing a KV head (R = 8 / HB),
// [heads of a pair, dim] fp32 plus [heads of a pair] LSE: its size depends
// on the CTA count and the pair's heads, not on the rows.  The same integer
// arithmetic as the kernels.
AttnPlan plan_attention(int rows, int q_heads, int kv_heads, int dim, int topk_width,
                        int use_decode_kernel) {
  (void)use_decode_kernel;
  AttnPlan plan{};
  const int hb = attention_heads_per_unit(q_heads, kv_heads);
  const int tt = 64 / hb;
  const int64_t pairs = static_cast<int64_t>(rows) * (kv_heads / hb);
  plan.heads_per_unit = hb;
  plan.pair_tiles = std::max(1, (topk_width + tt - 1) / tt);
  plan.units = pairs * plan.pair_tiles;
  plan.ctas = static_cast<int>(std::min<int64_t>(plan.units, std::min(num_sms(), kMaxSplit + 1)));
  if (plan.units <= 0) return plan;
  const int64_t U = plan.units, C = plan.ctas, T = plan.pair_tiles;
  auto owner = [&](int64_t x) { return ((x + 1) * C + U - 1) / U - 1; };
  // most CTAs meeting one split pair: pair of each range's last unit, when
  // the range holds the pair's first unit and not its last
  for (int64_t c = 0; c < C; ++c) {
    const int64_t first = ((U * (c + 1) / C) - 1) / T * T;
    const int64_t o1 = owner(first), o2 = owner(first + T - 1);
    if (o1 == c && o2 > c) {
      plan.merge_pieces = std::max<int>(plan.merge_pieces, static_cast<int>(o2 - c + 1));
      plan.split.cta[plan.split.n++] = static_cast<int16_t>(c);
    }
  }
  if (plan.merge_pieces == 0) return plan;
  plan.partials = 2 * (8 / hb);  // slot groups per CTA x partials per group
  const size_t hqp = static_cast<size_t>(hb) * (q_heads / kv_heads);
  const size_t slots = static_cast<size_t>(plan.partials) * plan.ctas;
  const size_t o_bytes = slots * hqp * dim * sizeof(float);
  plan.lse_offset = (o_bytes + 255) & ~static_cast<size_t>(255);
  plan.workspace_bytes = plan.lse_offset + slots * hqp * sizeof(float);
  return plan;
}

cudaError_t launch_attention(const AttnParams& p, const SplitList& split, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  const int group = p.q_heads / p.kv_heads;
  const int nt = group <= 8 ? 1 : 2;
  const int hb = attention_heads_per_unit(p.q_heads, p.kv_heads);
  if (p.dim == 128) return nt == 1 ? launch_dn<128, 1>(p, split, hb, stream) : launch_dn<128, 2>(p, split, hb, stream);
  if (p.dim == 64) return nt == 1 ? launch_dn<64, 1>(p, split, hb, stream) : launch_dn<64, 2>(p, split, hb, stream);
  return cudaErrorInvalidValue;
}

}  // namespace qsa
