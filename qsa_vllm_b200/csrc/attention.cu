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
//  * Persistent CTAs (one per SM) deal out (row, kv-head group, split) units.
//    A unit covers HB = up to 4 KV heads of one row: a selected token's K||V
//    rows of those heads are one contiguous run (2 KB at head_dim 128), moved
//    by ONE bulk copy (cp.async.bulk on the TMA engine) into a 4-stage
//    shared-memory ring guarded by mbarriers.  Token rows are padded by 16 B
//    so ldmatrix reads are bank-conflict free.  Invalid tokens are zero-filled.
//  * One producer warp issues the copies.  The token ids it needs are
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
//  * Per-warp softmax states are merged in shared memory at the end of a
//    unit; with more than one split, fp32 partials + LSE go to the caller's
//    workspace and a small merge kernel finishes (the reference's layout).
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

constexpr int kStages = 4;
constexpr int kGroups = 2;                        // consumer groups take alternate stages
constexpr int kGroupWarps = 4;                    // warps per group: one (head, sub-tile) each
constexpr int kConsumerWarps = kGroups * kGroupWarps;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kRing = 8;       // token-id ring slots (one per tile)
constexpr int kLookahead = 4;  // tiles of token ids in flight ahead of the copies
constexpr float kNegBig = -1.0e20f;

template <int D, int NT, int HB>
struct Smem {
  static constexpr int kTT = 64 / HB;           // tokens per stage
  static constexpr int kRow = HB * 4 * D + 16;  // K||V of HB heads + pad (bytes)
  static constexpr int kQRows = HB * 8 * NT;    // staged query head rows per unit
  alignas(128) uint8_t stage[kStages][kTT * kRow];
  alignas(128) uint8_t q[2][kQRows * 2 * D];
  float o_w[kConsumerWarps][8 * NT][D + 4];
  float m_w[kConsumerWarps][8 * NT];
  float l_w[kConsumerWarps][8 * NT];
  int32_t ring[kRing][64];
  uint64_t mask[kStages];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t qfull[2];
  uint64_t qempty[2];
  int abort_flag;
};

struct Unit {
  int row, hg, split, t0, t1, n_cols;
};

template <int TT>
__device__ __forceinline__ Unit decode_unit(const AttnParams& p, int u, int groups) {
  Unit x;
  x.split = u % p.splits;
  const int rest = u / p.splits;
  x.hg = rest % groups;
  x.row = rest / groups;
  int n = p.topk_width;
  if (p.valid_counts != nullptr) n = min(max(p.valid_counts[x.row], 0), p.topk_width);
  x.n_cols = n;
  const int tiles = (n + TT - 1) / TT;
  x.t0 = x.split * tiles / p.splits;
  x.t1 = (x.split + 1) * tiles / p.splits;
  return x;
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}

// Iterator over this CTA's (unit, tile) positions: the producer uses one to
// prefetch token ids ahead of the copies.
template <int TT>
struct Cursor {
  int u, t, units, groups;
  Unit x;
  bool live;
  __device__ void init(const AttnParams& p, int units_, int groups_) {
    units = units_;
    groups = groups_;
    u = blockIdx.x;
    live = u < units;
    if (live) {
      x = decode_unit<TT>(p, u, groups);
      t = x.t0;
      skip(p);
    }
  }
  __device__ void skip(const AttnParams& p) {
    while (live && t >= x.t1) {
      u += gridDim.x;
      live = u < units;
      if (live) {
        x = decode_unit<TT>(p, u, groups);
        t = x.t0;
      }
    }
  }
  __device__ void next(const AttnParams& p) {
    ++t;
    skip(p);
  }
};

template <int D, int NT, int HB>
__device__ void producer(const AttnParams& p, Smem<D, NT, HB>& sm, int units, int groups) {
  using S = Smem<D, NT, HB>;
  constexpr int TT = S::kTT;
  constexpr int kRow = S::kRow;
  const int lane = threadIdx.x & 31;
  const int group = p.q_heads / p.kv_heads;
  const uint8_t* kbase = static_cast<const uint8_t*>(p.k_cache);
  const uint8_t* vbase = static_cast<const uint8_t*>(p.v_cache);
  const uint8_t* qbase = static_cast<const uint8_t*>(p.q);

  Cursor<TT> ahead;
  ahead.init(p, units, groups);
  auto prefetch = [&](int slot) {
    if (ahead.live) {
      const int32_t* idx_row = p.indices + static_cast<int64_t>(ahead.x.row) * p.indices_row_stride;
      for (int j = lane; j < TT; j += 32) {
        const int col = ahead.t * TT + j;
        const bool v = col < ahead.x.n_cols;
        cp_async4(&sm.ring[slot][j], v ? idx_row + col : idx_row, v);
      }
      ahead.next(p);
    }
    cp_async_commit();
  };
#pragma unroll 1
  for (int i = 0; i < kLookahead; ++i) prefetch(i % kRing);

  int it = 0, k = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++k) {
    const Unit x = decode_unit<TT>(p, u, groups);
    // ---- the unit's query rows -> q[k & 1]
    const int qb = k & 1;
    if (k >= 2 && !mbar_wait(&sm.qempty[qb], ((k >> 1) - 1) & 1)) {
      record_error(p.err, kDeviceErrWaitTimeout);
      sm.abort_flag = 1;
      ok = false;
      break;
    }
    const int nq = HB * group;  // query head rows of this unit
    const uint8_t* qsrc = qbase + 2 * (static_cast<int64_t>(x.row) * p.q_row_stride +
                                       static_cast<int64_t>(x.hg * HB * group) * p.q_head_stride);
    if (lane == 0) {
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
    for (int t = x.t0; t < x.t1; ++t, ++it) {
      const int s = it % kStages;
      if (it >= kStages && !mbar_wait(&sm.empty[s], ((it / kStages) - 1) & 1)) {
        record_error(p.err, kDeviceErrWaitTimeout);
        sm.abort_flag = 1;
        ok = false;
        break;
      }
      if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) {
        ok = false;
        break;
      }
      // token ids of this tile: this lane's own cp.async writes (same lane
      // mapping as the prefetch), complete once all but the newest
      // kLookahead-1 groups are.
      cp_async_wait<kLookahead - 1>();
      // generic-proxy zero fills of an earlier use of this stage are ordered
      // before the async-proxy (bulk copy) writes issued below
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      uint8_t* stage = sm.stage[s];
      const int slot = it % kRing;
      int64_t off_k[2], off_v[2];
      bool valid[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = lane + 32 * h;
        const int col = t * TT + j;
        bool v = false;
        int page = 0, off = 0;
        if (j < TT && col < x.n_cols) {
          const int tok = sm.ring[slot][j];
          int lp;
          p.page_div.divmod(max(tok, 0), lp, off);
          if (p.physical) {
            page = lp;
            v = tok >= 0 && page < p.num_blocks;
          } else {
            v = req_ok && tok >= 0 && lp < p.table_width;
            page = v ? trow[lp] : -1;
            v = v && page >= 0 && page < p.num_blocks;
          }
        }
        valid[h] = v;
        off_k[h] = static_cast<int64_t>(page) * p.k_block_stride +
                   static_cast<int64_t>(off) * p.k_token_stride + head0 * p.k_head_stride;
        off_v[h] = static_cast<int64_t>(page) * p.v_block_stride +
                   static_cast<int64_t>(off) * p.v_token_stride + head0 * p.v_head_stride;
        if (!v && j < TT) {  // masked token: zeros, as the reference's masked loads
          uint4* z = reinterpret_cast<uint4*>(stage + j * kRow);
#pragma unroll 4
          for (int c = 0; c < (HB * 4 * D) / 16; ++c) z[c] = make_uint4(0, 0, 0, 0);
        }
      }
      const unsigned lo = __ballot_sync(0xffffffffu, valid[0]);
      const unsigned hi = __ballot_sync(0xffffffffu, valid[1]);
      if (lane == 0) {
        sm.mask[s] = static_cast<uint64_t>(lo) | (static_cast<uint64_t>(hi) << 32);
        mbar_expect_tx(&sm.full[s],
                       static_cast<uint32_t>(__popc(lo) + __popc(hi)) * (HB * 4u * D));
      }
      __syncwarp();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!valid[h]) continue;
        uint8_t* dst = stage + (lane + 32 * h) * kRow;
        if (p.kv_fused == 2) {  // all HB heads' K||V rows contiguous
          bulk_g2s(dst, kbase + 2 * off_k[h], HB * 4u * D, &sm.full[s]);
        } else {
#pragma unroll 1
          for (int hh = 0; hh < HB; ++hh) {
            if (p.kv_fused == 1) {
              bulk_g2s(dst + hh * 4 * D, kbase + 2 * (off_k[h] + hh * p.k_head_stride), 4u * D,
                       &sm.full[s]);
            } else {
              bulk_g2s(dst + hh * 4 * D, kbase + 2 * (off_k[h] + hh * p.k_head_stride), 2u * D,
                       &sm.full[s]);
              bulk_g2s(dst + hh * 4 * D + 2 * D, vbase + 2 * (off_v[h] + hh * p.v_head_stride),
                       2u * D, &sm.full[s]);
            }
          }
        }
      }
      mbar_arrive(&sm.full[s]);
      prefetch((it + kLookahead) % kRing);
    }
  }
  // Drain: never leave while a copy into this CTA's shared memory may be in
  // flight.  Wait (bounded) for the last issued phase of every barrier.
  cp_async_wait<0>();
  for (int j = std::max(0, it - kStages); j < it; ++j) {
    if (!mbar_wait(&sm.full[j % kStages], (j / kStages) & 1))
      record_error(p.err, kDeviceErrWaitTimeout);
  }
  for (int j = std::max(0, k - 2); j < k; ++j) {
    if (!mbar_wait(&sm.qfull[j & 1], (j >> 1) & 1)) record_error(p.err, kDeviceErrWaitTimeout);
  }
}

template <int D, int NT, int HB>
__device__ void consumer(const AttnParams& p, Smem<D, NT, HB>& sm, int units, int groups) {
  using S = Smem<D, NT, HB>;
  constexpr int TT = S::kTT;
  constexpr int kRow = S::kRow;
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
  constexpr uint32_t kStageBytes = TT * kRow;
  //   K (A operand of S^T, non-transposed): row = token, 16-byte chunk = dim/8
  const uint32_t a_off = static_cast<uint32_t>((sub * 16 + (lane & 15)) * kRow + hh * 4 * D +
                                               (lane >> 4) * 16);
  //   V (A operand of O^T, transposed): {tok0-7,d0-7},{tok0-7,d8-15},{tok8-15,d0-7},{tok8-15,d8-15}
  const int mi = lane >> 3;
  const uint32_t v_off = static_cast<uint32_t>(
      (sub * 16 + (lane & 7) + ((mi >> 1) << 3)) * kRow + hh * 4 * D + 2 * D + (mi & 1) * 16);

  int it = 0, k = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++k) {
    const Unit x = decode_unit<TT>(p, u, groups);
    const int qb = k & 1;
    if (!mbar_wait(&sm.qfull[qb], (k >> 1) & 1)) {
      record_error(p.err, kDeviceErrWaitTimeout);
      sm.abort_flag = 1;
      break;
    }
    // Q^T fragments (B operand of S^T): b0 = Q[head g][dims 2t4..], b1 = +8 dims.
    uint32_t qf[KS][NT][2];
    const uint8_t* qs = sm.q[qb];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
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
    if (lane == 0) mbar_arrive(&sm.qempty[qb]);

    float m[NT][2], l[NT][2];
    float o[KS][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = kNegBig;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
    }

    for (int t = x.t0; t < x.t1; ++t, ++it) {
      if ((it % kGroups) != cg) continue;  // the other group's stage
      const int s = it % kStages;
      if (!mbar_wait(&sm.full[s], (it / kStages) & 1)) {
        record_error(p.err, kDeviceErrWaitTimeout);
        sm.abort_flag = 1;
        ok = false;
        break;
      }
      const uint64_t mask = sm.mask[s];
      const bool v_lo = (mask >> (sub * 16 + g)) & 1ull;
      const bool v_hi = (mask >> (sub * 16 + g + 8)) & 1ull;
      const uint32_t sbase = stage0 + static_cast<uint32_t>(s) * kStageBytes;
      // two independent accumulator chains (even / odd k-steps) halve the
      // dependent MMA latency of S^T
      float acc[NT][4], acc2[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = acc2[nt][i] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
        uint32_t a[4], a2[4];
        ldsm_x4(a, sbase + a_off + ks * 32);
        ldsm_x4(a2, sbase + a_off + (ks + 1) * 32);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_bf16(acc[nt], a, qf[ks][nt][0], qf[ks][nt][1]);
          mma_bf16(acc2[nt], a2, qf[ks + 1][nt][0], qf[ks + 1][nt][1]);
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
        uint32_t a[4];
        ldsm_x4_trans(a, sbase + v_off + mt * 32);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16(o[mt][nt], a, pb[nt][0], pb[nt][1]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);
    }
    if (!ok) break;
    if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) break;

    // ---- merge the warps holding each head (sub-tiles x groups), finish.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        float lv = l[nt][hc];
        lv += __shfl_xor_sync(0xffffffffu, lv, 4);
        lv += __shfl_xor_sync(0xffffffffu, lv, 8);
        lv += __shfl_xor_sync(0xffffffffu, lv, 16);
        const int hl = 8 * nt + 2 * t4 + hc;
        if (g == 0) {
          sm.m_w[warp][hl] = m[nt][hc];
          sm.l_w[warp][hl] = lv;
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          sm.o_w[warp][hl][mt * 16 + g] = o[mt][nt][hc];
          sm.o_w[warp][hl][mt * 16 + g + 8] = o[mt][nt][2 + hc];
        }
      }
    }
    named_barrier(1, kConsumerWarps * 32);
    const int per_head = group * (D / 2);
    for (int e = threadIdx.x; e < HB * per_head; e += kConsumerWarps * 32) {
      const int h2 = e / per_head;
      const int rem = e % per_head;
      const int hl = rem / (D / 2);
      const int d0 = (rem % (D / 2)) * 2;
      float M = kNegBig;
#pragma unroll
      for (int gi = 0; gi < kGroups; ++gi)
#pragma unroll
        for (int sb = 0; sb < SUB; ++sb)
          M = fmaxf(M, sm.m_w[gi * kGroupWarps + h2 + HB * sb][hl]);
      float L = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int gi = 0; gi < kGroups; ++gi) {
#pragma unroll
        for (int sb = 0; sb < SUB; ++sb) {
          const int w = gi * kGroupWarps + h2 + HB * sb;
          const float f = fast_exp2(sm.m_w[w][hl] - M);
          L += sm.l_w[w][hl] * f;
          o0 += sm.o_w[w][hl][d0] * f;
          o1 += sm.o_w[w][hl][d0 + 1] * f;
        }
      }
      const bool has = L > 0.f;
      const float inv = has ? 1.f / fmaxf(L, 1.0e-20f) : 0.f;
      o0 = has ? o0 * inv : 0.f;
      o1 = has ? o1 * inv : 0.f;
      const int head = (x.hg * HB + h2) * group + hl;
      if (p.splits == 1) {
        if (p.gate != nullptr) {
          const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(p.gate) +
                                    static_cast<int64_t>(x.row) * p.gate_row_stride +
                                    static_cast<int64_t>(head) * p.gate_head_stride;
          const float g0 = __bfloat162float(gp[static_cast<int64_t>(d0) * p.gate_dim_stride]);
          const float g1 = __bfloat162float(gp[static_cast<int64_t>(d0 + 1) * p.gate_dim_stride]);
          o0 = __bfloat162float(__float2bfloat16_rn(o0)) / (1.f + __expf(-g0));
          o1 = __bfloat162float(__float2bfloat16_rn(o1)) / (1.f + __expf(-g1));
        }
        __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.out) +
                            static_cast<int64_t>(x.row) * p.out_row_stride +
                            static_cast<int64_t>(head) * p.out_head_stride + d0;
        *reinterpret_cast<__nv_bfloat162*>(op) = __floats2bfloat162_rn(o0, o1);
      } else {
        const int64_t base = (static_cast<int64_t>(x.split) * p.rows + x.row) * p.q_heads + head;
        *reinterpret_cast<float2*>(p.part_o + base * D + d0) = make_float2(o0, o1);
        if (d0 == 0) p.part_lse[base] = has ? M + log2f(fmaxf(L, 1.0e-20f)) : -INFINITY;
      }
    }
    named_barrier(1, kConsumerWarps * 32);
  }
}

template <int D, int NT, int HB>
__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<D, NT, HB>& sm = *reinterpret_cast<Smem<D, NT, HB>*>(smem_raw);
  const int groups = p.kv_heads / HB;
  const int units = p.rows * groups * p.splits;
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
  if (threadIdx.x >= kConsumerWarps * 32)
    producer<D, NT, HB>(p, sm, units, groups);
  else
    consumer<D, NT, HB>(p, sm, units, groups);
}

// Split merge (ops/qsa.py:306-362): one block per (row, query head).
template <int D>
__global__ void __launch_bounds__(D / 2) merge_kernel(const AttnParams p) {
  const int row = blockIdx.x, head = blockIdx.y;
  const int d0 = threadIdx.x * 2;
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s)
    M = fmaxf(M, p.part_lse[(static_cast<int64_t>(s) * p.rows + row) * p.q_heads + head]);
  float den = 0.f, o0 = 0.f, o1 = 0.f;
  if (M > -INFINITY) {
    for (int s = 0; s < p.splits; ++s) {
      const int64_t base = (static_cast<int64_t>(s) * p.rows + row) * p.q_heads + head;
      const float w = exp2f(p.part_lse[base] - M);
      den += w;
      const float2 v = *reinterpret_cast<const float2*>(p.part_o + base * D + d0);
      o0 += v.x * w;
      o1 += v.y * w;
    }
  }
  o0 = den > 0.f ? o0 / den : 0.f;
  o1 = den > 0.f ? o1 / den : 0.f;
  if (p.gate != nullptr) {
    const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(p.gate) +
                              static_cast<int64_t>(row) * p.gate_row_stride +
                              static_cast<int64_t>(head) * p.gate_head_stride;
    const float g0 = __bfloat162float(gp[static_cast<int64_t>(d0) * p.gate_dim_stride]);
    const float g1 = __bfloat162float(gp[static_cast<int64_t>(d0 + 1) * p.gate_dim_stride]);
    o0 = __bfloat162float(__float2bfloat16_rn(o0)) / (1.f + __expf(-g0));
    o1 = __bfloat162float(__float2bfloat16_rn(o1)) / (1.f + __expf(-g1));
  }
  __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.out) +
                      static_cast<int64_t>(row) * p.out_row_stride +
                      static_cast<int64_t>(head) * p.out_head_stride + d0;
  *reinterpret_cast<__nv_bfloat162*>(op) = __floats2bfloat162_rn(o0, o1);
}

template <int D, int NT, int HB>
cudaError_t launch_dnh(const AttnParams& p, cudaStream_t stream) {
  const size_t smem = sizeof(Smem<D, NT, HB>);
  cudaError_t e = set_attr_once(reinterpret_cast<const void*>(attention_kernel<D, NT, HB>),
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int units = p.rows * (p.kv_heads / HB) * p.splits;
  const int grid = std::min(units, num_sms());
  attention_kernel<D, NT, HB><<<grid, kThreads, smem, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess || p.splits == 1) return e;
  merge_kernel<D><<<dim3(p.rows, p.q_heads), D / 2, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int D, int NT>
cudaError_t launch_dn(const AttnParams& p, int hb, cudaStream_t stream) {
  switch (hb) {
    case 4:
      if constexpr (NT == 1) return launch_dnh<D, NT, 4>(p, stream);
      break;
    case 2: return launch_dnh<D, NT, 2>(p, stream);
    case 1: return launch_dnh<D, NT, 1>(p, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

// KV heads handled together by one unit: the largest of 4, 2, 1 dividing the
// KV head count (at most 2 for GQA groups above 8, to fit shared memory).
int attention_heads_per_unit(int q_heads, int kv_heads) {
  const int group = q_heads / kv_heads;
  const int cap = group <= 8 ? 4 : 2;
  for (int hb = cap; hb > 1; hb >>= 1)
    if (kv_heads % hb == 0) return hb;
  return 1;
}

AttnPlan plan_attention(int rows, int q_heads, int kv_heads, int dim, int topk_width,
                        int use_decode_kernel) {
  (void)use_decode_kernel;
  AttnPlan plan{1, 0};
  const int hb = attention_heads_per_unit(q_heads, kv_heads);
  const int tt = 64 / hb;
  const int base = rows * (kv_heads / hb);
  const int tiles = (topk_width + tt - 1) / tt;
  const int G = num_sms();  // persistent grid: one CTA per SM, units dealt round-robin
  if (base <= 0 || tiles <= 1 || base >= 4 * G) return plan;
  // Simulate the round-robin deal for each split count and keep the one whose
  // busiest CTA walks the fewest tiles (a unit's start + epilogue ~ three
  // tiles; the merge launch ~ two tiles).
  int best = 1;
  double best_cost = 1e30;
  const int max_split = std::min(tiles, 32);
  for (int S = 1; S <= max_split; ++S) {
    const int units = base * S;
    double worst = 0.0;
    for (int c = 0; c < std::min(units, G); ++c) {
      double load = 0.0;
      for (int u = c; u < units; u += G) {
        const int sp = u % S;
        load += ((sp + 1) * tiles / S - sp * tiles / S) + 3.0;
      }
      worst = std::max(worst, load);
    }
    const double cost = worst + (S > 1 ? 2.0 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = S;
    }
  }
  plan.splits = best;
  if (best > 1) {
    const size_t o_bytes = static_cast<size_t>(best) * rows * q_heads * dim * sizeof(float);
    const size_t l_bytes = static_cast<size_t>(best) * rows * q_heads * sizeof(float);
    plan.workspace_bytes = ((o_bytes + 255) & ~static_cast<size_t>(255)) + l_bytes;
  }
  return plan;
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  const int group = p.q_heads / p.kv_heads;
  const int nt = group <= 8 ? 1 : 2;
  const int hb = attention_heads_per_unit(p.q_heads, p.kv_heads);
  if (p.dim == 128) return nt == 1 ? launch_dn<128, 1>(p, hb, stream) : launch_dn<128, 2>(p, hb, stream);
  if (p.dim == 64) return nt == 1 ? launch_dn<64, 1>(p, hb, stream) : launch_dn<64, 2>(p, hb, stream);
  return cudaErrorInvalidValue;
}

}  // namespace qsa
