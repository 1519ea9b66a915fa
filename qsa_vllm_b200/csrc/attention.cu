// Paged sparse GQA attention over selected tokens (sm_100a).
//
// Semantics follow the reference split-K kernel and merge (ops/qsa.py:109-303,
// :306-362): s = (q . k) * d^-0.5 in fp32 with base-2 online softmax, P rounded
// to bf16 before P.V with fp32 accumulation, out = acc / max(l, 1e-20) (0 when
// no token is valid), optional bf16 rounding then * sigmoid(gate).  Decode
// indices are physical slots bounded by the per-row valid count; prefill
// indices are logical tokens mapped through the request's block table.
//
// Design (B200): the work is HBM-bound (8 flop/byte), so the kernel is built
// around the gather.  Persistent CTAs walk (row, kv head, split) units.  One
// producer warp turns 64 selected tokens at a time into per-token bulk copies
// (cp.async.bulk, executed by the TMA engine) of the contiguous K||V row of
// that token and kv head (512 B at head_dim 128) into a 4-stage shared-memory
// ring guarded by mbarriers; invalid tokens are zero-filled.  Four consumer
// warps each take 16 tokens of a stage: S^T = K.Q^T on mma.sync with the
// tokens as the M dimension and the (up to 8 or 16) query heads of the GQA
// group as N, so no MMA lane is padding for group 8; the P^T fragments are
// transposed in registers (movmatrix) into the B operand of O^T = V^T.P^T.
// Rows of the ring are padded by 16 B so ldmatrix is bank-conflict free.
// Per-warp softmax states are merged through shared memory at the end of a
// unit; with more than one split, fp32 partials + LSE go to the caller's
// workspace and a small merge kernel finishes (the reference's layout).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

constexpr int kTileN = 64;
constexpr int kStages = 4;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr float kNegBig = -1.0e20f;

template <int D, int NT>
struct Smem {
  static constexpr int kRowBytes = 4 * D + 16;
  alignas(128) uint8_t stage[kStages][kTileN * kRowBytes];
  float o_w[kConsumerWarps][8 * NT][D + 4];
  float m_w[kConsumerWarps][8 * NT];
  float l_w[kConsumerWarps][8 * NT];
  uint64_t mask[kStages];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int abort_flag;
};

struct Unit {
  int row, kvh, split, t0, t1, n_cols;
};

__device__ __forceinline__ Unit decode_unit(const AttnParams& p, int u) {
  Unit x;
  x.split = u % p.splits;
  const int rest = u / p.splits;
  x.kvh = rest % p.kv_heads;
  x.row = rest / p.kv_heads;
  int n = p.topk_width;
  if (p.valid_counts != nullptr) n = min(max(p.valid_counts[x.row], 0), p.topk_width);
  x.n_cols = n;
  const int tiles = (n + kTileN - 1) / kTileN;
  x.t0 = x.split * tiles / p.splits;
  x.t1 = (x.split + 1) * tiles / p.splits;
  return x;
}

template <int D, int NT>
__device__ void producer(const AttnParams& p, Smem<D, NT>& sm, int units) {
  const int lane = threadIdx.x & 31;
  constexpr int kRow = Smem<D, NT>::kRowBytes;
  const uint32_t tok_bytes = 4u * D;  // K (2D bytes) + V (2D bytes)
  const uint8_t* kbase = static_cast<const uint8_t*>(p.k_cache);
  const uint8_t* vbase = static_cast<const uint8_t*>(p.v_cache);
  int it = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
    const Unit x = decode_unit(p, u);
    int req = 0;
    bool req_ok = true;
    if (!p.physical) {
      req = p.token_to_req[x.row];
      req_ok = req >= 0 && req < p.num_requests;
    }
    const int32_t* idx_row = p.indices + static_cast<int64_t>(x.row) * p.indices_row_stride;
    const int32_t* trow =
        p.block_table + static_cast<int64_t>(req_ok ? req : 0) * p.table_row_stride;
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
      // Generic-proxy zero fills of an earlier use of this stage must be
      // ordered before the async-proxy (bulk copy) writes issued below.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      uint8_t* stage = sm.stage[s];
      const uint8_t* ksrc[2];
      const uint8_t* vsrc[2];
      bool valid[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = lane + 32 * h;
        const int col = t * kTileN + j;
        bool v = false;
        int page = 0, off = 0;
        if (col < x.n_cols) {
          const int tok = idx_row[col];
          const int safe = max(tok, 0);
          const int lp = safe / p.page_size;
          off = safe % p.page_size;
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
        ksrc[h] = kbase + 2 * (static_cast<int64_t>(page) * p.k_block_stride +
                               static_cast<int64_t>(off) * p.k_token_stride +
                               static_cast<int64_t>(x.kvh) * p.k_head_stride);
        vsrc[h] = vbase + 2 * (static_cast<int64_t>(page) * p.v_block_stride +
                               static_cast<int64_t>(off) * p.v_token_stride +
                               static_cast<int64_t>(x.kvh) * p.v_head_stride);
        if (!v) {  // masked token: zeros, as the reference's masked loads (other=0.0)
          uint4* z = reinterpret_cast<uint4*>(stage + j * kRow);
#pragma unroll 4
          for (int c = 0; c < (4 * D) / 16; ++c) z[c] = make_uint4(0, 0, 0, 0);
        }
      }
      const unsigned lo = __ballot_sync(0xffffffffu, valid[0]);
      const unsigned hi = __ballot_sync(0xffffffffu, valid[1]);
      if (lane == 0) {
        sm.mask[s] = static_cast<uint64_t>(lo) | (static_cast<uint64_t>(hi) << 32);
        mbar_expect_tx(&sm.full[s], static_cast<uint32_t>(__popc(lo) + __popc(hi)) * tok_bytes);
      }
      __syncwarp();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!valid[h]) continue;
        uint8_t* dst = stage + (lane + 32 * h) * kRow;
        if (p.kv_fused) {
          bulk_g2s(dst, ksrc[h], tok_bytes, &sm.full[s]);
        } else {
          bulk_g2s(dst, ksrc[h], 2u * D, &sm.full[s]);
          bulk_g2s(dst + 2 * D, vsrc[h], 2u * D, &sm.full[s]);
        }
      }
      mbar_arrive(&sm.full[s]);
    }
  }
  // Drain: never leave while a bulk copy into this CTA's shared memory may be
  // in flight.  Wait (bounded) for the last issued phase of every stage.
  for (int k = std::max(0, it - kStages); k < it; ++k) {
    if (!mbar_wait(&sm.full[k % kStages], (k / kStages) & 1))
      record_error(p.err, kDeviceErrWaitTimeout);
  }
}

template <int D, int NT>
__device__ void consumer(const AttnParams& p, Smem<D, NT>& sm, int units) {
  constexpr int KS = D / 16;  // k-steps of S^T, m-tiles of O^T
  constexpr int kRow = Smem<D, NT>::kRowBytes;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int group = p.q_heads / p.kv_heads;
  const float scale_log2 = p.scale_log2;
  const __nv_bfloat16* qbase = static_cast<const __nv_bfloat16*>(p.q);
  const uint32_t stage0 = smem_u32(&sm.stage[0][0]);
  constexpr uint32_t kStageBytes = kTileN * kRow;
  // ldmatrix row addresses (byte offsets inside a stage) of this lane.
  //   K (A operand of S^T, non-transposed): row = token, 16-byte chunk = dim/8.
  const uint32_t a_row = static_cast<uint32_t>(warp * 16 + (lane & 15));
  const uint32_t a_off = a_row * kRow + static_cast<uint32_t>((lane >> 4) * 16);
  //   V (A operand of O^T, transposed): matrices {tok0-7,d0-7},{tok0-7,d8-15},{tok8-15,d0-7},{tok8-15,d8-15}
  const int mi = lane >> 3;
  const uint32_t v_row = static_cast<uint32_t>(warp * 16 + (lane & 7) + ((mi >> 1) << 3));
  const uint32_t v_off = v_row * kRow + 2 * D + static_cast<uint32_t>((mi & 1) * 16);

  int it = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const Unit x = decode_unit(p, u);
    // Q^T fragments (B operand of S^T): b0 = Q[head g][dims 2t4..], b1 = +8 dims.
    uint32_t qf[KS][NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int hl = g + 8 * nt;
      const bool hv = hl < group;
      const __nv_bfloat16* qrow = qbase + static_cast<int64_t>(x.row) * p.q_row_stride +
                                  static_cast<int64_t>(x.kvh * group + (hv ? hl : 0)) *
                                      p.q_head_stride;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[ks][nt][0] = hv ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t4) : 0u;
        qf[ks][nt][1] = hv ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t4) : 0u;
      }
    }
    float m[NT][2], l[NT][2];
    float o[KS][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = kNegBig;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
    }

    for (int t = x.t0; t < x.t1 && ok; ++t, ++it) {
      const int s = it % kStages;
      if (!mbar_wait(&sm.full[s], (it / kStages) & 1)) {
        record_error(p.err, kDeviceErrWaitTimeout);
        sm.abort_flag = 1;
        ok = false;
        break;
      }
      const uint64_t mask = sm.mask[s];
      const bool v_lo = (mask >> (warp * 16 + g)) & 1ull;
      const bool v_hi = (mask >> (warp * 16 + g + 8)) & 1ull;
      const uint32_t sbase = stage0 + static_cast<uint32_t>(s) * kStageBytes;
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, sbase + a_off + ks * 32);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16(acc[nt], a, qf[ks][nt][0], qf[ks][nt][1]);
      }
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float pr[4];
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const float s_lo = v_lo ? acc[nt][hc] * scale_log2 : kNegBig;
          const float s_hi = v_hi ? acc[nt][2 + hc] * scale_log2 : kNegBig;
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

    // ---- merge the four warps' softmax states of this unit.
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
    const int ctid = threadIdx.x;  // 0..127
    const int pairs = group * (D / 2);
    for (int e = ctid; e < pairs; e += kConsumerWarps * 32) {
      const int hl = e / (D / 2);
      const int d0 = (e % (D / 2)) * 2;
      float M = kNegBig;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.m_w[w][hl]);
      float L = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float f = fast_exp2(sm.m_w[w][hl] - M);
        L += sm.l_w[w][hl] * f;
        o0 += sm.o_w[w][hl][d0] * f;
        o1 += sm.o_w[w][hl][d0 + 1] * f;
      }
      const bool has = L > 0.f;
      const float inv = has ? 1.f / fmaxf(L, 1.0e-20f) : 0.f;
      o0 = has ? o0 * inv : 0.f;
      o1 = has ? o1 * inv : 0.f;
      const int head = x.kvh * group + hl;
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

template <int D, int NT>
__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<D, NT>& sm = *reinterpret_cast<Smem<D, NT>*>(smem_raw);
  const int units = p.rows * p.kv_heads * p.splits;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 32);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= kConsumerWarps * 32)
    producer<D, NT>(p, sm, units);
  else
    consumer<D, NT>(p, sm, units);
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

template <int D, int NT>
cudaError_t launch_dn(const AttnParams& p, cudaStream_t stream) {
  const size_t smem = sizeof(Smem<D, NT>);
  cudaError_t e = set_attr_once(reinterpret_cast<const void*>(attention_kernel<D, NT>), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int units = p.rows * p.kv_heads * p.splits;
  const int grid = std::min(units, num_sms());
  attention_kernel<D, NT><<<grid, kThreads, smem, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess || p.splits == 1) return e;
  merge_kernel<D><<<dim3(p.rows, p.q_heads), D / 2, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

AttnPlan plan_attention(int rows, int q_heads, int kv_heads, int dim, int topk_width,
                        int use_decode_kernel) {
  (void)use_decode_kernel;
  AttnPlan plan{1, 0};
  const int base = rows * kv_heads;
  const int tiles = (topk_width + kTileN - 1) / kTileN;
  const int G = num_sms();  // persistent grid: one CTA per SM, units dealt round-robin
  if (base <= 0 || tiles <= 1 || base >= 4 * G) return plan;
  // Simulate the round-robin deal for each split count and keep the one whose
  // busiest CTA walks the fewest tiles (a unit's epilogue ~ half a tile; the
  // merge launch ~ one tile).
  int best = 1;
  double best_cost = 1e30;
  const int max_split = std::min(tiles, 16);
  for (int S = 1; S <= max_split; ++S) {
    const int units = base * S;
    double worst = 0.0;
    for (int c = 0; c < std::min(units, G); ++c) {
      double load = 0.0;
      for (int u = c; u < units; u += G) {
        const int sp = u % S;
        load += ((sp + 1) * tiles / S - sp * tiles / S) + 0.5;
      }
      worst = std::max(worst, load);
    }
    const double cost = worst + (S > 1 ? 1.0 : 0.0);
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
  if (p.dim == 128) return nt == 1 ? launch_dn<128, 1>(p, stream) : launch_dn<128, 2>(p, stream);
  if (p.dim == 64) return nt == 1 ? launch_dn<64, 1>(p, stream) : launch_dn<64, 2>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace qsa
