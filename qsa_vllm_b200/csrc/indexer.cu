// Indexer scores: logits[r, c] = scale * sum_h w[r,h] * relu(q[r,h] . key(c)) (sm_100a).
//
// Semantics follow the reference scoring kernels (ops/indexer.py:24-114 uniform
// decode, :117-223 packed prefill): bf16 inputs, fp32 products, ReLU per head,
// head sum, times head_dim^-0.5; only columns below the row's visible count
// (and the page-table capacity) are written.
//
// This translation unit holds the warp-level MMA formulation (mma.sync), used
// for shapes the tcgen05 kernel does not take.  A CTA owns the query columns of
// one request (decode: its decode_query_len rows; prefill: up to 128/H rows of
// one request) and a contiguous chunk of that request's keys.  Keys are paged,
// so each 128/256-byte key row is fetched with 16-byte cp.async into a 4-stage
// ring whose 16-byte chunks are XOR-swizzled by row (conflict-free ldmatrix).
// S^T = K.Q^T runs with keys as M; the epilogue applies ReLU and the head
// weights in registers, reduces the heads of a row with warp shuffles and
// stores coalesced fp32 logits.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

constexpr int kKeyTile = 64;
constexpr int kStages = 4;
constexpr int kThreads = 128;
constexpr int kMaxKeysPerCta = 1024;
constexpr int kMaxPages = kMaxKeysPerCta + 2;  // page size 1 worst case

template <int D, int NT>
struct IdxSmem {
  static constexpr int kRowBytes = 2 * D;
  alignas(128) uint8_t k[kStages][kKeyTile * kRowBytes];
  alignas(128) uint8_t q[8 * NT * kRowBytes];
  float w[8 * NT];
  int limit[8 * NT];  // per row of the CTA: columns below this are stored
  int pages[kMaxPages];  // physical page of each logical page of this CTA's keys
};

// byte offset of 16-byte chunk `c` of row `r` in a swizzled tile
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * (2 * D) + ((c ^ (r & 7)) << 4));
}

template <int D, int NT>
__global__ void __launch_bounds__(kThreads) indexer_kernel(const IndexerParams p, int rows_per_cta,
                                                           int keys_per_cta) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  auto& sm = *reinterpret_cast<IdxSmem<D, NT>*>(smem_raw);
  constexpr int CPR = D / 8;  // 16-byte chunks per key row
  constexpr int N = 8 * NT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = p.heads;

  // ---- rows of this CTA (absolute packed rows) and their request.
  const int req = blockIdx.x;
  int r0, r1;
  if (p.query_start_loc == nullptr) {
    r0 = req * p.decode_query_len;
    r1 = r0 + p.decode_query_len;
  } else {
    const int base = p.query_start_loc[0];
    const int qend = p.query_offset + p.num_rows;
    const int rs = max(p.query_start_loc[req] - base, p.query_offset);
    const int re = min(p.query_start_loc[req + 1] - base, qend);
    r0 = rs + blockIdx.y * rows_per_cta;
    r1 = min(r0 + rows_per_cta, re);
  }
  if (r0 >= r1) return;
  const int nrows = r1 - r0;
  const int num_columns = p.table_width * p.page_size;
  const int cap = min(num_columns, p.logits_width);
  int maxvis = 0;
  for (int i = 0; i < nrows; ++i) maxvis = max(maxvis, min(row_visible(p, r0 + i), cap));
  const int k0 = blockIdx.z * keys_per_cta;
  const int k1 = min(k0 + keys_per_cta, maxvis);
  if (k0 >= k1) return;

  if (tid < N) {
    const int ri = tid / H, h = tid % H;
    const bool v = ri < nrows;
    sm.w[tid] = v ? (p.weights ? p.weights[static_cast<int64_t>(r0 + ri) * p.w_row_stride +
                                            static_cast<int64_t>(h) * p.w_head_stride]
                               : 1.f)
                  : 0.f;
    sm.limit[tid] = tid < nrows ? min(row_visible(p, r0 + tid), cap) : 0;
  }

  // ---- query tile: column n = (row n / H, head n % H)
  const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(p.q);
  for (int ch = tid; ch < N * CPR; ch += kThreads) {
    const int n = ch / CPR, c = ch % CPR;
    const int ri = n / H, h = n % H;
    const bool v = ri < nrows;
    const __nv_bfloat16* src = qb + static_cast<int64_t>(v ? r0 + ri : r0) * p.q_row_stride +
                               static_cast<int64_t>(v ? h : 0) * p.q_head_stride + c * 8;
    cp_async16(sm.q + swz<D>(n, c), src, v);
  }

  // ---- this CTA's slice of the page table, staged once in shared memory so
  // the key-tile loads below never wait on a dependent global lookup.
  const int32_t* trow = p.table + static_cast<int64_t>(req) * p.table_row_stride;
  const int pg0 = static_cast<int>(p.page_div.div(k0));
  const int npg = static_cast<int>(p.page_div.div(k1 - 1)) - pg0 + 1;
  for (int i = tid; i < npg; i += kThreads) sm.pages[i] = trow[pg0 + i];
  __syncthreads();
  const __nv_bfloat16* kb = static_cast<const __nv_bfloat16*>(p.k_cache);
  const int ntiles = (k1 - k0 + kKeyTile - 1) / kKeyTile;
  auto load_tile = [&](int t) {
    uint8_t* dst = sm.k[t % kStages];
    for (int ch = tid; ch < kKeyTile * CPR; ch += kThreads) {
      const int key = ch / CPR, c = ch % CPR;
      const int col = k0 + t * kKeyTile + key;
      bool v = col < k1;
      int page = 0, lp = 0, off = 0;
      if (v) {
        p.page_div.divmod(col, lp, off);
        page = sm.pages[lp - pg0];
        v = page >= 0 && page < p.num_blocks;
      }
      const __nv_bfloat16* src =
          kb + (v ? static_cast<int64_t>(page) * p.block_stride +
                        static_cast<int64_t>(off) * p.token_stride
                  : 0) +
          c * 8;
      cp_async16(dst + swz<D>(key, c), src, v);
    }
  };
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < ntiles) load_tile(s);
    cp_async_commit();
  }

  const int g = lane >> 2, t4 = lane & 3;
  const float scale = p.scale;
  const uint32_t q_base = smem_u32(sm.q);
  for (int t = 0; t < ntiles; ++t) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    if (t + kStages - 1 < ntiles) load_tile(t + kStages - 1);
    cp_async_commit();

    const uint32_t k_base = smem_u32(sm.k[t % kStages]);
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[4];
      const int arow = warp * 16 + (lane & 15);
      ldsm_x4(a, k_base + swz<D>(arow, 2 * ks + (lane >> 4)));
      if constexpr (NT == 1) {
        uint32_t b[2];
        ldsm_x2(b, q_base + swz<D>(lane & 7, 2 * ks + ((lane >> 3) & 1)));
        mma_bf16(acc[0], a, b[0], b[1]);
      } else {
#pragma unroll
        for (int nt = 0; nt < NT; nt += 2) {
          uint32_t b[4];
          const int qrow = 8 * nt + (lane & 7) + ((lane >> 4) << 3);
          ldsm_x4(b, q_base + swz<D>(qrow, 2 * ks + ((lane >> 3) & 1)));
          mma_bf16(acc[nt], a, b[0], b[1]);
          mma_bf16(acc[nt + 1], a, b[2], b[3]);
        }
      }
    }

    // ---- epilogue: relu * w, sum the H heads of each row, scale, store.
    const int key_lo = k0 + t * kKeyTile + warp * 16 + g;
    const int key_hi = key_lo + 8;
    auto store = [&](int ri, int key, float v) {
      if (ri < nrows && key < sm.limit[ri])
        p.logits[static_cast<int64_t>(r0 + ri - p.query_offset) * p.logits_row_stride + key] =
            v * scale;
    };
    if (H == 1) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int c0 = 8 * nt + 2 * t4;
        store(c0, key_lo, fmaxf(acc[nt][0], 0.f) * sm.w[c0]);
        store(c0 + 1, key_lo, fmaxf(acc[nt][1], 0.f) * sm.w[c0 + 1]);
        store(c0, key_hi, fmaxf(acc[nt][2], 0.f) * sm.w[c0]);
        store(c0 + 1, key_hi, fmaxf(acc[nt][3], 0.f) * sm.w[c0 + 1]);
      }
    } else if (H <= 8) {
      const int half = H >> 1;  // lanes sharing one row inside an n-tile
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int c0 = 8 * nt + 2 * t4;
        const float w0 = sm.w[c0], w1 = sm.w[c0 + 1];
        float vlo = fmaxf(acc[nt][0], 0.f) * w0 + fmaxf(acc[nt][1], 0.f) * w1;
        float vhi = fmaxf(acc[nt][2], 0.f) * w0 + fmaxf(acc[nt][3], 0.f) * w1;
        for (int o = 1; o < half; o <<= 1) {
          vlo += __shfl_xor_sync(0xffffffffu, vlo, o);
          vhi += __shfl_xor_sync(0xffffffffu, vhi, o);
        }
        if ((t4 & (half - 1)) == 0) {
          store(c0 / H, key_lo, vlo);
          store(c0 / H, key_hi, vhi);
        }
      }
    } else {  // H a multiple of 8: H/8 consecutive n-tiles form one row
      const int per_row = H >> 3;
      for (int nt0 = 0; nt0 < NT; nt0 += per_row) {
        float vlo = 0.f, vhi = 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt < nt0 || nt >= nt0 + per_row) continue;
          const int c0 = 8 * nt + 2 * t4;
          const float w0 = sm.w[c0], w1 = sm.w[c0 + 1];
          vlo += fmaxf(acc[nt][0], 0.f) * w0 + fmaxf(acc[nt][1], 0.f) * w1;
          vhi += fmaxf(acc[nt][2], 0.f) * w0 + fmaxf(acc[nt][3], 0.f) * w1;
        }
        vlo += __shfl_xor_sync(0xffffffffu, vlo, 1);
        vhi += __shfl_xor_sync(0xffffffffu, vhi, 1);
        vlo += __shfl_xor_sync(0xffffffffu, vlo, 2);
        vhi += __shfl_xor_sync(0xffffffffu, vhi, 2);
        if (t4 == 0) {
          store(nt0 / per_row, key_lo, vlo);
          store(nt0 / per_row, key_hi, vhi);
        }
      }
    }
  }
  cp_async_wait<0>();
}

template <int D, int NT>
cudaError_t launch_dn(const IndexerParams& p, dim3 grid, int rows_per_cta, int keys_per_cta,
                      cudaStream_t stream) {
  const size_t smem = sizeof(IdxSmem<D, NT>);
  cudaError_t e = set_attr_once(reinterpret_cast<const void*>(indexer_kernel<D, NT>), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return count_launches(launch_kernel(indexer_kernel<D, NT>, grid, dim3(kThreads), smem, stream,
                                      1, p, rows_per_cta, keys_per_cta));
}

template <int D>
cudaError_t launch_d(const IndexerParams& p, int nt, dim3 grid, int rpc, int kpc,
                     cudaStream_t s) {
  switch (nt) {
    case 1: return launch_dn<D, 1>(p, grid, rpc, kpc, s);
    case 2: return launch_dn<D, 2>(p, grid, rpc, kpc, s);
    case 4: return launch_dn<D, 4>(p, grid, rpc, kpc, s);
    case 8: return launch_dn<D, 8>(p, grid, rpc, kpc, s);
    case 16: return launch_dn<D, 16>(p, grid, rpc, kpc, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_indexer(const IndexerParams& p, cudaStream_t stream) {
  if (p.num_rows <= 0) return cudaSuccess;
  // The tensor-core kernel takes every shape its tensor maps can address;
  // the mma.sync kernel covers the rest (pages not a multiple of 8 rows).
  if (indexer_tc_eligible(p)) {
    const cudaError_t e = launch_indexer_tc(p, stream);
    if (e != cudaErrorNotSupported) return e;  // else: tensor maps refused these strides
  }
  const bool decode = p.query_start_loc == nullptr;
  const int H = p.heads;
  int rows_per_cta, requests, row_tiles, keys_per_cta;
  if (decode) {
    rows_per_cta = p.decode_query_len;
    requests = p.num_rows / p.decode_query_len;
    row_tiles = 1;
    keys_per_cta = kMaxKeysPerCta;
  } else {
    rows_per_cta = std::max(1, 128 / H);
    requests = p.num_requests;
    row_tiles = (std::min(p.num_rows, p.max_query_len) + rows_per_cta - 1) / rows_per_cta;
    keys_per_cta = 512;
  }
  const int n = rows_per_cta * H;
  int nt = 1;
  while (nt * 8 < n) nt <<= 1;
  if (nt > 16) return cudaErrorInvalidValue;
  const int cap = std::min(p.logits_width, p.table_width * p.page_size);
  const int chunks = std::max(1, (cap + keys_per_cta - 1) / keys_per_cta);
  if (requests <= 0 || row_tiles <= 0) return cudaSuccess;
  const dim3 grid(requests, row_tiles, chunks);
  if (p.dim == 64) return launch_d<64>(p, nt, grid, rows_per_cta, keys_per_cta, stream);
  if (p.dim == 128) return launch_d<128>(p, nt, grid, rows_per_cta, keys_per_cta, stream);
  return cudaErrorInvalidValue;
}

}  // namespace qsa

namespace qsa {
namespace {
__global__ void visible_blocks_kernel(const int64_t* positions, const int32_t* seq_lens,
                                      int num_requests, const int32_t* token_to_req, int rows,
                                      int ratio, int32_t* visible) {
  // Unlike the other kernels, this one lets its dependents start only after
  // its counts are written and made visible device-wide (the fence): the
  // next kernel may read them before its own wait, as step metadata.
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) visible[r] = visible_of(positions, seq_lens, num_requests, token_to_req, ratio, r);
  __threadfence();
  pdl_trigger();
}
}  // namespace

cudaError_t launch_visible_blocks(const int64_t* positions, const int32_t* seq_lens,
                                  int num_requests, const int32_t* token_to_req, int rows,
                                  int ratio, int32_t* visible, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  return count_launches(launch_kernel(visible_blocks_kernel, dim3((rows + 255) / 256), dim3(256),
                                      0, stream, 1, positions, seq_lens, num_requests,
                                      token_to_req, rows, ratio, visible));
}
}  // namespace qsa
