// Indexer scores on the 5th-generation tensor cores (tcgen05 + TMA), sm_100a.
//
// logits[r, c] = scale * sum_h w[r,h] * relu(q[r,h] . key(c)) for c < visible[r]
// (reference ops/indexer.py:24-114 decode, :117-223 prefill: bf16 inputs, fp32
// products, ReLU per head, head sum, head_dim^-0.5).
//
// One CTA owns the query columns of a request (decode: its decode_query_len
// rows; prefill: up to 128/H rows) and a chunk of that request's keys.
//  * warp 0: TMA producer.  Key tiles of 128 keys are loaded page by page
//    with 3-D tensor copies (dims: head dim, slot-in-page, physical page),
//    128-byte swizzled, into a 4-stage shared-memory ring (mbarrier
//    transaction counts).  An unmapped page is loaded through an
//    out-of-bounds page coordinate, which the TMA unit fills with zeros.
//  * warp 1: allocates TMEM and issues tcgen05.mma (M = 128 keys, N = the
//    CTA's query columns (rows x heads, padded to 16), K = 16 per
//    instruction) into a double-buffered fp32 TMEM accumulator; completion
//    is signalled with tcgen05.commit on mbarriers.
//  * warps 2-5: epilogue.  Each thread owns one key (one TMEM lane):
//    tcgen05.ld of its row of scores, ReLU, head weights, head sum, scale,
//    and a coalesced fp32 store per query row.
// Every wait is bounded; on expiry an error bit is recorded and the CTA
// drains its copies and MMAs before releasing TMEM and returning.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

constexpr int kTcThreads = 192;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kTcStages = 4;
constexpr int kTileKeys = 128;
constexpr int kTcMaxKeysPerCta = 1024;
constexpr int kTcMaxPages = kTcMaxKeysPerCta / 8 + 2;

template <int D, int NQ>
struct TcSmem {
  static constexpr int kSub = D / 64;                  // 128-byte sub-rows per key
  static constexpr int kSubBytes = kTileKeys * 128;    // one sub-tile: 128 rows x 128 B
  static constexpr int kStageBytes = kSub * kSubBytes;
  alignas(1024) uint8_t k[kTcStages][kStageBytes];     // [sub][key][128 B], SW128
  alignas(1024) uint8_t q[kSub][NQ * 128];             // [sub][column][128 B], SW128
  float w[NQ];
  int limit[NQ];
  int pages[kTcMaxPages];
  uint64_t full[kTcStages], empty[kTcStages], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

// UMMA shared-memory descriptor, K-major operand in the 128-byte swizzle
// atom layout: rows of 128 B, 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused here)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: 8-row atoms
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                  // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: D fp32, A/B bf16, both K-major, M x N.
template <int M, int N>
constexpr uint32_t instr_desc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1 : 0)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <int D, int NQ>
__global__ void __launch_bounds__(kTcThreads) indexer_tc_kernel(
    const __grid_constant__ CUtensorMap kmap, const IndexerParams p, int rows_per_cta,
    int keys_per_cta, int box_rows) {
  using S = TcSmem<D, NQ>;
  constexpr int kCols = 2 * NQ < 32 ? 32 : 2 * NQ;  // TMEM columns: two accumulators
  constexpr uint32_t kIdesc = instr_desc<kTileKeys, NQ>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the 128-byte swizzle pattern is taken from address bits: 1024-byte align
  S& sm = *reinterpret_cast<S*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
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
  const int cap = min(p.table_width * p.page_size, p.logits_width);
  int maxvis = 0;
  for (int i = 0; i < nrows; ++i) maxvis = max(maxvis, min(p.visible[r0 + i], cap));
  const int k0 = blockIdx.z * keys_per_cta;
  const int k1 = min(k0 + keys_per_cta, maxvis);
  if (k0 >= k1) return;  // uniform: before any barrier or TMEM allocation
  const int ntiles = (k1 - k0 + kTileKeys - 1) / kTileKeys;

  // ---- setup: barriers, TMEM, query tile (swizzled), weights, page slice.
  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.tfull[b], 1);
      mbar_init(&sm.tempty[b], 4);
    }
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid < NQ) {
    const int ri = tid / H, h = tid % H;
    const bool v = ri < nrows;
    sm.w[tid] = v ? (p.weights ? p.weights[static_cast<int64_t>(r0 + ri) * p.w_row_stride +
                                            static_cast<int64_t>(h) * p.w_head_stride]
                               : 1.f)
                  : 0.f;
    sm.limit[tid] = tid < nrows ? min(p.visible[r0 + tid], cap) : 0;
  }
  const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(p.q);
  for (int ch = tid; ch < NQ * (D / 8); ch += kTcThreads) {
    const int n = ch / (D / 8), c16 = ch % (D / 8);  // column n, 16-byte chunk c16 of D*2 bytes
    const int sub = c16 >> 3, c = c16 & 7;
    const int ri = n / H, h = n % H;
    const bool v = ri < nrows;
    const __nv_bfloat16* src = qb + static_cast<int64_t>(v ? r0 + ri : r0) * p.q_row_stride +
                               static_cast<int64_t>(v ? h : 0) * p.q_head_stride + c16 * 8;
    cp_async16(sm.q[sub] + n * 128 + ((c ^ (n & 7)) << 4), src, v);
  }
  const int32_t* trow = p.table + static_cast<int64_t>(req) * p.table_row_stride;
  const int pg0 = static_cast<int>(p.page_div.div(k0));
  const int pg1 = static_cast<int>(p.page_div.div(k1 - 1));
  for (int i = tid; i <= pg1 - pg0; i += kTcThreads) sm.pages[i] = trow[pg0 + i];
  cp_async_commit();
  cp_async_wait<0>();
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // q tile -> tensor-core reads
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int boxes = kTileKeys / box_rows;
      int t = 0;
      for (; t < ntiles; ++t) {
        const int s = t % kTcStages;
        if (t >= kTcStages && !mbar_wait(&sm.empty[s], ((t / kTcStages) - 1) & 1)) {
          record_error(p.err, kDeviceErrWaitTimeout);
          sm.abort_flag = 1;
          break;
        }
        mbar_expect_tx(&sm.full[s], S::kStageBytes);
        for (int bx = 0; bx < boxes; ++bx) {
          const int key = k0 + t * kTileKeys + bx * box_rows;  // first key of the box
          int lp, off;
          p.page_div.divmod(key, lp, off);
          int page = (lp <= pg1) ? sm.pages[lp - pg0] : -1;
          if (page < 0 || page >= p.num_blocks) page = p.num_blocks;  // OOB: zero-filled
#pragma unroll
          for (int sub = 0; sub < S::kSub; ++sub)
            tma_load_3d(sm.k[s] + sub * S::kSubBytes + bx * box_rows * 128, &kmap, sub * 64, off,
                        page, &sm.full[s]);
        }
        mbar_arrive(&sm.full[s]);
      }
      // drain: every issued tile has landed before the CTA may retire
      for (int j = std::max(0, t - kTcStages); j < t; ++j)
        if (!mbar_wait(&sm.full[j % kTcStages], (j / kTcStages) & 1))
          record_error(p.err, kDeviceErrWaitTimeout);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int t = 0;
      for (; t < ntiles; ++t) {
        const int s = t % kTcStages, b = t & 1;
        if (!mbar_wait(&sm.full[s], (t / kTcStages) & 1) ||
            (t >= 2 && !mbar_wait(&sm.tempty[b], ((t >> 1) - 1) & 1))) {
          record_error(p.err, kDeviceErrWaitTimeout);
          sm.abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t kbase = smem_u32(sm.k[s]);
        const uint32_t qbase = smem_u32(sm.q[0]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int sub = kk >> 2, part = kk & 3;
          const uint64_t ad = sw128_desc(kbase + sub * S::kSubBytes + part * 32);
          const uint64_t bd = sw128_desc(qbase + sub * NQ * 128 + part * 32);
          umma_bf16(tmem + b * NQ, ad, bd, kIdesc, kk > 0);
        }
        umma_commit(&sm.empty[s]);   // stage reusable once these MMAs have read it
        umma_commit(&sm.tfull[b]);   // accumulator b ready for the epilogue
      }
      // drain: the last MMAs have completed before TMEM is released
      if (t > 0 && !mbar_wait(&sm.tfull[(t - 1) & 1], ((t - 1) >> 1) & 1))
        record_error(p.err, kDeviceErrWaitTimeout);
    }
  } else {
    // ------------------------------------------------------ epilogue
    const int quad = warp & 3;          // TMEM lanes 32*quad .. +31 = keys of this warp
    const int key_in_tile = quad * 32 + lane;
    const float scale = p.scale;
    const int rows_here = NQ / H < nrows ? NQ / H : nrows;
    for (int t = 0; t < ntiles; ++t) {
      const int b = t & 1;
      // warp-uniform decisions: the tcgen05.ld below is .sync.aligned
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&sm.abort_flag))) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.tfull[b], (t >> 1) & 1))) {
        if (lane == 0) {
          record_error(p.err, kDeviceErrWaitTimeout);
          sm.abort_flag = 1;
        }
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // scores of this thread's key for all NQ columns, 16 columns per load;
      // column n = (row n / H, head n % H): heads of a row are consecutive
      const int key = k0 + t * kTileKeys + key_in_tile;
      float acc = 0.f;
      int h = 0, ri = 0;
#pragma unroll
      for (int c = 0; c < NQ; c += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * NQ + c, v);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc += fmaxf(__uint_as_float(v[j]), 0.f) * sm.w[c + j];
          if (++h == H) {
            if (ri < rows_here && key < sm.limit[ri])
              p.logits[static_cast<int64_t>(r0 + ri - p.query_offset) * p.logits_row_stride +
                       key] = acc * scale;
            acc = 0.f;
            h = 0;
            ++ri;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tempty[b]);
    }
  }
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------- host side
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

template <int D, int NQ>
cudaError_t launch_tc(const IndexerParams& p, const CUtensorMap& map, dim3 grid, int rpc, int kpc,
                      int box_rows, cudaStream_t stream) {
  const size_t smem = sizeof(TcSmem<D, NQ>) + 1024;  // + slack for 1024-byte alignment
  cudaError_t e = set_attr_once(reinterpret_cast<const void*>(indexer_tc_kernel<D, NQ>),
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  indexer_tc_kernel<D, NQ><<<grid, kTcThreads, smem, stream>>>(map, p, rpc, kpc, box_rows);
  return cudaGetLastError();
}

}  // namespace

// Whether the tensor-core indexer takes these shapes (else the mma.sync path):
// head dim 64 / 128, page size a multiple of 8 (whole 8-row swizzle atoms per
// TMA box), 16-byte aligned strides, <= 128 query columns per CTA.
bool indexer_tc_eligible(const IndexerParams& p) {
  if (p.dim != 64 && p.dim != 128) return false;
  if (p.heads <= 0 || p.heads > 128) return false;
  if (p.page_size % 8 != 0) return false;
  if ((p.token_stride * 2) % 16 != 0 || (p.block_stride * 2) % 16 != 0) return false;
  if (reinterpret_cast<uintptr_t>(p.k_cache) % 16 != 0) return false;
  if (p.num_blocks <= 0) return false;
  if (p.query_start_loc == nullptr && p.decode_query_len * p.heads > 128) return false;
  return tensor_map_encoder() != nullptr;
}

cudaError_t launch_indexer_tc(const IndexerParams& p, cudaStream_t stream) {
  const bool decode = p.query_start_loc == nullptr;
  const int H = p.heads;
  int rows_per_cta, requests, row_tiles, keys_per_cta;
  if (decode) {
    rows_per_cta = p.decode_query_len;
    requests = p.num_rows / p.decode_query_len;
    row_tiles = 1;
    keys_per_cta = kTcMaxKeysPerCta;
  } else {
    rows_per_cta = std::max(1, 128 / H);
    requests = p.num_requests;
    row_tiles = (std::min(p.num_rows, p.max_query_len) + rows_per_cta - 1) / rows_per_cta;
    keys_per_cta = 512;
  }
  const int n = rows_per_cta * H;
  const int nq = n <= 16 ? 16 : n <= 32 ? 32 : n <= 64 ? 64 : 128;
  const int cap = std::min(p.logits_width, p.table_width * p.page_size);
  const int chunks = std::max(1, (cap + keys_per_cta - 1) / keys_per_cta);
  if (requests <= 0 || row_tiles <= 0) return cudaSuccess;
  const int box_rows = gcd_int(p.page_size, kTileKeys);

  // 3-D tensor map over the key cache: (head dim, slot in page, page).
  CUtensorMap map;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.dim),
                              static_cast<cuuint64_t>(p.page_size),
                              static_cast<cuuint64_t>(p.num_blocks)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.token_stride) * 2,
                                 static_cast<cuuint64_t>(p.block_stride) * 2};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = tensor_map_encoder()(
      &map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p.k_cache), dims, strides,
      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const dim3 grid(requests, row_tiles, chunks);
  if (p.dim == 64) {
    switch (nq) {
      case 16: return launch_tc<64, 16>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
      case 32: return launch_tc<64, 32>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
      case 64: return launch_tc<64, 64>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
      default: return launch_tc<64, 128>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
    }
  }
  switch (nq) {
    case 16: return launch_tc<128, 16>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
    case 32: return launch_tc<128, 32>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
    case 64: return launch_tc<128, 64>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
    default: return launch_tc<128, 128>(p, map, grid, rows_per_cta, keys_per_cta, box_rows, stream);
  }
}

}  // namespace qsa
