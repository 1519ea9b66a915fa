// tcgen05 / TMA building blocks shared by the tensor-core kernels (sm_100a):
// UMMA shared-memory and instruction descriptors, tensor-map TMA loads,
// tcgen05.mma / commit / ld wrappers, and warp-uniform bounded waits.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace qsa {

// Tensor-map encoder from the driver (cuTensorMapEncodeTiled), resolved once;
// nullptr when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
int gcd_int(int a, int b);
// Tensor maps of the indexer's key cache and query rows (indexer_tc.cu).
bool encode_indexer_maps(const IndexerParams& p, int box_rows, int rows_per_seg, int q_rows,
                         CUtensorMap* kmap, CUtensorMap* qmap);

namespace {

constexpr int kTileKeys = 128;  // keys per tcgen05.mma (M)

// UMMA shared-memory descriptor of a K-major operand in the 128-byte swizzle
// atom layout: rows of 128 B, 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused: swizzled)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: 8-row atoms
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                  // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor of kind::f16: D fp32, A and B bf16, both K-major, M x N.
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

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// A read-only load that is issued exactly where it is written (the page-id
// window is fetched ahead of its use).
__device__ __forceinline__ int ld_once(const int32_t* ptr) {
  int v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(ptr));
  return v;
}

// Warp-uniform bounded wait: true when the phase completed for every lane.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

__device__ __forceinline__ bool aborted(const int* flag) {
  return __any_sync(0xffffffffu, *reinterpret_cast<const volatile int*>(flag) != 0);
}

}  // namespace
}  // namespace qsa
