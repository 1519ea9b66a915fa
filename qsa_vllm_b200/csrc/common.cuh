// Shared device helpers for the sm_100a QSA kernels: inline-PTX wrappers for
// mbarriers, bulk (TMA-engine) copies, cp.async, ldmatrix / movmatrix,
// bf16 mma.sync, and bounded waits that record an error instead of hanging.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <utility>

namespace qsa {

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s
constexpr int kDeviceErrWaitTimeout = 1;
// An index (slot, page, position, request) outside its buffer: the access was skipped.
constexpr int kDeviceErrOutOfRange = 2;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// Arrive without release semantics: for a consumer that hands a buffer back
// after it has finished reading it (no writes of its own to publish), so the
// arrive need not wait for the thread's outstanding global stores.
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.relaxed.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete.  Returns false (and
// never hangs) when the wait exceeds kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - start > kWaitLimitNs) return false;
  }
}

// ------------------------------------------------------------ bulk copies
// Non-tensor bulk copy global -> this CTA's shared memory, completing as
// transaction bytes on `bar`.  Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bulk prefetch of [src, src+bytes) into L2 (no shared memory involved).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------- tensor-core ops
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// D += A(16x16, row) * B(16x8, col), bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 2^x on the SFU (the same instruction the reference's tl.math.exp2 lowers to).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void record_error(int* err, int bits) {
  if (err != nullptr) atomicOr(err, bits);
}

// Division of non-negative 32-bit integers by a run-time constant through a
// multiply-high (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, unsigned case): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1,  n / d = (t + ((n - t) >> min(l,1))) >> max(l-1,0)
// where t = umulhi(m, n).  Exact for all n < 2^32, 1 <= d < 2^31.
struct FastDiv {
  uint32_t d, m, s1, s2;
  __host__ __device__ FastDiv() : d(1), m(1), s1(0), s2(0) {}
  __host__ explicit FastDiv(uint32_t divisor) : d(divisor) {
    uint32_t l = 0;
    while ((1ull << l) < divisor) ++l;
    m = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - divisor)) / divisor + 1);
    s1 = l < 1 ? l : 1;
    s2 = l > 0 ? l - 1 : 0;
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    const uint32_t t = __umulhi(m, n);
    return (t + ((n - t) >> s1)) >> s2;
  }
  // quotient and remainder of a non-negative int
  __device__ __forceinline__ void divmod(int n, int& q, int& r) const {
    q = static_cast<int>(div(static_cast<uint32_t>(n)));
    r = n - q * static_cast<int>(d);
  }
};

// ------------------------------------------------------ visible block count
// Python floor division (b > 0).
__device__ __forceinline__ long long floor_div_ll(long long a, long long b) {
  const long long q = a / b;
  return (a % b != 0 && a < 0) ? q - 1 : q;
}
// Compressed blocks row r may attend: min((pos + 1) // ratio, seq_len // ratio)
// for a row mapped to a request, else 0 (reference ops/indexer.py:363-369).
__device__ __forceinline__ int visible_of(const int64_t* positions, const int32_t* seq_lens,
                                          int num_sequences, const int32_t* token_to_req,
                                          int ratio, int r) {
  const int req = token_to_req[r];
  if (req < 0 || req >= num_sequences) return 0;
  const long long a = floor_div_ll(positions[r] + 1, ratio);
  const long long b = floor_div_ll(seq_lens[req], ratio);
  return static_cast<int>(a < b ? a : b);
}

// ------------------------------------------- programmatic dependent launch
// Every kernel of this library waits for the grids it depends on (the
// preceding kernels of its stream) before its first global memory access, and
// lets its own dependents launch right after.  Launched with programmatic
// stream serialization, a kernel's launch and prologue (barrier set-up, TMEM
// allocation, tensor-map prefetch) then overlap the tail of the kernel before
// it; launched without it, the wait returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// QSA_PDL=0 launches every kernel with plain stream order.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("QSA_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

// cudaLaunchKernelEx with programmatic stream serialization (when enabled)
// plus an optional cluster shape.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace qsa
