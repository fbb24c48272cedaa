// Shared device helpers for the kvbm_b200 sm_100a kernel library.
//
// Everything here is written for Blackwell (sm_100a): 16-byte vector global
// accesses, 1-D bulk async copies (cp.async.bulk into this CTA's own shared
// memory from this GPU's own memory) tracked by shared-memory mbarriers, and
// %globaltimer-bounded spin waits that give up with an error status instead
// of hanging the GPU.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#define KVBM_DEVICE __device__ __forceinline__

namespace kvbm {

// Status codes written into device-visible status words by kernels that can
// give up (bounded waits) or detect bad arguments at run time.
enum KvbmStatus : int {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,
  kStatusBadIndex = 2,
  kStatusPipelineTimeout = 3,
};

KVBM_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- 16-byte vector memory ops -------------------------------------------

KVBM_DEVICE int4 ld_v4(const void* p) {
  return *reinterpret_cast<const int4*>(p);
}
// Streaming load: data is touched once, do not keep it in L1.
KVBM_DEVICE int4 ld_v4_stream(const void* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
KVBM_DEVICE void st_v4(void* p, int4 v) { *reinterpret_cast<int4*>(p) = v; }

// ---- release/acquire flags at system scope (peer GPUs and host) ----------

KVBM_DEVICE void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
KVBM_DEVICE uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
KVBM_DEVICE void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// ---- mbarrier + bulk async copy (Hopper/Blackwell TMA engine) ------------

KVBM_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
KVBM_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
KVBM_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
KVBM_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
KVBM_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
KVBM_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
KVBM_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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
// Bounded wait: returns false if the phase did not complete within
// `limit_ns` nanoseconds of %globaltimer.
KVBM_DEVICE bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// `bar` in bytes. `src` must be LOCAL device memory (never a peer mapping),
// 16-byte aligned; `bytes` a multiple of 16.
KVBM_DEVICE void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy this CTA's shared memory -> global (TMA store), tracked in
// bulk async-groups. `gmem_dst` 16-byte aligned; `bytes` a multiple of 16.
KVBM_DEVICE void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
KVBM_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups still read shared memory.
template <int N>
KVBM_DEVICE void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups are incomplete (writes done).
template <int N>
KVBM_DEVICE void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// A status word a kernel may write from any thread: plain stores (the word
// can live in mapped host memory, where device atomics are not available on
// every host link), made visible at system scope.
KVBM_DEVICE void report_status(int* status, int code) {
  if (status != nullptr) {
    *reinterpret_cast<volatile int*>(status) = code;
    __threadfence_system();
  }
}

// ---- division by a run-time invariant ------------------------------------
//
// Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication" (PLDI 1994), round-up variant: for 1 <= d < 2^31 and
// 0 <= n < 2^31, q = (umulhi(n, m) + n) >> l with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1. Computed on the host, applied in
// three instructions on the device.
struct FastDiv {
  uint32_t d = 1, m = 0, l = 0;
  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t div) : d(div) {
    l = 0;
    while ((1ull << l) < d) ++l;
    m = static_cast<uint32_t>((((1ull << l) - d) << 32) / d + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
  __device__ __forceinline__ uint32_t mod(uint32_t n, uint32_t q) const { return n - q * d; }
};

// ---- warp reductions -------------------------------------------------------

KVBM_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
KVBM_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace kvbm
