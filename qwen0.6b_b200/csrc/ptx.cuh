// Hand-written PTX helpers for sm_100a: mbarriers, bulk (TMA) copies,
// flag-carrying 8-byte handoff words, bounded waits.
//
// Every wait here is bounded: it gives up after a wall-clock limit read from
// %globaltimer, or as soon as the CTA-local or kernel-wide abort flag is set,
// and reports failure to the caller instead of spinning forever.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace qb200 {

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
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

// Non-blocking probe of a phase (cheaper than try_wait when it has completed).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// ------------------------------------------------------------- bulk copies
// Non-tensor bulk copy global -> this CTA's shared memory, completing on an
// mbarrier with a byte count.  No cluster multicast: every copy reads this
// GPU's own global memory into this CTA only.  src, dst 16-byte aligned and
// bytes a multiple of 16 (checked by the caller before issue).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Starts pulling `bytes` at `src` into L2 (no destination, no completion
// signal); src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Orders this thread's prior generic-proxy global writes before later
// async-proxy (bulk copy) accesses, in both directions.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ------------------------------------------------ 8-byte flag-carrying words
// A handoff word is 64 bits: low 32 = payload, high 32 = epoch.  8-byte
// aligned relaxed accesses at gpu scope are single-copy atomic, so a reader
// that sees the expected epoch also sees the payload written with it, and
// the read never hits a stale L1 line.
// No "memory" clobber: these relaxed accesses order nothing else, and a
// clobber would force every value the compiler holds from memory (kernel
// parameters included) to be reloaded after each handoff access.
__device__ __forceinline__ void ll_store(uint64_t *p, uint32_t payload, uint32_t epoch) {
  uint64_t v = (static_cast<uint64_t>(epoch) << 32) | payload;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v));
}

__device__ __forceinline__ uint64_t ll_load(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add_u32(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Programmatic dependent launch.  griddep_wait blocks until the preceding
// kernel in the stream has completed and its memory is visible (a no-op when
// this kernel was not launched as a dependent); griddep_launch_dependents lets
// the next kernel's CTAs be scheduled once every CTA of this grid has called
// it or exited (they still wait for this grid before reading its outputs).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Consumer-only named barrier (the producer warp never joins it).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads, so
// every thread leaves with the same value (used for uniform abort decisions).
__device__ __forceinline__ bool named_bar_or(uint32_t id, uint32_t nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t h2u(__half h) { return static_cast<uint32_t>(__half_as_ushort(h)); }
__device__ __forceinline__ __half u2h(uint32_t u) { return __ushort_as_half(static_cast<unsigned short>(u & 0xffffu)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// fp32 dot of 8 fp16 weights with 8 fp16 activations (fp32 products).
__device__ __forceinline__ float dot8_hh(const uint4 &w, const uint4 &x, float acc) {
  const __half2 *wh = reinterpret_cast<const __half2 *>(&w);
  const __half2 *xh = reinterpret_cast<const __half2 *>(&x);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 a = __half22float2(wh[i]);
    float2 b = __half22float2(xh[i]);
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
  }
  return acc;
}

// fp32 dot of 8 fp16 weights with 8 fp32 activations.
__device__ __forceinline__ float dot8_hf(const uint4 &w, const float4 &x0, const float4 &x1,
                                         float acc) {
  const __half2 *wh = reinterpret_cast<const __half2 *>(&w);
  float2 a = __half22float2(wh[0]);
  acc = fmaf(a.x, x0.x, acc);
  acc = fmaf(a.y, x0.y, acc);
  a = __half22float2(wh[1]);
  acc = fmaf(a.x, x0.z, acc);
  acc = fmaf(a.y, x0.w, acc);
  a = __half22float2(wh[2]);
  acc = fmaf(a.x, x1.x, acc);
  acc = fmaf(a.y, x1.y, acc);
  a = __half22float2(wh[3]);
  acc = fmaf(a.x, x1.z, acc);
  acc = fmaf(a.y, x1.w, acc);
  return acc;
}

}  // namespace qb200
