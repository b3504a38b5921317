// tma.cuh -- sm_100a async-copy and launch-chaining primitives (inline PTX).
//
// * 1-D bulk copies global -> shared (cp.async.bulk) completing on an
//   mbarrier transaction count; this CTA's own shared memory only, no
//   cluster multicast.
// * mbarrier init / arrive / bounded parity wait.
// * programmatic dependent launch: griddepcontrol.wait blocks until the
//   preceding grid in the stream has completed and flushed its writes;
//   griddepcontrol.launch_dependents lets the next grid start launching.
#pragma once

#include <stdint.h>

namespace mcpo {

// Iterations of a try_wait loop before a wait is declared failed.
constexpr int kWaitLimit = 1 << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the warp is parked (no issue slots
// spent polling) until the phase completes or `ns` nanoseconds pass.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded parked wait for a whole warp waiting on the same barrier (at most
// kSleepLimit hints of 2 us, about 2 s).
constexpr int kSleepLimit = 1 << 20;
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* err) {
  for (int i = 0; i < kSleepLimit; ++i)
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
  if (err) atomicExch(err, 1);
  return false;
}

// Bounded wait: returns false (and raises *err) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (int i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicExch(err, 1);
  return false;
}

// Bounded wait that also gives up, without raising *err, once *abort is set
// (checked every 64 polls): used where another party may abandon the work.
__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity, int* err, const volatile int* abort) {
  for (int i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && (i & 63) == 63 && *abort) return false;
  }
  if (err) atomicExch(err, 1);
  return false;
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global memory into this CTA's shared memory; completes on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// L2 policy for data read once per decode step (weights, KV rows): evicted
// first, so the step's weight stream does not push code, activations and
// small tables out of the 126 MB L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_load with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Kernel timelines are compiled in only with MCPO_TRACE=1 (a diagnostic
// build): even untaken stamp code slows the GEMV's hot loop measurably.
#ifndef MCPO_TRACE
#define MCPO_TRACE 0
#endif

// globaltimer (ns) into t[i] when a timeline is being recorded.
__device__ __forceinline__ void trace_stamp(unsigned long long* t, int i) {
  if (t) {
    unsigned long long v;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(v));
    t[i] = v;
  }
}
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace mcpo
