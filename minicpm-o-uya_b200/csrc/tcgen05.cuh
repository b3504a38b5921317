// tcgen05.cuh -- sm_100a tensor-core primitives shared by the batched
// decode GEMM (gemm.cu) and the prefill GEMM (pgemm.cu): shared-memory
// matrix descriptors, tensor-memory allocation, MMA completion, fences and
// the bounded mbarrier wait with an abort flag (inline PTX).
#pragma once

#include <stdint.h>

#include "tma.cuh"

namespace mcpo {

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes stored contiguously (128 bytes); lbo = byte distance
// between the two 16-byte K-chunks of one MMA, sbo = byte distance between
// consecutive 8-row groups.  Version 1 (sm_100), base offset 0.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// Arrives on `bar` once every tcgen05 operation this thread issued before it
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Bounded wait that leaves early once the CTA's abort flag is set; raises
// the error word and the flag when it gives up.
__device__ __forceinline__ bool gwait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_s) {
  for (int i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && *abort_s) return false;
  }
  *abort_s = 1;
  if (err) atomicExch(err, 1);
  return false;
}

}  // namespace mcpo
