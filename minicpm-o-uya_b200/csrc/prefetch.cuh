// prefetch.cuh -- L2 prefetch of weight bytes that later kernels of the
// decode step will stream.
//
// Batch-1 decode is a weight stream cut into ~180 dependent kernels per
// token; HBM idles during every prologue, attention and kernel boundary.
// A kernel therefore asks L2 for a window of the bytes the next kernels
// will read (cp.async.bulk.prefetch.L2: no shared memory, no completion to
// wait for), so that HBM keeps streaming while the dependency chain runs,
// and the later kernels read those bytes at L2 speed.  Which bytes each
// kernel prefetches is planned on the host (the step's weights in
// consumption order, a sliding window ahead of each kernel).
#pragma once

#include <stdint.h>

namespace mcpo {

// Byte ranges (16-byte aligned start, size a multiple of 16) one launch
// prefetches; every CTA of the launch takes its 1/gridDim share of each.
constexpr int kMaxPf = 4;
struct PfRange {
  const uint8_t* p;
  unsigned long long bytes;
};
struct PfList {
  PfRange r[kMaxPf];
  int n;
};

// One prefetch request covers at most this many bytes.
constexpr unsigned kPfChunk = 32768;

#ifdef __CUDACC__
__device__ __forceinline__ void l2_prefetch_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// CTA b of G prefetches its share of every range: bytes [lo, hi) with lo,
// hi the 16-byte boundaries b/G and (b+1)/G of the range, in chunks of up
// to kPfChunk bytes spread over nl lanes (this thread is lane `lane`).
__device__ __forceinline__ void l2_prefetch_share(const PfList& pf, int b, int G, int lane, int nl) {
  for (int i = 0; i < pf.n && i < kMaxPf; ++i) {
    const unsigned long long n16 = pf.r[i].bytes >> 4;
    const unsigned long long lo = (n16 * (unsigned long long)b / (unsigned long long)G) << 4;
    const unsigned long long hi = (n16 * (unsigned long long)(b + 1) / (unsigned long long)G) << 4;
    for (unsigned long long o = lo + (unsigned long long)lane * kPfChunk; o < hi;
         o += (unsigned long long)nl * kPfChunk) {
      const unsigned long long left = hi - o;
      l2_prefetch_bulk(pf.r[i].p + o, (uint32_t)(left < kPfChunk ? left : kPfChunk));
    }
  }
}
#endif

}  // namespace mcpo
