// chain.cu -- GEMV chains as one persistent launch (see chain.cuh).
//
// Synchronisation:
//  * stage k+1 starts once every CTA has finished stage k: an arrival
//    counter per barrier (zeroed before each launch), release by a CTA
//    barrier then thread 0's red.release, acquire by thread 0's
//    ld.acquire polling then a CTA barrier; the wait is
//    bounded (1 s of globaltimer), after which the CTA raises the error word
//    and the abort flag, and the other CTAs leave at their next barrier;
//  * the producer warp waits for its consumers' free slots with bounded
//    waits that also give up once the abort flag is set, and leaves only
//    after every copy it issued into shared memory has landed;
//  * every CTA must be resident at once: one CTA per SM, grid = SM count,
//    and the next kernel may launch only after all of this grid's CTAs have
//    started (each CTA allows it at its start), so it cannot take the SMs a
//    CTA of this grid still needs.
#include "chain.cuh"

#include <algorithm>

#include "gemv_dev.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr size_t kChainSmemMax = 232448;  // opt-in shared memory per CTA on sm_100
// Consumer warps at most (+1 producer warp).  Sixteen do not fit beside a
// 12288-column activation region and two 6.7 KB Q6_K slots per warp, and
// 512 threads leave each thread 128 registers, which the stage loop needs
// without spilling.
constexpr int kChainMaxConsumers = 15;

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t chain_timer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// This CTA's warp-rows of a stage: the standalone GEMV's partition (whole
// 32-row blocks per CTA when the stage writes Q8_1 output blocks).
__device__ __forceinline__ void chain_range(const GemvArgs& a, int b, int G, int& wr0, int& nwr, int& blk0,
                                            int& nblk) {
  const int T = a.total_wr;
  if (a.q8_out) {
    const int NB = (a.seg[0].rows + 31) / 32, wpb = 32 / a.seg[0].rpw;
    blk0 = (int)((long long)b * NB / G);
    nblk = (int)((long long)(b + 1) * NB / G) - blk0;
    wr0 = min(blk0 * wpb, T);
    nwr = min((blk0 + nblk) * wpb, T) - wr0;
  } else {
    blk0 = nblk = 0;
    wr0 = (int)((long long)b * T / G);
    nwr = (int)((long long)(b + 1) * T / G) - wr0;
  }
}

// Barrier k over the grid, for the NC*32 consumer threads (named barrier
// 1); false when this CTA is to leave (the wait gave up or another CTA did).
// The CTA barrier orders every consumer's stores of the stage before thread
// 0's release-add; thread 0's acquire polls, then the CTA barrier, order
// the next stage's loads after every CTA's arrival (no full fence: a
// sequentially consistent fence costs microseconds under the weight
// stream).
__device__ bool chain_grid_sync(const GemvChain& c, int k, int nthr, volatile int* abort_s) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  if (threadIdx.x == 0 && !*abort_s) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(c.bar + k) : "memory");
    const uint64_t t0 = chain_timer();
    for (unsigned it = 0;; ++it) {
      if (ld_acquire_gpu_u32(c.bar + k) >= gridDim.x) break;
      if (*reinterpret_cast<volatile int*>(c.abort)) {
        *abort_s = 1;
        break;
      }
      if ((it & 255u) == 255u && (chain_timer() - t0 > 1000000000ull || it > (1u << 24))) {
        *abort_s = 1;
        atomicExch(c.err, 1);
        atomicExch(c.abort, 1);
        break;
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  return *abort_s == 0;
}

template <int kClass>
__global__ void __launch_bounds__((kChainMaxConsumers + 1) * 32, 1) k_gemv_chain(const GemvChain c) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ GemvArgs sa[kMaxChain];  // every stage's arguments (consumers)
  __shared__ int abort_s;
  const int NC = c.nc, S = c.S, slot = c.slot;
  uint8_t* xbase = smem;
  uint8_t* ring = smem + c.x_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)NC * S * slot);
  uint64_t* empty = full + NC * S;
  float* q8stage = reinterpret_cast<float*>(empty + NC * S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x, G = gridDim.x;

  if (threadIdx.x == 0) {
    abort_s = 0;
    for (int i = 0; i < NC * S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_fence_init();
    pdl_launch_dependents();
  }
  __syncthreads();

  if (warp == NC) {
    // ---- producer: lane w feeds consumer warp w's ring with every stage's
    // step blocks in order; the weights need nothing from earlier work, so
    // it runs ahead across the barriers as far as the ring allows
    const int w = lane;
    if (w >= NC) return;
    const uint64_t policy = l2_evict_first_policy();
    int n = 0;
    bool ok = true;
    for (int st = 0; st < c.n && ok; ++st) {
      const GemvArgs& a = c.stages[st];
      int wr0, nwr, blk0, nblk;
      chain_range(a, b, G, wr0, nwr, blk0, nblk);
      const int ks = a.seg[0].ks, spi = ks * (a.seg[0].epi == kEpiSwiglu ? 2 : 1);
      const int steps = (nwr > w ? (nwr - w + NC - 1) / NC : 0) * spi;
      for (int k = 0; k < steps; ++k, ++n) {
        const int sidx = n % S;
        if (n >= S && !mbar_wait_abort(&empty[w * S + sidx], (uint32_t)((n / S) - 1) & 1u, c.err, c.abort)) {
          ok = false;
          break;
        }
        const int item = k / spi, rem = k % spi, part = rem / ks, kk = rem % ks;
        const int wr = wr0 + w + NC * item;
        const GemvSeg& s = seg_of(a, wr);
        const uint8_t* src = (part ? s.w2 : s.w) + (size_t)(wr - s.wr_begin) * s.wr_bytes + (size_t)kk * s.step_bytes;
        mbar_arrive_expect_tx(&full[w * S + sidx], (uint32_t)s.step_bytes);
        bulk_load_hint(ring + (size_t)(w * S + sidx) * slot, src, (uint32_t)s.step_bytes, &full[w * S + sidx], policy);
      }
    }
    // leave only once every copy issued into this CTA's shared memory has landed
    for (int m = n - S > 0 ? n - S : 0; m < n; ++m)
      if (!mbar_wait(&full[w * S + m % S], (uint32_t)(m / S) & 1u, c.err)) break;
    return;
  }

  // ---- consumers: the stages in turn.  Every stage's arguments are
  // copied into shared memory once, while the previous kernel finishes.
  const int nthr = NC * 32, tid = threadIdx.x;
  for (int st = 0; st < c.n; ++st) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(c.stages + st);
    uint32_t* dst = reinterpret_cast<uint32_t*>(&sa[st]);
    for (int i = tid; i < (int)(sizeof(GemvArgs) / 4); i += nthr) dst[i] = src[i];
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  int n = 0;
  for (int st = 0; st < c.n; ++st) {
    const GemvArgs& a = sa[st];
#if MCPO_TRACE
    unsigned long long* tr = c.trace ? c.trace + ((size_t)(st / 2) * c.trace_ctas + b) * 8 + (st % 2) * 4 : nullptr;
#endif
    // the RMSNorm weights need nothing from earlier stages: loaded before
    // the wait for them
    float wpre[8];
    gemv_norm_weights(a, warp, lane, wpre);
    if (st == 0) {
      pdl_wait();  // the first stage's activations come from the previous kernel
    } else if (!chain_grid_sync(c, st - 1, nthr, &abort_s)) {
      break;
    }
#if MCPO_TRACE
    if (tid == 0) trace_stamp(tr, 0);
#endif
    int wr0, nwr, blk0, nblk;
    chain_range(a, b, G, wr0, nwr, blk0, nblk);
    gemv_build_x<false>(a, xbase, NC, warp, lane, wpre);
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
#if MCPO_TRACE
    if (tid == 0) trace_stamp(tr, 1);
#endif
    const XShared x = gemv_x_view(xbase, a.cols);
    if (!gemv_items<kClass, false>(a, x, ring, full, empty, S, slot, wr0, nwr, NC, warp, lane, n, nullptr,
                                   a.q8_out ? q8stage : nullptr, blk0 * 32)) {
      atomicExch(c.abort, 1);
    }
#if MCPO_TRACE
    if (tr) {
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
      if (tid == 0) trace_stamp(tr, 2);
    }
#endif
    if (a.q8_out) {
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
      const int rows = a.seg[0].rows;
      for (int bb = warp; bb < nblk; bb += NC) {
        const int r = (blk0 + bb) * 32 + lane;
        quant_block_warp(r < rows ? q8stage[bb * 32 + lane] : 0.0f, a.q8_out + (size_t)(blk0 + bb) * 36, lane);
      }
    }
#if MCPO_TRACE
    if (tr) {
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
      if (tid == 0) trace_stamp(tr, 3);
    }
#endif
  }
}

template <int kClass>
cudaError_t set_chain_attr() {
  return cudaFuncSetAttribute(k_gemv_chain<kClass>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)(kChainSmemMax - 2048 - kMaxChain * sizeof(GemvArgs)));
}

}  // namespace

cudaError_t chain_init() {
  const cudaError_t r[] = {set_chain_attr<kClassQ4K>(), set_chain_attr<kClassQ6K>(), set_chain_attr<kClassQ80>(),
                           set_chain_attr<kClassQ4K6K>()};
  for (cudaError_t e : r)
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

bool chain_layout(const GemvArgs* stages, const int* dtype_masks, int n, int sm_count, GemvChain* c, size_t* smem) {
  if (n < 1 || n > kMaxChain || sm_count < 1) return false;
  int slot = 0, cols = 0, q8 = 0, mask = 0;
  for (int i = 0; i < n; ++i) {
    const GemvArgs& a = stages[i];
    mask |= dtype_masks[i];
    if (a.nvec > 1 || a.dots || a.input == kInRmsNormTp || a.seg[0].epi == kEpiTpPush || a.total_wr < 1) return false;
    slot = std::max(slot, a.slot_bytes);
    cols = std::max(cols, a.cols);
    if (a.q8_out) {
      const int NB = (a.seg[0].rows + 31) / 32;
      q8 = std::max(q8, (NB + sm_count - 1) / sm_count * 32);
    }
  }
  // bit 0 Q4_K, 1 Q6_K, 2 Q8_0 (gemv_prepare); Q8_0 does not mix with the K-quants
  if ((mask & 4) && (mask & 3)) return false;
  c->cls = (mask & 4) ? kClassQ80 : (mask & 3) == 3 ? kClassQ4K6K : (mask & 2) ? kClassQ6K : kClassQ4K;
  const size_t xb = gemv_x_bytes_host(cols);
  const size_t budget = kChainSmemMax - 2048 - kMaxChain * sizeof(GemvArgs);
  const size_t fixed = xb + (size_t)q8 * 4;
  if (fixed >= budget) return false;
  // the deepest ring (up to 4 slots) that still gives every consumer warp
  // a ring, else 2 slots and as many warps as fit
  int S = 2, nc = 0;
  for (int s = 4; s >= 2; --s) {
    nc = (int)std::min<size_t>((budget - fixed) / ((size_t)s * ((size_t)slot + 16)), kChainMaxConsumers);
    S = s;
    if (nc == kChainMaxConsumers) break;
  }
  if (nc < 8) return false;
  c->n = n;
  c->nc = nc;
  c->S = S;
  c->slot = slot;
  c->x_bytes = (int)xb;
  c->q8_floats = q8;
  *smem = fixed + (size_t)nc * S * slot + (size_t)2 * nc * S * 8;
  return true;
}

cudaError_t launch_gemv_chain(const GemvChain& c, int grid, size_t smem, cudaStream_t st) {
  if (c.n < 1 || c.n > kMaxChain || c.nc < 1 || c.nc > kChainMaxConsumers || c.S < 1 || grid < 1 || !c.stages || !c.bar ||
      !c.abort)
    return cudaErrorInvalidValue;
  const dim3 block((c.nc + 1) * 32);
  switch (c.cls) {
    case kClassQ4K: return launch_k(k_gemv_chain<kClassQ4K>, dim3(grid), block, smem, st, true, c);
    case kClassQ6K: return launch_k(k_gemv_chain<kClassQ6K>, dim3(grid), block, smem, st, true, c);
    case kClassQ80: return launch_k(k_gemv_chain<kClassQ80>, dim3(grid), block, smem, st, true, c);
    case kClassQ4K6K: return launch_k(k_gemv_chain<kClassQ4K6K>, dim3(grid), block, smem, st, true, c);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mcpo
