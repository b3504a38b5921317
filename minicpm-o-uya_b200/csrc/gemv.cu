// gemv.cu -- batch-1 quantised GEMV (Q4_K / Q6_K / Q8_0 weights x Q8_1
// activations) for sm_100a, plus the Q8_1 activation producers.
//
// Arithmetic follows the reference CUDA path (gpu_shim.c:746-878): per
// 32-value (Q4_K, Q8_0) or 16-value (Q6_K) block an exact int32 dot of the
// weight quants with the Q8_1 quants (dp4a), scaled in f32:
//   Q4_K: d*sum_j(sc_j*d8_j*dot_j) - dmin*sum_j(m_j*d8_j*sum(q8_j))
//   Q6_K: d*sum_g(sc_g*d8*(sum((q6-32)*q8)))
//   Q8_0: sum_b(d_w*d8*dot_b)
// The Q4_K min term uses the integer sum of the block's q8 values, the same
// quantity as dp4a(0x01010101, q8) in gpu_shim.c:797-800.
//
// Design (batch-1 decode is a weight stream):
//  * weights are pre-tiled at upload (layout.cuh) into 16-byte aligned step
//    blocks; a persistent CTA per SM owns a contiguous range of warp-rows;
//  * one producer thread streams step blocks with cp.async.bulk (TMA) into a
//    ring of shared-memory slots per consumer warp (mbarrier full/empty
//    handshake, bounded waits), keeping ~100+ KB per SM in flight, and starts
//    before the previous kernel has finished (programmatic dependent launch:
//    weights do not depend on it);
//  * eight consumer warps read their slots with conflict-free 16-byte shared
//    loads, decode scales in registers and reduce with dp4a and xor
//    butterflies;
//  * the Q8_1 activation vector lives in shared memory, transposed to
//    [16-byte chunk][super-block] so lanes of a row read consecutive 16-byte
//    words without bank conflicts;
//  * up to three matrices sharing one input (q/k/v) are one launch over a
//    common warp-row space, dtype chosen per warp-row;
//  * epilogues: store, residual add, SwiGLU pairing of gate and up rows.
// Float arithmetic uses only correctly rounded operations in a fixed order
// (per lane over its super-blocks, then the butterfly), so results do not
// depend on the launch shape.
#include "gemv.cuh"

#include <math.h>
#include <stdlib.h>

#include "gemv_dev.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {
// kTp: the tensor-parallel variant (summing prologue and/or push epilogue);
// the single-GPU kernel compiles none of that code.
template <int kClass, bool kDots, bool kTp>
__global__ void __launch_bounds__((kMaxConsumers + 1) * 32, 1) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int cols = a.cols;
  const int S = a.stages;
  const int slot = a.slot_bytes;
  const int NC = (int)(blockDim.x >> 5) - 1;  // consumer warps; the last warp produces
  uint8_t* ring = smem + gemv_x_region(cols, a.input);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)NC * S * slot);
  uint64_t* empty = full + NC * S;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#if MCPO_TRACE
  unsigned long long* tr = a.trace ? a.trace + (size_t)blockIdx.x * 8 : nullptr;
  if (threadIdx.x == 0) trace_stamp(tr, 0);
#endif
  const int T = a.total_wr, G = gridDim.x;
  int wr0, wr1, blk0 = 0, nblk = 0;
  if (a.q8_out) {
    // Q8_1 output: whole 32-row blocks per CTA, so each CTA quantises the
    // blocks of its own rows
    const int NB = (a.seg[0].rows + 31) / 32, wpb = 32 / a.seg[0].rpw;
    blk0 = (int)((long long)blockIdx.x * NB / G);
    nblk = (int)((long long)(blockIdx.x + 1) * NB / G) - blk0;
    wr0 = min(blk0 * wpb, T);
    wr1 = min((blk0 + nblk) * wpb, T);
  } else {
    wr0 = (int)((long long)blockIdx.x * T / G);
    wr1 = (int)((long long)(blockIdx.x + 1) * T / G);
  }
  const int nwr = wr1 - wr0;
  const bool swiglu = a.seg[0].epi == kEpiSwiglu;
  const int ks = a.seg[0].ks;
  const int spi = ks * (swiglu ? 2 : 1);  // steps per warp-row

  if (threadIdx.x == 0) {
    for (int i = 0; i < NC * S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == NC) {
    // ---- producer warp: lane w streams consumer warp w's step blocks into
    // that warp's ring (independent lanes, so one slow consumer never holds
    // up the copies of another).  Needs nothing from the previous kernel, so
    // it does not wait for it.
    const int w = lane;
    if (w >= NC) return;
    const int steps = (nwr > w ? (nwr - w + NC - 1) / NC : 0) * spi;
    const uint64_t policy = l2_evict_first_policy();
    bool ok = true;
    for (int n = 0; n < steps; ++n) {
      const int sidx = n % S;
      if (n >= S && !mbar_wait(&empty[w * S + sidx], (uint32_t)((n / S) - 1) & 1u, a.err)) {
        ok = false;
        break;
      }
      const int item = n / spi, rem = n % spi, part = rem / ks, k = rem % ks;
      const int wr = wr0 + w + NC * item;
      const GemvSeg& s = seg_of(a, wr);
      const uint8_t* src = (part ? s.w2 : s.w) + (size_t)(wr - s.wr_begin) * s.wr_bytes + (size_t)k * s.step_bytes;
      mbar_arrive_expect_tx(&full[w * S + sidx], (uint32_t)s.step_bytes);
      bulk_load_hint(ring + (size_t)(w * S + sidx) * slot, src, (uint32_t)s.step_bytes, &full[w * S + sidx], policy);
    }
    // Leave only once every copy issued into this CTA's shared memory has
    // landed (the consumers normally see to that; this covers their bail-out).
    (void)ok;
    for (int n = steps - S > 0 ? steps - S : 0; n < steps; ++n)
      if (!mbar_wait(&full[w * S + n % S], (uint32_t)(n / S) & 1u, a.err)) return;
    return;
  }

  // ---- consumers ----
  float wpre[8];
  gemv_norm_weights(a, warp, lane, wpre);
  pdl_wait();  // the activations (and y for the residual add) come from earlier kernels
#if MCPO_TRACE
  if (threadIdx.x == 0) trace_stamp(tr, 1);
#endif
  gemv_build_x<kTp>(a, smem, NC, warp, lane, wpre);
  asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
#if MCPO_TRACE
  if (threadIdx.x == 0) trace_stamp(tr, 2);
#endif
  if (threadIdx.x == 0) pdl_launch_dependents();
  const XShared x = gemv_x_view(smem, cols);
  int n = 0;
  float* stage = a.q8_out ? reinterpret_cast<float*>(empty + NC * S) : nullptr;
  gemv_items<kClass, kDots, kTp>(a, x, ring, full, empty, S, slot, wr0, nwr, NC, warp, lane, n, nullptr, stage,
                                 blk0 * 32);
  if (a.q8_out) {
    // every consumer warp arrives here once (also after a wait gave up)
    asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
    const int rows = a.seg[0].rows;
    for (int b = warp; b < nblk; b += NC) {
      const int r = (blk0 + b) * 32 + lane;
      quant_block_warp(r < rows ? stage[b * 32 + lane] : 0.0f, a.q8_out + (size_t)(blk0 + b) * 36, lane);
    }
  }
#if MCPO_TRACE
  if (tr) {
    asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
    if (threadIdx.x == 0) trace_stamp(tr, 3);
  }
#endif
}

// The same GEMV over a.nvec (2..kGemvMaxVec) input vectors: one x region per
// vector (built with the one-vector prologue), the weights streamed once.
template <int kClass>
__global__ void __launch_bounds__((kMaxConsumers + 1) * 32, 1) k_gemv_multi(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int cols = a.cols;
  const int S = a.stages;
  const int slot = a.slot_bytes;
  const int nvec = a.nvec;
  const size_t xb = gemv_x_bytes(cols);
  const int NC = (int)(blockDim.x >> 5) - 1;
  uint8_t* ring = smem + (size_t)nvec * xb;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)NC * S * slot);
  uint64_t* empty = full + NC * S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.total_wr, G = gridDim.x;
  const int wr0 = (int)((long long)blockIdx.x * T / G);
  const int wr1 = (int)((long long)(blockIdx.x + 1) * T / G);
  const int nwr = wr1 - wr0;
  const int spi = a.seg[0].ks * (a.seg[0].epi == kEpiSwiglu ? 2 : 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NC * S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == NC) {  // producer, as k_gemv
    const int w = lane;
    if (w >= NC) return;
    const int steps = (nwr > w ? (nwr - w + NC - 1) / NC : 0) * spi;
    const uint64_t policy = l2_evict_first_policy();
    for (int n = 0; n < steps; ++n) {
      const int sidx = n % S;
      if (n >= S && !mbar_wait(&empty[w * S + sidx], (uint32_t)((n / S) - 1) & 1u, a.err)) break;
      const int item = n / spi, rem = n % spi, part = rem / a.seg[0].ks, k = rem % a.seg[0].ks;
      const int wr = wr0 + w + NC * item;
      const GemvSeg& sg = seg_of(a, wr);
      const uint8_t* src = (part ? sg.w2 : sg.w) + (size_t)(wr - sg.wr_begin) * sg.wr_bytes + (size_t)k * sg.step_bytes;
      mbar_arrive_expect_tx(&full[w * S + sidx], (uint32_t)sg.step_bytes);
      bulk_load_hint(ring + (size_t)(w * S + sidx) * slot, src, (uint32_t)sg.step_bytes, &full[w * S + sidx], policy);
    }
    for (int n = steps - S > 0 ? steps - S : 0; n < steps; ++n)
      if (!mbar_wait(&full[w * S + n % S], (uint32_t)(n / S) & 1u, a.err)) return;
    return;
  }
  pdl_wait();
  XShared xv[kGemvMaxVec];
  for (int v = 0; v < nvec; ++v) {
    GemvArgs av = a;
    av.xf = a.xf ? a.xf + (size_t)v * a.x_stride : nullptr;
    av.xq = a.xq ? a.xq + (size_t)v * a.xq_stride : nullptr;
    gemv_build_x<false>(av, smem + (size_t)v * xb, NC, warp, lane);
    asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
  }
  for (int v = 0; v < kGemvMaxVec; ++v) xv[v] = gemv_x_view(smem + (size_t)(v < nvec ? v : 0) * xb, cols);
  if (threadIdx.x == 0) pdl_launch_dependents();
  gemv_items_multi<kClass>(a, xv, nvec, ring, full, empty, S, slot, wr0, nwr, NC, warp, lane);
}

// ---------------------------------------------------------------------
// Q8_1 producers
// ---------------------------------------------------------------------


__global__ void k_quantize_q8_1(const float* __restrict__ x, int n, uint8_t* __restrict__ xq) {
  pdl_wait();
  pdl_launch_dependents();
  const int warps = (blockDim.x >> 5) * gridDim.x;
  const int lane = threadIdx.x & 31;
  for (int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n / 32; b += warps)
    quant_block_warp(x[b * 32 + lane], xq + (size_t)b * 36, lane);
}

// RMSNorm with the reduction order of gpu_shim.c:694-718 (blockDim 256):
// lane t sums x[t], x[t+256], ... in order; then a halving tree.  Each CTA
// recomputes the (tiny) sum and then normalises/quantises its share of the
// blocks, so any number of CTAs produce identical bits.
__global__ void __launch_bounds__(256) k_rmsnorm_q8_1(const float* __restrict__ x, const void* __restrict__ w,
                                                      int w_dtype, int n, float eps, float* __restrict__ out,
                                                      uint8_t* __restrict__ xq) {
  __shared__ float part[256];
  __shared__ float inv_s;
  const int t = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  float p = 0.0f;
  for (int i = t; i < n; i += 256) p = __fadd_rn(p, __fmul_rn(x[i], x[i]));
  part[t] = p;
  __syncthreads();
  for (int stride = 128; stride >= 32; stride >>= 1) {
    if (t < stride) part[t] = __fadd_rn(part[t], part[t + stride]);
    __syncthreads();
  }
  if (t < 32) {
    float v = part[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
    if (t == 0) inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)n), eps)));
  }
  __syncthreads();
  const float inv = inv_s;
  const int lane = t & 31;
  const int warps = 8 * gridDim.x;
  for (int b = blockIdx.x * 8 + (t >> 5); b < (n + 31) / 32; b += warps) {
    const int i = b * 32 + lane;
    float v = 0.0f;
    if (i < n) {
      v = __fmul_rn(__fmul_rn(x[i], inv), load_weight(w, w_dtype, i));
      if (out) out[i] = v;
    }
    if (xq && n % 32 == 0) quant_block_warp(v, xq + (size_t)b * 36, lane);
  }
}

// ---------------------------------------------------------------------
// dense GEMV (F32/F16/BF16 rows, f32 activations), warp per row
// ---------------------------------------------------------------------
__global__ void k_dense_gemv(const void* __restrict__ w, int dtype, int rows, int cols, const float* __restrict__ x,
                             float* __restrict__ y) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  if (warp >= rows) return;
  float acc = 0.0f;
  if (dtype == kF32) {
    const float* r = reinterpret_cast<const float*>(w) + (size_t)warp * cols;
    for (int i = lane; i < cols; i += 32) acc = fmaf(r[i], x[i], acc);
  } else {
    const uint16_t* r = reinterpret_cast<const uint16_t*>(w) + (size_t)warp * cols;
    if (dtype == kBF16)
      for (int i = lane; i < cols; i += 32) acc = fmaf(bf16_to_f32(r[i]), x[i], acc);
    else
      for (int i = lane; i < cols; i += 32) acc = fmaf(f16_to_f32(r[i]), x[i], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[warp] = acc;
}

}  // namespace

namespace {
constexpr size_t kGemvSmemBudget = 220 * 1024;

// Tuning overrides (MCPO_GEMV_STAGES: ring slots per consumer warp,
// MCPO_GEMV_CONSUMERS: consumer warps per CTA); read once.
int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : fallback;
}
int stages_cfg() {
  static const int v = env_int("MCPO_GEMV_STAGES", 2);
  return v;
}
int consumers_cfg() {
  static const int v = env_int("MCPO_GEMV_CONSUMERS", 16);
  return v;
}


template <int kClass, bool kDots>
cudaError_t set_smem_attr() {
  cudaError_t e = cudaFuncSetAttribute(k_gemv<kClass, kDots, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       227 * 1024);
  if (e == cudaSuccess && !kDots)
    e = cudaFuncSetAttribute(k_gemv<kClass, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e == cudaSuccess && !kDots)
    e = cudaFuncSetAttribute(k_gemv_multi<kClass>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  return e;
}

template <int kClass>
cudaError_t launch_class(const GemvArgs& a, int grid, int nc, size_t smem, cudaStream_t st, bool pdl) {
  const dim3 block((nc + 1) * 32);
  if (a.nvec > 1) return launch_k(k_gemv_multi<kClass>, dim3(grid), block, smem, st, pdl, a);
  if (a.dots) return launch_k(k_gemv<kClass, true, false>, dim3(grid), block, smem, st, pdl, a);
  if (a.input == kInRmsNormTp || a.seg[0].epi == kEpiTpPush)
    return launch_k(k_gemv<kClass, false, true>, dim3(grid), block, smem, st, pdl, a);
  return launch_k(k_gemv<kClass, false, false>, dim3(grid), block, smem, st, pdl, a);
}
}  // namespace

cudaError_t gemv_init() {
  cudaError_t e = cudaSuccess;
  const cudaError_t r[] = {set_smem_attr<kClassQ4K, false>(), set_smem_attr<kClassQ4K, true>(),
                           set_smem_attr<kClassQ6K, false>(), set_smem_attr<kClassQ6K, true>(),
                           set_smem_attr<kClassQ80, false>(), set_smem_attr<kClassQ80, true>(),
                           set_smem_attr<kClassQ4K6K, false>(), set_smem_attr<kClassQ4K6K, true>()};
  for (cudaError_t x : r)
    if (x != cudaSuccess) e = x;
  return e;
}

size_t gemv_x_bytes_host(int cols) { return gemv_x_bytes(cols); }

cudaError_t gemv_prepare(GemvArgs& a, int* dtypes_mask) {
  int wr = 0, slot = 0, mask = 0;
  if (a.nseg < 1 || a.nseg > kMaxSegs) return cudaErrorInvalidValue;
  for (int i = 0; i < a.nseg; ++i) {
    a.seg[i].wr_begin = wr;
    wr += a.seg[i].n_wr;
    slot = a.seg[i].step_bytes > slot ? a.seg[i].step_bytes : slot;
    mask |= a.seg[i].dtype == kQ4_K ? 1 : a.seg[i].dtype == kQ6_K ? 2 : a.seg[i].dtype == kQ8_0 ? 4 : 8;
    if (a.seg[i].ks != a.seg[0].ks || a.seg[i].lpr != a.seg[0].lpr) return cudaErrorInvalidValue;
  }
  if (a.seg[0].epi == kEpiSwiglu && a.nseg != 1) return cudaErrorInvalidValue;
  const bool norm = a.input == kInRmsNorm || a.input == kInRmsNormTp;
  if (a.input == kInQ8_1 ? !a.xq : (!a.xf || (norm && !a.norm_w) || a.input > kInRmsNormTp))
    return cudaErrorInvalidValue;
  const bool push = a.seg[0].epi == kEpiTpPush;
  for (int i = 1; i < a.nseg; ++i)
    if (a.seg[i].epi == kEpiTpPush) return cudaErrorInvalidValue;
  if ((push || a.input == kInRmsNormTp) &&
      (a.tp.world < 1 || a.tp.world > kTpMaxWorld || (a.tp.world & (a.tp.world - 1)) || a.nvec > 1 || a.dots))
    return cudaErrorInvalidValue;
  if (push && (a.nseg != 1 || a.q8_out)) return cudaErrorInvalidValue;
  if ((push || a.input == kInRmsNormTp) && (!a.tp.step || a.tp.nx < 1 || a.tp.x < 0 || a.tp.x >= a.tp.nx))
    return cudaErrorInvalidValue;
  for (int d = 0; d < a.tp.world; ++d)
    if ((push && !a.tp.dst[d]) || (a.input == kInRmsNormTp && !a.tp.src[d])) return cudaErrorInvalidValue;
  if (a.input == kInRmsNormTp && (!a.tp.sum_out || a.tp.rows != a.cols))
    return cudaErrorInvalidValue;
  if ((mask & 8) || ((mask & 4) && (mask & 3))) return cudaErrorInvalidValue;  // no mixed Q8_0 kernel
  a.total_wr = wr;
  a.slot_bytes = slot;
  if (dtypes_mask) *dtypes_mask = mask;
  return cudaSuccess;
}

cudaError_t launch_gemv(GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
  int mask = 0;
  cudaError_t pe = gemv_prepare(a, &mask);
  if (pe != cudaSuccess) return pe;
  const bool has4 = mask & 1, has6 = mask & 2, has8 = mask & 4;
  const int wr = a.total_wr, slot = a.slot_bytes;
  const int stages = stages_cfg() < 1 ? 1 : stages_cfg();
  a.stages = stages;

  if (wr == 0) return cudaSuccess;
  if (a.nvec > kGemvMaxVec || (a.nvec > 1 && a.dots)) return cudaErrorInvalidValue;
  const size_t xb = a.nvec > 1 ? gemv_x_bytes(a.cols) * (size_t)a.nvec : gemv_x_region(a.cols, a.input);
  const size_t per_warp = (size_t)stages * (slot + 16);
  int nc = kGemvSmemBudget > xb ? (int)((kGemvSmemBudget - xb) / per_warp) : 0;
  const int want = consumers_cfg() > kMaxConsumers ? kMaxConsumers : consumers_cfg();
  nc = nc > want ? want : nc;
  if (nc < 1) return cudaErrorInvalidValue;
  size_t smem = xb + (size_t)nc * stages * slot + (size_t)2 * nc * stages * 8;
  if (grid <= 0 || grid > wr) grid = wr;
  if (a.q8_out) {
    // whole 32-row blocks per CTA: as few CTAs as give every CTA the same
    // largest block count
    const GemvSeg& s0 = a.seg[0];
    if (a.nseg != 1 || a.nvec > 1 || a.dots || s0.rpw < 1 || 32 % s0.rpw != 0) return cudaErrorInvalidValue;
    const int nb = (s0.rows + 31) / 32;
    const int per = (nb + grid - 1) / grid;
    grid = (nb + per - 1) / per;
    smem += (size_t)per * 32 * 4;
    if (smem > (size_t)227 * 1024) return cudaErrorInvalidValue;
  }
  if (has4 && has6) return launch_class<kClassQ4K6K>(a, grid, nc, smem, st, pdl);
  if (has6) return launch_class<kClassQ6K>(a, grid, nc, smem, st, pdl);
  if (has8) return launch_class<kClassQ80>(a, grid, nc, smem, st, pdl);
  return launch_class<kClassQ4K>(a, grid, nc, smem, st, pdl);
}

cudaError_t launch_quantize_q8_1(const float* x, int n, uint8_t* xq, cudaStream_t st, bool pdl) {
  const int blocks = n / 32;
  const int grid = (blocks + 7) / 8;
  return launch_k(k_quantize_q8_1, dim3(grid), dim3(256), 0, st, pdl, x, n, xq);
}

cudaError_t launch_rmsnorm_q8_1(const float* x, const void* w, int w_dtype, int n, float eps, float* out, uint8_t* xq,
                                cudaStream_t st, bool pdl) {
  const int blocks = (n + 31) / 32;
  int grid = (blocks + 7) / 8;
  if (grid > 32) grid = 32;
  return launch_k(k_rmsnorm_q8_1, dim3(grid), dim3(256), 0, st, pdl, x, w, w_dtype, n, eps, out, xq);
}

cudaError_t launch_dense_gemv(const void* w, int dtype, int rows, int cols, const float* x, float* y, cudaStream_t st,
                              bool pdl) {
  const int grid = (rows * 32 + 255) / 256;
  return launch_k(k_dense_gemv, dim3(grid), dim3(256), 0, st, pdl, w, dtype, rows, cols, x, y);
}

}  // namespace mcpo
