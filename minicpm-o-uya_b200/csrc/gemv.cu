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

#include "tma.cuh"

namespace mcpo {

namespace {

// All per-super-block arrays are stored [index within the SB][SB] so that
// the lanes of a row (consecutive SBs) hit consecutive banks.
struct XShared {
  const uint4* xs;    // [16][nb] 16-byte chunks of q8
  const float* xd;    // [8][nb]  d8 of each Q8_1 block (f32 of the f16 d)
  const float* xds;   // [8][nb]  d8 * sum(q8)
  const int* xs16;    // [16][nb] sum(q8) over each 16 values
  int nb;
};

__device__ __forceinline__ int dot4(uint4 w, uint4 x, int acc) {
  acc = dp4a((int)w.x, (int)x.x, acc);
  acc = dp4a((int)w.y, (int)x.y, acc);
  acc = dp4a((int)w.z, (int)x.z, acc);
  acc = dp4a((int)w.w, (int)x.w, acc);
  return acc;
}


// dp4a with the first operand as unsigned bytes (for masked high nibbles /
// bit pairs that reach 0xf0 / 0xc0).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int dot4_mask(uint4 w, uint4 x, uint32_t m, int acc) {
  acc = dp4a_us(w.x & m, x.x, acc);
  acc = dp4a_us(w.y & m, x.y, acc);
  acc = dp4a_us(w.z & m, x.z, acc);
  acc = dp4a_us(w.w & m, x.w, acc);
  return acc;
}

// ---- Q4_K super-block: c[0] = {d, dmin, scales}, c[1..8] = qs ----
// Per sub-block j: dot_j = sum q4*q8 (exact int); the row value is
//   d*sum_j(d8_j*(sc_j*dot_j)) - dmin*sum_j(d8_j*sumq8_j*m_j)
// evaluated as fma chains in j order (see the device-order oracle).
template <bool kDots>
__device__ __forceinline__ float sb_dot_q4k(const uint4* c, const XShared& x, int sb, int* dots) {
  const uint4 h = c[0];
  const float d = f16_to_f32((uint16_t)(h.x & 0xffffu));
  const float dmin = f16_to_f32((uint16_t)(h.x >> 16));
  // 6-bit scales/mins (qwen3.uya:859-867), four at a time per 32-bit word.
  const uint32_t sc_lo = h.y & 0x3f3f3f3fu;
  const uint32_t mn_lo = h.z & 0x3f3f3f3fu;
  const uint32_t sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
  const uint32_t mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
  float sum_d = 0.0f, sum_m = 0.0f;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint4 q0 = c[1 + 2 * g], q1 = c[2 + 2 * g];
    const uint4 x0 = x.xs[(4 * g + 0) * x.nb + sb];
    const uint4 x1 = x.xs[(4 * g + 1) * x.nb + sb];
    const uint4 x2 = x.xs[(4 * g + 2) * x.nb + sb];
    const uint4 x3 = x.xs[(4 * g + 3) * x.nb + sb];
    const int dlo = dot4_mask(q1, x1, 0x0f0f0f0fu, dot4_mask(q0, x0, 0x0f0f0f0fu, 0));
    const int dhi = dot4_mask(q1, x3, 0xf0f0f0f0u, dot4_mask(q0, x2, 0xf0f0f0f0u, 0)) >> 4;
    const int j0 = 2 * g, j1 = 2 * g + 1;
    const uint32_t scw = j0 < 4 ? sc_lo : sc_hi, mnw = j0 < 4 ? mn_lo : mn_hi;
    const int s0 = (scw >> (8 * (j0 & 3))) & 0xff, s1 = (scw >> (8 * (j1 & 3))) & 0xff;
    const int m0 = (mnw >> (8 * (j0 & 3))) & 0xff, m1 = (mnw >> (8 * (j1 & 3))) & 0xff;
    sum_d = __fmaf_rn(x.xd[j0 * x.nb + sb], (float)(s0 * dlo), sum_d);
    sum_d = __fmaf_rn(x.xd[j1 * x.nb + sb], (float)(s1 * dhi), sum_d);
    sum_m = __fmaf_rn(x.xds[j0 * x.nb + sb], (float)m0, sum_m);
    sum_m = __fmaf_rn(x.xds[j1 * x.nb + sb], (float)m1, sum_m);
    if (kDots && dots) {
      dots[sb * 8 + j0] = dlo;
      dots[sb * 8 + j1] = dhi;
    }
  }
  return __fmaf_rn(d, sum_d, -__fmul_rn(dmin, sum_m));
}

// ---- Q6_K super-block: c[0..7] = ql, c[8..11] = qh, c[12] = sc, d separate ----
// Per 16-value group g: dot_g = sum (q6-32)*q8, with q6 = lo4 + 16*hi2 taken
// as two masked dp4a terms; the two groups of a Q8_1 block are combined in
// integers: sum_b(d8_b * (sc_2b*dot_2b + sc_2b+1*dot_2b+1)), then times d.
template <bool kDots>
__device__ __forceinline__ float sb_dot_q6k(const uint4* c, uint16_t dbits, const XShared& x, int sb, int* dots) {
  const float d = f16_to_f32(dbits);
  const uint4 scv = c[12];
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
  float sum = 0.0f;
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      int dg[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int g = 8 * n + 2 * qq + h;
        const uint4 qlw = c[4 * n + ((qq & 1) ? 2 : 0) + h];
        const uint4 qhw = c[8 + 2 * n + h];
        const uint4 xv = x.xs[g * x.nb + sb];
        int lo, hi;
        if (qq == 0) {
          lo = dot4_mask(qlw, xv, 0x0f0f0f0fu, 0);
          hi = dot4_mask(qhw, xv, 0x03030303u, 0) * 16;
        } else if (qq == 1) {
          lo = dot4_mask(qlw, xv, 0x0f0f0f0fu, 0);
          hi = dot4_mask(qhw, xv, 0x0c0c0c0cu, 0) * 4;
        } else if (qq == 2) {
          lo = dot4_mask(qlw, xv, 0xf0f0f0f0u, 0) >> 4;
          hi = dot4_mask(qhw, xv, 0x30303030u, 0);
        } else {
          lo = dot4_mask(qlw, xv, 0xf0f0f0f0u, 0) >> 4;
          hi = dot4_mask(qhw, xv, 0xc0c0c0c0u, 0) >> 2;
        }
        dg[h] = lo + hi - 32 * x.xs16[g * x.nb + sb];
        if (kDots && dots) dots[sb * 16 + g] = dg[h];
      }
      const int g0 = 8 * n + 2 * qq;
      const int sc0 = (int)(int8_t)((scw[g0 >> 2] >> (8 * (g0 & 3))) & 0xff);
      const int sc1 = (int)(int8_t)((scw[(g0 + 1) >> 2] >> (8 * ((g0 + 1) & 3))) & 0xff);
      sum = __fmaf_rn(x.xd[(g0 >> 1) * x.nb + sb], (float)(sc0 * dg[0] + sc1 * dg[1]), sum);
    }
  }
  return __fmul_rn(d, sum);
}

// ---- Q8_0 256-value group: c[0] = 8 f16 d's, c[1..16] = qs ----
template <bool kDots>
__device__ __forceinline__ float sb_dot_q80(const uint4* c, const XShared& x, int sb, int* dots) {
  const uint4 dv = c[0];
  const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
  float sum = 0.0f;
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    int acc = dot4(c[1 + 2 * b], x.xs[(2 * b) * x.nb + sb], 0);
    acc = dot4(c[2 + 2 * b], x.xs[(2 * b + 1) * x.nb + sb], acc);
    const float dwf = f16_to_f32((uint16_t)((dw[b >> 1] >> (16 * (b & 1))) & 0xffffu));
    sum = __fmaf_rn(__fmul_rn(dwf, x.xd[b * x.nb + sb]), (float)acc, sum);
    if (kDots && dots) dots[sb * 8 + b] = acc;
  }
  return sum;
}


// Kernel instantiations by the dtypes they can meet (smaller code per kernel).
enum GemvClass : int { kClassQ4K = 0, kClassQ6K = 1, kClassQ80 = 2, kClassQ4K6K = 3 };

// Value of one super-block for this lane from its step block in shared memory.
template <bool kDots>
__device__ __forceinline__ float step_q4k(const uint8_t* blk, int lane, const XShared& x, int sb, int* dots) {
  uint4 c[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) c[i] = *reinterpret_cast<const uint4*>(blk + i * 512 + lane * 16);
  return sb_dot_q4k<kDots>(c, x, sb, dots);
}

template <bool kDots>
__device__ __forceinline__ float step_q6k(const uint8_t* blk, int lane, const XShared& x, int sb, int* dots) {
  uint4 c[13];
#pragma unroll
  for (int i = 0; i < 13; ++i) c[i] = *reinterpret_cast<const uint4*>(blk + i * 512 + lane * 16);
  const uint16_t db = *reinterpret_cast<const uint16_t*>(blk + 13 * 512 + lane * 2);
  return sb_dot_q6k<kDots>(c, db, x, sb, dots);
}

template <bool kDots>
__device__ __forceinline__ float step_q80(const uint8_t* blk, int lane, const XShared& x, int sb, int* dots) {
  uint4 c[17];
#pragma unroll
  for (int i = 0; i < 17; ++i) c[i] = *reinterpret_cast<const uint4*>(blk + i * 512 + lane * 16);
  return sb_dot_q80<kDots>(c, x, sb, dots);
}

template <int kClass, bool kDots>
__device__ __forceinline__ float step_value(int dtype, const uint8_t* blk, int lane, const XShared& x, int sb,
                                            int* dots) {
  if constexpr (kClass == kClassQ4K) {
    return step_q4k<kDots>(blk, lane, x, sb, dots);
  } else if constexpr (kClass == kClassQ6K) {
    return step_q6k<kDots>(blk, lane, x, sb, dots);
  } else if constexpr (kClass == kClassQ80) {
    return step_q80<kDots>(blk, lane, x, sb, dots);
  } else {
    if (dtype == kQ4_K) return step_q4k<kDots>(blk, lane, x, sb, dots);
    return step_q6k<kDots>(blk, lane, x, sb, dots);
  }
}

// Butterfly over the lpr lanes of a row (xor lpr/2 .. 1); the row's value is
// the one of its first lane.
__device__ __forceinline__ float reduce_row(float v, int lpr) {
  for (int o = lpr >> 1; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ const GemvSeg& seg_of(const GemvArgs& a, int wr) {
  if (a.nseg > 2 && wr >= a.seg[2].wr_begin) return a.seg[2];
  if (a.nseg > 1 && wr >= a.seg[1].wr_begin) return a.seg[1];
  return a.seg[0];
}

constexpr int kMaxConsumers = 16;  // consumer warps per CTA (+1 producer warp)

// x region: xs, xd, xds, xs16, then 256 floats + 1 of RMSNorm reduction space.
__host__ __device__ inline size_t gemv_x_bytes(int cols) {
  const size_t b = (size_t)cols + (size_t)(cols / 32) * 8 + (size_t)(cols / 16) * 4 + 257 * 4;
  return (b + 127) / 128 * 128;
}

// Writes one Q8_1 block (32 values, one per lane) straight into the
// transposed shared-memory layout: the quants and d of q8_1_quant_lane (the
// bits k_quantize_q8_1 stores), and the exact integer sums of each half.
__device__ __forceinline__ void x_block_from_f32(float v, int b, int nb, int lane, uint4* xs, float* xd, float* xds,
                                                 int* xs16) {
  uint16_t dbits;
  bool zero;
  const int q = q8_1_quant_lane(v, &dbits, &zero);
  const int sb = b >> 3, j = b & 7, c = j * 2;
  // quant byte straight into its 16-byte chunk: chunk c holds values 0..15
  reinterpret_cast<int8_t*>(xs + (size_t)(c + (lane >> 4)) * nb + sb)[lane & 15] = (int8_t)q;
  const int s_lo = __reduce_add_sync(0xffffffffu, lane < 16 ? q : 0);
  const int s_hi = __reduce_add_sync(0xffffffffu, lane < 16 ? 0 : q);
  if (lane == 0) {
    const float d8 = f16_to_f32(dbits);
    xd[j * nb + sb] = d8;
    xds[j * nb + sb] = __fmul_rn(d8, (float)(s_lo + s_hi));
    xs16[c * nb + sb] = s_lo;
    xs16[(c + 1) * nb + sb] = s_hi;
  }
}

template <int kClass, bool kDots>
__global__ void __launch_bounds__((kMaxConsumers + 1) * 32, 1) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int cols = a.cols;
  const int nb = cols / 256;
  const int nblk = cols / 32;
  uint4* xs = reinterpret_cast<uint4*>(smem);
  float* xd = reinterpret_cast<float*>(smem + cols);
  float* xds = xd + nblk;
  int* xs16 = reinterpret_cast<int*>(xds + nblk);
  const int S = a.stages;
  const int slot = a.slot_bytes;
  const int NC = (int)(blockDim.x >> 5) - 1;  // consumer warps; the last warp produces
  uint8_t* ring = smem + gemv_x_bytes(cols);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)NC * S * slot);
  uint64_t* empty = full + NC * S;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.total_wr, G = gridDim.x;
  const int wr0 = (int)((long long)blockIdx.x * T / G);
  const int wr1 = (int)((long long)(blockIdx.x + 1) * T / G);
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
  pdl_wait();  // the activations (and y for the residual add) come from earlier kernels
  const int nthr = NC * 32;
  if (a.input == kInQ8_1) {
    for (int b = threadIdx.x; b < nblk; b += nthr) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(a.xq + (size_t)b * 36);
      const uint32_t hdr = src[0];
      uint32_t q[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = src[1 + i];
      int s_lo = 0, s_hi = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) s_lo = dp4a((int)q[i], 0x01010101, s_lo);
#pragma unroll
      for (int i = 4; i < 8; ++i) s_hi = dp4a((int)q[i], 0x01010101, s_hi);
      const float d8 = f16_to_f32((uint16_t)(hdr & 0xffffu));
      const int sb = b >> 3, j = b & 7, c = j * 2;
      xd[j * nb + sb] = d8;
      xds[j * nb + sb] = __fmul_rn(d8, (float)(s_lo + s_hi));
      xs16[c * nb + sb] = s_lo;
      xs16[(c + 1) * nb + sb] = s_hi;
      xs[c * nb + sb] = make_uint4(q[0], q[1], q[2], q[3]);
      xs[(c + 1) * nb + sb] = make_uint4(q[4], q[5], q[6], q[7]);
    }
  } else {
    // f32 input: every load is issued before the arithmetic that needs it
    // (batches of kXB blocks per warp), so the prologue costs about two L2
    // round trips instead of one per block.
    constexpr int kXB = 8;
    const float* xf = a.xf;
    const bool norm = a.input == kInRmsNorm;
    float v[kXB], wv[kXB];
    auto load_batch = [&](int b0) {
#pragma unroll
      for (int u = 0; u < kXB; ++u) {
        const int b = b0 + u * NC;
        if (b < nblk) {
          v[u] = xf[b * 32 + lane];
          wv[u] = norm ? load_weight(a.norm_w, a.norm_dtype, b * 32 + lane) : 1.0f;
        }
      }
    };
    load_batch(warp);
    float inv = 1.0f;
    if (norm) {
      // sum of squares in k_rmsnorm_q8_1's order: 256 strided partial sums
      // (each sequential in i), a halving tree, then a warp tree
      float* red = reinterpret_cast<float*>(xs16 + cols / 16);
      const int per = cols / 256;
      for (int t = threadIdx.x; t < 256; t += nthr) {
        float p = 0.0f;
        int k = 0;
        for (; k + 8 <= per; k += 8) {
          float r[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) r[u] = xf[t + 256 * (k + u)];
#pragma unroll
          for (int u = 0; u < 8; ++u) p = __fadd_rn(p, __fmul_rn(r[u], r[u]));
        }
        for (; k < per; ++k) {
          const float r = xf[t + 256 * k];
          p = __fadd_rn(p, __fmul_rn(r, r));
        }
        red[t] = p;
      }
      for (int stride = 128; stride >= 32; stride >>= 1) {
        asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
        for (int t = threadIdx.x; t < stride; t += nthr) red[t] = __fadd_rn(red[t], red[t + stride]);
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
      if (warp == 0) {
        float r = red[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) r = __fadd_rn(r, __shfl_down_sync(0xffffffffu, r, o));
        if (lane == 0) red[256] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(r, (float)cols), a.eps)));
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
      inv = red[256];
    }
    for (int b0 = warp; b0 < nblk; b0 += NC * kXB) {
      if (b0 != warp) load_batch(b0);
#pragma unroll
      for (int u = 0; u < kXB; ++u) {
        const int b = b0 + u * NC;
        if (b < nblk) {
          const float x = norm ? __fmul_rn(__fmul_rn(v[u], inv), wv[u]) : v[u];
          x_block_from_f32(x, b, nb, lane, xs, xd, xds, xs16);
        }
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
  if (threadIdx.x == 0) pdl_launch_dependents();
  const XShared x{xs, xd, xds, xs16, nb};

  const int items = nwr > warp ? (nwr - warp + NC - 1) / NC : 0;
  int n = 0;
  for (int item = 0; item < items; ++item) {
    const int wr = wr0 + warp + NC * item;
    const GemvSeg s = seg_of(a, wr);
    const int local = wr - s.wr_begin;
    const int row_in_warp = lane / s.lpr, lane_in_row = lane % s.lpr;
    const int row = local * s.rpw + row_in_warp;
    int* dots = nullptr;
    if (kDots && row < s.rows) dots = a.dots + (size_t)row * (s.dtype == kQ6_K ? cols / 16 : cols / 32);
    float acc[2] = {0.0f, 0.0f};
    for (int part = 0; part < (swiglu ? 2 : 1); ++part) {
      for (int k = 0; k < ks; ++k, ++n) {
        const int sidx = n % S;
        if (!mbar_wait(&full[warp * S + sidx], (uint32_t)(n / S) & 1u, a.err)) return;
        const uint8_t* blk = ring + (size_t)(warp * S + sidx) * slot;
        const float v =
            step_value<kClass, kDots>(s.dtype, blk, lane, x, k * s.lpr + lane_in_row, part == 0 ? dots : nullptr);
        acc[part] = __fadd_rn(acc[part], v);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[warp * S + sidx]);
      }
    }
    const float g = reduce_row(acc[0], s.lpr);
    if (swiglu) {
      const float u = reduce_row(acc[1], s.lpr);
      if (lane_in_row == 0 && row < s.rows) s.y[row] = silu_mul_det(g, u);
    } else if (lane_in_row == 0 && row < s.rows) {
      if (s.epi == kEpiAdd)
        s.y[row] = __fadd_rn(s.y[row], g);
      else
        s.y[row] = g;
    }
  }
}

// ---------------------------------------------------------------------
// Q8_1 producers
// ---------------------------------------------------------------------

// One warp per 32-value block; writes the reference's 36-byte block with the
// sequential f16 sum s (gpu_shim.c:343-378).
__device__ __forceinline__ void quant_block_warp(float v, uint8_t* dst, int lane) {
  uint16_t dbits;
  bool zero;
  const int q = q8_1_quant_lane(v, &dbits, &zero);
  const float s = warp_seq_sum(v);
  const uint16_t sbits = zero ? (uint16_t)0 : f32_to_f16_ref(s);
  // pack 4 quants per lane group into words
  const uint32_t qb = (uint32_t)(q & 0xff);
  uint32_t word = qb << (8 * (lane & 3));
  word |= __shfl_xor_sync(0xffffffffu, word, 1);
  word |= __shfl_xor_sync(0xffffffffu, word, 2);
  uint32_t* o = reinterpret_cast<uint32_t*>(dst);
  if (lane == 0) o[0] = (uint32_t)dbits | ((uint32_t)sbits << 16);
  if ((lane & 3) == 0) o[1 + (lane >> 2)] = word;
}

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
  return cudaFuncSetAttribute(k_gemv<kClass, kDots>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

template <int kClass>
cudaError_t launch_class(const GemvArgs& a, int grid, int nc, size_t smem, cudaStream_t st, bool pdl) {
  const dim3 block((nc + 1) * 32);
  if (a.dots) return launch_k(k_gemv<kClass, true>, dim3(grid), block, smem, st, pdl, a);
  return launch_k(k_gemv<kClass, false>, dim3(grid), block, smem, st, pdl, a);
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

cudaError_t launch_gemv(GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
  int wr = 0, slot = 0;
  bool has4 = false, has6 = false, has8 = false;
  for (int i = 0; i < a.nseg; ++i) {
    a.seg[i].wr_begin = wr;
    wr += a.seg[i].n_wr;
    slot = a.seg[i].step_bytes > slot ? a.seg[i].step_bytes : slot;
    has4 |= a.seg[i].dtype == kQ4_K;
    has6 |= a.seg[i].dtype == kQ6_K;
    has8 |= a.seg[i].dtype == kQ8_0;
    if (a.seg[i].ks != a.seg[0].ks || a.seg[i].lpr != a.seg[0].lpr) return cudaErrorInvalidValue;
  }
  if (a.seg[0].epi == kEpiSwiglu && a.nseg != 1) return cudaErrorInvalidValue;
  if (a.input == kInQ8_1 ? !a.xq : (!a.xf || (a.input == kInRmsNorm && !a.norm_w) || a.input > kInRmsNorm))
    return cudaErrorInvalidValue;
  if (has8 && (has4 || has6)) return cudaErrorInvalidValue;  // no mixed Q8_0 kernel
  a.total_wr = wr;
  a.slot_bytes = slot;
  const int stages = stages_cfg() < 1 ? 1 : stages_cfg();
  a.stages = stages;
  if (wr == 0) return cudaSuccess;
  const size_t xb = gemv_x_bytes(a.cols);
  const size_t per_warp = (size_t)stages * (slot + 16);
  int nc = kGemvSmemBudget > xb ? (int)((kGemvSmemBudget - xb) / per_warp) : 0;
  const int want = consumers_cfg() > kMaxConsumers ? kMaxConsumers : consumers_cfg();
  nc = nc > want ? want : nc;
  if (nc < 1) return cudaErrorInvalidValue;
  const size_t smem = xb + (size_t)nc * stages * slot + (size_t)2 * nc * stages * 8;
  if (grid <= 0 || grid > wr) grid = wr;
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
