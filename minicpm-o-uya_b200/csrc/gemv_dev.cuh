// gemv_dev.cuh -- device building blocks of the quantised GEMV, shared by
// the standalone GEMV kernel and the persistent decode-step kernel:
// super-block dot products on a step block in shared memory, the activation
// prologue (Q8_1 input, or f32 input quantised here, optionally after
// RMSNorm) and the consumer loop over a CTA's warp-rows.
#pragma once

#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"
#include "tp_proto.h"

namespace mcpo {

// All per-super-block arrays are stored [index within the SB][SB] so that
// the lanes of a row (consecutive SBs) hit consecutive banks.
struct XShared {
  const uint4* xs;    // [16][nb] 16-byte chunks of q8
  const float* xd;    // [8][nb]  d8 of each Q8_1 block (f32 of the f16 d)
  const float* xds;   // [8][nb]  d8 * sum(q8)
  const int* xs16;    // [16][nb] sum(q8) over each 16 values
  int nb;
};

// Integer dot products are exact, so the four dp4a run as two independent
// pairs (shorter dependency chains) and are added at the end.
__device__ __forceinline__ int dot4(uint4 w, uint4 x, int acc) {
  const int a0 = dp4a((int)w.y, (int)x.y, dp4a((int)w.x, (int)x.x, 0));
  const int a1 = dp4a((int)w.w, (int)x.w, dp4a((int)w.z, (int)x.z, 0));
  return acc + a0 + a1;
}


// dp4a with the first operand as unsigned bytes (for masked high nibbles /
// bit pairs that reach 0xf0 / 0xc0).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int dot4_mask(uint4 w, uint4 x, uint32_t m, int acc) {
  const int a0 = dp4a_us(w.y & m, x.y, dp4a_us(w.x & m, x.x, 0));
  const int a1 = dp4a_us(w.w & m, x.w, dp4a_us(w.z & m, x.z, 0));
  return acc + a0 + a1;
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
    const int dlo = dot4_mask(q0, x0, 0x0f0f0f0fu, 0) + dot4_mask(q1, x1, 0x0f0f0f0fu, 0);
    const int dhi = (dot4_mask(q0, x2, 0xf0f0f0f0u, 0) + dot4_mask(q1, x3, 0xf0f0f0f0u, 0)) >> 4;
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
    const int acc = dot4(c[1 + 2 * b], x.xs[(2 * b) * x.nb + sb], 0) + dot4(c[2 + 2 * b], x.xs[(2 * b + 1) * x.nb + sb], 0);
    const float dwf = f16_to_f32((uint16_t)((dw[b >> 1] >> (16 * (b & 1))) & 0xffffu));
    sum = __fmaf_rn(__fmul_rn(dwf, x.xd[b * x.nb + sb]), (float)acc, sum);
    if (kDots && dots) dots[sb * 8 + b] = acc;
  }
  return sum;
}


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

// The activation region of one launch: the x region, plus the summed input
// vector (f32) of a tensor-parallel summing prologue.
__host__ __device__ inline size_t gemv_x_region(int cols, int input) {
  return gemv_x_bytes(cols) + (input == kInRmsNormTp ? ((size_t)cols * 4 + 127) / 128 * 128 : 0);
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t gemv_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The tensor-parallel summing prologue: the NC*32 consumer threads write
// sx[i] = xf[i] + rank-order sum of the partials, each value once every
// rank's tagged word of it has arrived (bounded wait, 1 s), and this CTA's
// share of sx to tp.sum_out.  Ends with the consumers synchronised.
__device__ __forceinline__ void gemv_tp_sum(const GemvArgs& a, float* sx, int tid, int nthr) {
  const TpXchg& t = a.tp;
  const uint32_t tag = tp_xchg_tag(t, *t.step);
  const uint64_t deadline = tp_now_ns() + 1000000000ull;
  bool ok = true;
  const int cols = a.cols;
  // tp_rank_sum: base + (p_0 + ... + p_{world-1})
  tp_gather_sums(t, tag, tid, nthr, cols, deadline, &ok, [&](int i, float s) { sx[i] = a.xf[i] + s; });
  if (!ok && a.err) atomicExch(a.err, 1);
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  const int G = gridDim.x, b = blockIdx.x;
  const int lo = (int)((long long)cols * b / G), hi = (int)((long long)cols * (b + 1) / G);
  for (int i = lo + tid; i < hi; i += nthr) t.sum_out[i] = sx[i];
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

// kB blocks b0, b0 + stride, ... (those < nblk) at once, with the
// arithmetic of q8_1_quant_lane: each phase runs for all kB blocks before the
// next, so the blocks' dependency chains (reductions, IEEE divisions)
// overlap instead of running back to back.
template <int kB>
__device__ __forceinline__ void x_blocks_from_f32(const float (&x)[kB], int b0, int stride, int nblk, int nb, int lane,
                                                  uint4* xs, float* xd, float* xds, int* xs16) {
  float amax[kB], d[kB];
  int q[kB];
#pragma unroll
  for (int u = 0; u < kB; ++u) {
    const float ax = fabsf(x[u]);
    amax[u] = __uint_as_float(__reduce_max_sync(0xffffffffu, ax == ax ? __float_as_uint(ax) : 0u));
  }
#pragma unroll
  for (int u = 0; u < kB; ++u) d[u] = __fdiv_rn(amax[u], 127.0f);
#pragma unroll
  for (int u = 0; u < kB; ++u) {
    float t = __fmul_rn(x[u], __frcp_rn(d[u]));
    const float at = fabsf(t);
    if (!(fabsf(__fsub_rn(__fsub_rn(at, floorf(at)), 0.5f)) >= 1e-4f)) t = __fdiv_rn(x[u], d[u]);
    int qq = __float2int_rz(t >= 0.0f ? __fadd_rn(t, 0.5f) : __fsub_rn(t, 0.5f));
    qq = qq > 127 ? 127 : (qq < -128 ? -128 : qq);
    q[u] = amax[u] == 0.0f ? 0 : qq;
  }
#pragma unroll
  for (int u = 0; u < kB; ++u) {
    const int b = b0 + u * stride;
    if (b < nblk) {
      const int sb = b >> 3, j = b & 7, c = j * 2;
      reinterpret_cast<int8_t*>(xs + (size_t)(c + (lane >> 4)) * nb + sb)[lane & 15] = (int8_t)q[u];
      const int s_lo = __reduce_add_sync(0xffffffffu, lane < 16 ? q[u] : 0);
      const int s_hi = __reduce_add_sync(0xffffffffu, lane < 16 ? 0 : q[u]);
      if (lane == 0) {
        const float d8 = amax[u] == 0.0f ? 0.0f : f16_to_f32(f32_to_f16_ref(d[u]));
        xd[j * nb + sb] = d8;
        xds[j * nb + sb] = __fmul_rn(d8, (float)(s_lo + s_hi));
        xs16[c * nb + sb] = s_lo;
        xs16[(c + 1) * nb + sb] = s_hi;
      }
    }
  }
}

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// One Q8_1 block (32 values held by ONE thread) into the transposed
// shared-memory layout, with the arithmetic of q8_1_quant_lane per element:
// d = amax/127 (IEEE division), q = trunc(x/d +- 0.5) clamped to
// [-128, 127].  x/d is taken as x*rcp(d) except within 2.5e-4 of a
// half-integer, where the exact quotient decides: for |x/d| <= 128 the
// product is within 7e-5 of the correctly rounded quotient (approximate
// reciprocal, relative error < 2^-21, plus two roundings), and trunc(v +-
// 0.5) only changes within 2^-17 of a half-integer.
__device__ __forceinline__ int q8_round(float t) {
  const int q = __float2int_rz(t >= 0.0f ? __fadd_rn(t, 0.5f) : __fsub_rn(t, 0.5f));
  return q > 127 ? 127 : (q < -128 ? -128 : q);
}

__device__ __forceinline__ void x_block_quarter(const float (&v)[8], int b, int nblk, int part, int nb, uint4* xs,
                                                float* xd, float* xds, int* xs16) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float ax = fabsf(v[i]);
    amax = ax > amax ? ax : amax;  // NaN never wins (the reference's scan)
  }
  float o = __shfl_xor_sync(0xffffffffu, amax, 1);
  amax = o > amax ? o : amax;
  o = __shfl_xor_sync(0xffffffffu, amax, 2);
  amax = o > amax ? o : amax;
  const float d = __fdiv_rn(amax, 127.0f);
  const float r = rcp_approx(d);
  // fast pass: x*rcp(d); elements near a rounding boundary are flagged and
  // redone with the exact quotient outside the loop (no division on the
  // common path)
  uint32_t w[2];
  uint32_t near = 0;
  int sum = 0;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * k + e;
      const float t = __fmul_rn(v[i], r);
      const float at = fabsf(t);
      if (!(fabsf(__fsub_rn(__fsub_rn(at, floorf(at)), 0.5f)) >= 2.5e-4f)) near |= 1u << i;
      const int q = amax == 0.0f ? 0 : q8_round(t);
      word |= (uint32_t)(q & 0xff) << (8 * e);
      sum += q;
    }
    w[k] = word;
  }
  if (near && amax != 0.0f) {  // rare: one value in ~2000
#pragma unroll
    for (int k = 0; k < 2; ++k) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if ((near >> (4 * k + e)) & 1u) {
          const int qn = q8_round(__fdiv_rn(v[4 * k + e], d));
          const int qo = (int)(int8_t)((w[k] >> (8 * e)) & 0xffu);
          w[k] = (w[k] & ~(0xffu << (8 * e))) | ((uint32_t)(qn & 0xff) << (8 * e));
          sum += qn - qo;
        }
      }
    }
  }
  // parts 0,1 hold values 0..15, parts 2,3 values 16..31
  const int half = sum + __shfl_xor_sync(0xffffffffu, sum, 1);
  const int other = __shfl_xor_sync(0xffffffffu, half, 2);
  if (b < nblk) {
    const int sb = b >> 3, j = b & 7, c = j * 2;
    reinterpret_cast<uint2*>(xs + (size_t)(c + (part >> 1)) * nb + sb)[part & 1] = make_uint2(w[0], w[1]);
    if (part == 0) {
      const float d8 = amax == 0.0f ? 0.0f : f16_to_f32(f32_to_f16_ref(d));
      xd[j * nb + sb] = d8;
      xds[j * nb + sb] = __fmul_rn(d8, (float)(half + other));
      xs16[c * nb + sb] = half;
      xs16[(c + 1) * nb + sb] = other;
    }
  }
}

// Builds this CTA's shared-memory copy of the activations (the x region at
// xbase, gemv_x_bytes(cols) bytes) from a's input: Q8_1 blocks, or f32 values
// quantised here, optionally after RMSNorm.  Called by the NC consumer warps
// (thread tid = warp*32 + lane); uses named barrier 1 for those NC*32
// threads and ends without a barrier (the caller synchronises).
// The RMSNorm weights of this thread's first activation tile (the weights
// do not depend on earlier kernels, so they can be requested before the
// wait for them); zeros for other inputs.
__device__ __forceinline__ void gemv_norm_weights(const GemvArgs& a, int warp, int lane, float (&wv)[8]) {
  const int nblk = a.cols / 32;
  const int b = warp * 8 + (lane >> 2);
  const bool on = (a.input == kInRmsNorm || a.input == kInRmsNormTp) && b < nblk;
#pragma unroll
  for (int i = 0; i < 8; ++i) wv[i] = on ? load_weight(a.norm_w, a.norm_dtype, b * 32 + (lane & 3) * 8 + i) : 0.0f;
}

// wpre: the weights gemv_norm_weights gave (null: loaded here).  kTp: the
// input may be the tensor-parallel sum (kInRmsNormTp).
template <bool kTp = false>
__device__ __forceinline__ void gemv_build_x(const GemvArgs& a, uint8_t* xbase, int NC, int warp, int lane,
                                             const float* wpre = nullptr) {
  const int cols = a.cols;
  const int nb = cols / 256;
  const int nblk = cols / 32;
  const int tid = warp * 32 + lane;
  uint4* xs = reinterpret_cast<uint4*>(xbase);
  float* xd = reinterpret_cast<float*>(xbase + cols);
  float* xds = xd + nblk;
  int* xs16 = reinterpret_cast<int*>(xds + nblk);
  const int nthr = NC * 32;
  if (a.input == kInQ8_1) {
    for (int b = tid; b < nblk; b += nthr) {
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
    // f32 input: four lanes per 32-value block, eight values each (a warp
    // covers 8 consecutive blocks, 1 KB of coalesced loads).  A warp's tiles
    // (up to three; with RMSNorm one) are all requested at once, before the
    // RMSNorm reduction; larger inputs request each tile while the one
    // before it is quantised.  Arithmetic per element as q8_1_quant_lane.
    // The tensor-parallel input is first summed into shared memory.
    const float* xf = a.xf;
    if constexpr (kTp) {
      if (a.input == kInRmsNormTp) {
        float* sx = reinterpret_cast<float*>(xbase + gemv_x_bytes(cols));
        gemv_tp_sum(a, sx, tid, NC * 32);
        xf = sx;
      }
    }
    const bool norm = a.input == kInRmsNorm || (kTp && a.input == kInRmsNormTp);
    const void* nw = a.norm_w;
    const int ndt = a.norm_dtype;
    const float eps = a.eps;
    const int part = lane & 3;
    const int ntile = (nblk + 7) / 8;
    // all of a warp's tiles requested at once: up to two with RMSNorm
    // (their weights in wv, wv1), three without
    const bool at_once = norm ? ntile <= 2 * NC : ntile <= 3 * NC;
    float xv[3][8], wv[8], wv1[8];
    auto load_x = [&](int tile, float (&dst)[8]) {
      const int b = tile * 8 + (lane >> 2);
      if (b < nblk) {
        const float4* src = reinterpret_cast<const float4*>(xf + (size_t)b * 32 + part * 8);
        const float4 t0 = src[0], t1 = src[1];
        dst[0] = t0.x; dst[1] = t0.y; dst[2] = t0.z; dst[3] = t0.w;
        dst[4] = t1.x; dst[5] = t1.y; dst[6] = t1.z; dst[7] = t1.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = 0.0f;
      }
    };
    auto load_w = [&](int tile, float (&dst)[8]) {
      const int b = tile * 8 + (lane >> 2);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = b < nblk ? load_weight(nw, ndt, b * 32 + part * 8 + i) : 0.0f;
    };
    if (at_once) {
#pragma unroll
      for (int u = 0; u < 3; ++u)
        if (warp + u * NC < ntile) load_x(warp + u * NC, xv[u]);
    } else if (warp < ntile) {
      load_x(warp, xv[0]);
    }
    if (norm && warp < ntile) {
      if (wpre) {
#pragma unroll
        for (int i = 0; i < 8; ++i) wv[i] = wpre[i];
      } else {
        load_w(warp, wv);
      }
      if (at_once && warp + NC < ntile) load_w(warp + NC, wv1);
    }
    float inv = 1.0f;
    if (norm) {
      // sum of squares in k_rmsnorm_q8_1's order: 256 strided partial sums
      // (each sequential in i), a halving tree (strides 128, 64, 32), then a
      // warp tree -- the trees computed by every warp from the partials in
      // registers (lane l adds partials l + 32k in the halving order)
      float* red = reinterpret_cast<float*>(xs16 + cols / 16);
      const int per = cols / 256;
      for (int t = tid; t < 256; t += nthr) {
        float p = 0.0f;
        int k = 0;
        for (; k + 16 <= per; k += 16) {
          float r[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) r[u] = xf[t + 256 * (k + u)];
#pragma unroll
          for (int u = 0; u < 16; ++u) p = __fadd_rn(p, __fmul_rn(r[u], r[u]));
        }
        for (; k < per; ++k) {
          const float r = xf[t + 256 * k];
          p = __fadd_rn(p, __fmul_rn(r, r));
        }
        red[t] = p;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
      float q[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = red[lane + 32 * k];
      float r = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[4]), __fadd_rn(q[2], q[6])),
                          __fadd_rn(__fadd_rn(q[1], q[5]), __fadd_rn(q[3], q[7])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) r = __fadd_rn(r, __shfl_down_sync(0xffffffffu, r, o));
      r = __shfl_sync(0xffffffffu, r, 0);
      inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(r, (float)cols), eps)));
    }
    if (at_once) {
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const int tile = warp + u * NC;
        if (tile < ntile) {
          float x[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = norm ? __fmul_rn(__fmul_rn(xv[u][i], inv), u == 0 ? wv[i] : wv1[i]) : xv[u][i];
          x_block_quarter(x, tile * 8 + (lane >> 2), nblk, part, nb, xs, xd, xds, xs16);
        }
      }
    } else {
      for (int tile = warp; tile < ntile; tile += NC) {
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = norm ? __fmul_rn(__fmul_rn(xv[0][i], inv), wv[i]) : xv[0][i];
        if (tile + NC < ntile) {
          load_x(tile + NC, xv[0]);
          if (norm) load_w(tile + NC, wv);
        }
        x_block_quarter(x, tile * 8 + (lane >> 2), nblk, part, nb, xs, xd, xds, xs16);
      }
    }
  }
}

__device__ __forceinline__ XShared gemv_x_view(uint8_t* xbase, int cols) {
  const int nblk = cols / 32;
  float* xd = reinterpret_cast<float*>(xbase + cols);
  return XShared{reinterpret_cast<const uint4*>(xbase), xd, xd + nblk, reinterpret_cast<const int*>(xd + 2 * nblk),
                 cols / 256};
}

// The consumer loop of one GEMV over warp-rows [wr0, wr0 + nwr) of a CTA:
// warp `warp` of NC takes items warp, warp + NC, ...; its step blocks arrive
// in order in its ring (S slots of `slot` bytes; full/empty mbarriers), n
// counting the blocks this warp has consumed so far.  Returns false when a
// wait gave up (error raised) or *abort was set.
// kTp: outputs of a push epilogue (kEpiTpPush) go to every rank's exchange
// slot instead of y.
template <int kClass, bool kDots, bool kTp = false>
__device__ __forceinline__ bool gemv_items(const GemvArgs& a, const XShared& x, uint8_t* ring, uint64_t* full,
                                           uint64_t* empty, int S, int slot, int wr0, int nwr, int NC, int warp,
                                           int lane, int& n, const volatile int* abort, float* stage = nullptr,
                                           int stage_r0 = 0) {
  const int cols = a.cols;
  const bool swiglu = a.seg[0].epi == kEpiSwiglu;
  const int ks = a.seg[0].ks;
  const int items = nwr > warp ? (nwr - warp + NC - 1) / NC : 0;
  uint32_t tag = 0;
  if constexpr (kTp) {
    if (a.seg[0].epi == kEpiTpPush) tag = tp_xchg_tag(a.tp, *a.tp.step);
  }
  for (int item = 0; item < items; ++item) {
    const int wr = wr0 + warp + NC * item;
    const GemvSeg s = seg_of(a, wr);
    const int local = wr - s.wr_begin;
    const int row_in_warp = lane / s.lpr, lane_in_row = lane % s.lpr;
    const int row = local * s.rpw + row_in_warp;
    int* dots = nullptr;
    if (kDots && row < s.rows) dots = a.dots + (size_t)row * (s.dtype == kQ6_K ? cols / 16 : cols / 32);
    // residual add: the old value is requested before the dot products
    const bool add = !swiglu && s.epi == kEpiAdd && lane_in_row == 0 && row < s.rows;
    const float yold = add ? s.y[row] : 0.0f;
    float acc[2] = {0.0f, 0.0f};
    for (int part = 0; part < (swiglu ? 2 : 1); ++part) {
      for (int k = 0; k < ks; ++k, ++n) {
        const int sidx = n % S;
        if (abort ? !mbar_wait_abort(&full[warp * S + sidx], (uint32_t)(n / S) & 1u, a.err, abort)
                  : !mbar_wait_sleep(&full[warp * S + sidx], (uint32_t)(n / S) & 1u, a.err))
          return false;
        const uint8_t* blk = ring + (size_t)(warp * S + sidx) * slot;
        const float v =
            step_value<kClass, kDots>(s.dtype, blk, lane, x, k * s.lpr + lane_in_row, part == 0 ? dots : nullptr);
        acc[part] = __fadd_rn(acc[part], v);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[warp * S + sidx]);
      }
    }
    const float g = reduce_row(acc[0], s.lpr);
    // (every lane takes part in both butterflies)
    const float u = swiglu ? reduce_row(acc[1], s.lpr) : 0.0f;
    if (lane_in_row == 0 && row < s.rows) {
      const float out = swiglu ? silu_mul_det(g, u) : add ? __fadd_rn(yold, g) : g;
      if constexpr (kTp) {
        if (s.epi == kEpiTpPush) {
          // this rank's slot on every rank, the value with the exchange's tag
          const uint64_t w = tp_ll_pack(__float_as_uint(out), tag);
          for (int d = 0; d < a.tp.world; ++d) tp_st_word(a.tp.dst[d] + row, w);
        } else {
          s.y[row] = out;
          if (stage) stage[row - stage_r0] = out;
        }
      } else {
        s.y[row] = out;
        if (stage) stage[row - stage_r0] = out;
      }
    }
  }
  return true;
}

// gemv_items over nvec (<= kGemvMaxVec) input vectors: each step block is
// dotted with every vector (the same step_value per vector as the one-vector
// loop, so every vector's rows get the bits a one-vector launch gives).
template <int kClass>
__device__ __forceinline__ bool gemv_items_multi(const GemvArgs& a, const XShared* xv, int nvec, uint8_t* ring,
                                                 uint64_t* full, uint64_t* empty, int S, int slot, int wr0, int nwr,
                                                 int NC, int warp, int lane) {
  const bool swiglu = a.seg[0].epi == kEpiSwiglu;
  const int ks = a.seg[0].ks;
  const int items = nwr > warp ? (nwr - warp + NC - 1) / NC : 0;
  int n = 0;
  for (int item = 0; item < items; ++item) {
    const int wr = wr0 + warp + NC * item;
    const GemvSeg s = seg_of(a, wr);
    const int local = wr - s.wr_begin;
    const int row_in_warp = lane / s.lpr, lane_in_row = lane % s.lpr;
    const int row = local * s.rpw + row_in_warp;
    const bool add = !swiglu && s.epi == kEpiAdd && lane_in_row == 0 && row < s.rows;
    float yold[kGemvMaxVec];
#pragma unroll
    for (int v = 0; v < kGemvMaxVec; ++v) yold[v] = add && v < nvec ? s.y[(size_t)v * a.y_stride + row] : 0.0f;
    float acc[kGemvMaxVec][2];
#pragma unroll
    for (int v = 0; v < kGemvMaxVec; ++v) acc[v][0] = acc[v][1] = 0.0f;
    for (int part = 0; part < (swiglu ? 2 : 1); ++part) {
      for (int k = 0; k < ks; ++k, ++n) {
        const int sidx = n % S;
        if (!mbar_wait_sleep(&full[warp * S + sidx], (uint32_t)(n / S) & 1u, a.err)) return false;
        const uint8_t* blk = ring + (size_t)(warp * S + sidx) * slot;
#pragma unroll
        for (int v = 0; v < kGemvMaxVec; ++v)
          if (v < nvec)
            acc[v][part] = __fadd_rn(acc[v][part],
                                     step_value<kClass, false>(s.dtype, blk, lane, xv[v], k * s.lpr + lane_in_row, nullptr));
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[warp * S + sidx]);
      }
    }
#pragma unroll
    for (int v = 0; v < kGemvMaxVec; ++v) {
      if (v < nvec) {
        float* y = s.y + (size_t)v * a.y_stride;
        const float g = reduce_row(acc[v][0], s.lpr);
        if (swiglu) {
          const float u = reduce_row(acc[v][1], s.lpr);
          if (lane_in_row == 0 && row < s.rows) y[row] = silu_mul_det(g, u);
        } else if (lane_in_row == 0 && row < s.rows) {
          y[row] = add ? __fadd_rn(yold[v], g) : g;
        }
      }
    }
  }
  return true;
}

}  // namespace mcpo
