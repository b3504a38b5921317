// common.cuh -- device helpers shared by the sm_100a kernels of
// libminicpmo_gpu_helper.so.
//
// Data formats (GGUF block layouts used by the reference,
// src/minicpmo/qwen3.uya:847-1000, gpu_shim.c:37-41):
//   Q4_K  256 values / 144 B : f16 d, f16 dmin, u8 scales[12], u8 qs[128]
//   Q6_K  256 values / 210 B : u8 ql[128], u8 qh[64], i8 sc[16], f16 d
//   Q8_0   32 values /  34 B : f16 d, i8 qs[32]
//   Q8_1   32 values /  36 B : f16 d, f16 s, i8 qs[32]  (activations)
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mcpo {

// Uya TensorDType ordinals, the dtype integers of the reference ABI
// (src/minicpmo/tensor.uya:31-54; the shim tests 10/12, gpu_shim.c:323).
enum DType : int { kF32 = 0, kF16 = 1, kQ8_0 = 6, kQ4_K = 10, kQ6_K = 12, kBF16 = 20 };

constexpr int kGemvWarps = 8;           // consumer warps per GEMV CTA
constexpr int kGemvThreads = kGemvWarps * 32;

// ---------------------------------------------------------------------
// f16 conversions with the reference's rounding.
// f16 -> f32 is exact; the hardware conversion gives the same bits as
// kernels.uya:48-78.  f32 -> f16 follows kernels.uya:79-108 /
// gpu_shim.c:2157-2192: truncate, then add one unit when the first dropped
// bit is set (ties away from zero, not IEEE round-to-nearest-even).
// ---------------------------------------------------------------------
__device__ __forceinline__ float f16_to_f32(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

__device__ __forceinline__ uint16_t f32_to_f16_ref(float v) {
  uint32_t u = __float_as_uint(v);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t e = (u >> 23) & 0xffu;
  uint32_t frac = u & 0x7fffffu;
  if (e == 255u) return (uint16_t)(sign | (frac != 0u ? 0x7e00u : 0x7c00u));
  if (e > 142u) return (uint16_t)(sign | 0x7c00u);
  if (e < 113u) {
    if (e < 103u) return (uint16_t)sign;
    frac |= 0x800000u;
    uint16_t out = (uint16_t)(sign | (frac >> (126u - e)));
    if ((frac >> (125u - e)) & 1u) out = (uint16_t)(out + 1u);
    return out;
  }
  uint16_t out = (uint16_t)(sign | ((e - 112u) << 10) | (frac >> 13));
  if (frac & 0x1000u) out = (uint16_t)(out + 1u);
  return out;
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ float load_weight(const void* w, int dtype, int i) {
  if (dtype == kF32) return reinterpret_cast<const float*>(w)[i];
  if (dtype == kBF16) return bf16_to_f32(reinterpret_cast<const uint16_t*>(w)[i]);
  return f16_to_f32(reinterpret_cast<const uint16_t*>(w)[i]);
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// 16-byte streaming load that bypasses L1 (weights are read once per token).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Butterfly sum (xor 16, 8, 4, 2, 1).  Lanes may end with differently
// ordered totals; callers that need one value broadcast lane 0's.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Number of KV splits of the decode attention: a function of the kv-head
// count only, so results do not depend on the GPU's SM count.
// Splits of the positions per kv head: ceil(256 / n_kv) CTAs' worth of
// parallelism, at most 16 (one thread-block cluster per kv head).
__host__ __device__ inline int attn_n_split(int n_kv) {
  int s = (256 + n_kv - 1) / n_kv;
  return s < 1 ? 1 : (s > 16 ? 16 : s);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Q8_1 quantisation of one 32-value block held one value per lane
// (gpu_shim.c:336-378, "variant B"): d = amax/127 (IEEE division),
// q = trunc(x/d +- 0.5) clamped to [-128, 127].  Returns q for this lane and
// the f16 bits of d in *d_bits; *all_zero is set when amax == 0 (then the
// block is all zeros, s included).  d may underflow to f16 zero while
// amax > 0: the quants are still computed with the f32 d, as the reference
// does.  Every lane gets the same d_bits.  Uses only round-to-nearest IEEE
// operations so the result is bit-identical to the reference's host
// quantiser.
__device__ __forceinline__ int q8_1_quant_lane(float x, uint16_t* d_bits, bool* all_zero) {
  // amax: one warp reduction over the bit patterns (order-preserving for
  // non-negative floats); NaN inputs count as 0, as in the reference's
  // `fabsf(x) > amax` scan
  const float ax = fabsf(x);
  const float amax = __int_as_float((int)__reduce_max_sync(0xffffffffu, ax == ax ? (unsigned)__float_as_int(ax) : 0u));
  *all_zero = amax == 0.0f;
  if (amax == 0.0f) {
    *d_bits = 0;
    return 0;
  }
  const float d = __fdiv_rn(amax, 127.0f);
  *d_bits = f32_to_f16_ref(d);
  // q = trunc(v +- 0.5) with v = x/d correctly rounded.  x * rcp(d) is
  // within 2.3e-5 of v for |v| <= 128 (two roundings of 2^-24 relative each,
  // plus half an ulp of v), and trunc(v +- 0.5) only changes where |v| is
  // within 2^-17 of a half-integer; so away from a 1e-4 window around the
  // half-integers the product gives the same q, and inside it (or when
  // rcp(d) overflows) the exact quotient is used.
  float v = __fmul_rn(x, __frcp_rn(d));
  const float a = fabsf(v);
  if (!(fabsf(__fsub_rn(__fsub_rn(a, floorf(a)), 0.5f)) >= 1e-4f)) v = __fdiv_rn(x, d);
  int q = __float2int_rz(v >= 0.0f ? __fadd_rn(v, 0.5f) : __fsub_rn(v, 0.5f));
  q = q > 127 ? 127 : q;
  q = q < -128 ? -128 : q;
  return q;
}

// Sequential x0 + x1 + ... + x31 across lanes (the reference's s field),
// result valid in every lane.
__device__ __forceinline__ float warp_seq_sum(float x) {
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) s = __fadd_rn(s, __shfl_sync(0xffffffffu, x, i));
  return s;
}

// Deterministic exp: Cody-Waite argument reduction x = k*ln2 + r (ln2 split
// into a 15-bit head and a tail, so k*LN2_HI is exact) and the degree-7
// Taylor polynomial of e^r on |r| <= ln2/2 in Horner form, then an exact
// scaling by 2^k.  Every step is a correctly rounded IEEE operation (rint,
// fma, mul), so the CPU oracle's C restatement returns the same bits.
// Relative error below 2 ulp over the float range.
__device__ __forceinline__ float expf_det(float x) {
  if (x != x) return x;
  if (x >= 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x <= -103.97208404541015625f) return 0.0f;
  const float k = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(-k, 0.693145751953125f, x);
  r = __fmaf_rn(-k, 1.428606765330187045e-06f, r);
  float p = 1.98412698412698e-4f;
  p = __fmaf_rn(p, r, 1.38888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ki = (int)k;
  if (ki > 127) {
    p = __fmul_rn(p, 2.0f);
    ki = 127;
  }
  if (ki < -126) {
    p = __fmul_rn(p, 5.42101086242752217e-20f);  // 2^-64
    ki += 64;
  }
  return __fmul_rn(p, __int_as_float((ki + 127) << 23));
}

// silu(g) * u with the deterministic exp (kernels.uya:198: g / (1 + e^-g)).
__device__ __forceinline__ float silu_mul_det(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_det(-g))), u);
}

// Bounded spin helper: every wait in this library gives up after a limit
// and reports through an error word instead of hanging the GPU.
constexpr long long kSpinLimit = 1ll << 26;

}  // namespace mcpo
