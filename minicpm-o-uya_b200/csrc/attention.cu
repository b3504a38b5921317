// attention.cu -- single-query (decode) causal GQA attention for sm_100a.
//
// Semantics (src/minicpmo/qwen3.uya:1664-1713, gpu_shim.c:926-979): for q
// head h the kv head is (h*n_kv)/n_head; scores = q.k_t * scale for t <= pos,
// softmax over t, out = sum_t p_t v_t.  KV cache layout [layer][pos][kv_dim]
// as the reference (qwen3.uya:1664-1666), f32 (reference) or f16.
//
// B200 design: split-K flash decoding.  grid = (n_kv, n_split); a CTA owns one
// kv head and a contiguous range of positions, serves every q head of its
// GQA group from one pass over K and V (each K/V row is read once per
// token), keeps an online softmax per head in registers and writes one
// partial (m, l, acc) per head.  The last CTA to finish a kv head (atomic
// ticket) merges the partials, writes the f32 output and, optionally, its
// Q8_1 blocks for the o-projection -- no separate combine launch.
//
// Fused mode also performs, for the current position, the per-head
// QK-RMSNorm (qwen3.uya:1543-1558, eps 1e-6, reduction order of
// gpu_shim.c:719-745 with an exact 1/sqrtf), NeoX RoPE from the host-built
// cos/sin table (qwen3.uya:1605-1662) and the KV append
// (qwen3.uya:1668-1675), so q/k never round-trip through separate kernels.
#include "attention.cuh"

#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "gemv.cuh"
#include "rowops.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kGMax = 8;

struct AttnSmem {
  float* q;     // [kGMax][HD]
  float* kpos;  // [HD]
  float* vpos;  // [HD]
  float* sq;    // [kAttnWarps][256]
  float* rm;    // [kAttnWarps][kGMax]
  float* rl;    // [kAttnWarps][kGMax]
  float* racc;  // [kAttnWarps][kGMax][HD]
};

__device__ __forceinline__ AttnSmem carve(float* base, int hd) {
  AttnSmem s;
  s.q = base;
  s.kpos = s.q + kGMax * hd;
  s.vpos = s.kpos + hd;
  s.sq = s.vpos + hd;
  s.rm = s.sq + kAttnWarps * 256;
  s.rl = s.rm + kAttnWarps * kGMax;
  s.racc = s.rl + kAttnWarps * kGMax;
  return s;
}

template <typename T>
__device__ __forceinline__ float kv_load(const void* p, size_t i) {
  if constexpr (sizeof(T) == 2)
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
  else
    return reinterpret_cast<const float*>(p)[i];
}

template <typename T>
__device__ __forceinline__ void kv_store(void* p, size_t i, float v) {
  if constexpr (sizeof(T) == 2)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

// J = elements per lane (hd = 32*J), or J = 1 with hd <= 32 (masked).
template <int J, typename T>
__global__ void __launch_bounds__(kAttnWarps * 32) k_attention(const AttnArgs a) {
  extern __shared__ __align__(16) float smem_f[];
  const int hd = a.head_dim;
  const AttnSmem sm = carve(smem_f, hd);
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  const int hb = (kvh * a.n_head + a.n_kv - 1) / a.n_kv;
  const int he = ((kvh + 1) * a.n_head + a.n_kv - 1) / a.n_kv;
  const int pos = a.pos_ptr ? *a.pos_ptr : a.pos_static;
  const int n_pos = pos + 1;
  int chunk = (n_pos + a.n_split - 1) / a.n_split;
  if (chunk < 32) chunk = 32;
  const int n_active = (n_pos + chunk - 1) / chunk;
  const int t0 = split * chunk;
  const int t1 = min(t0 + chunk, n_pos);
  const int kv_dim = a.n_kv * hd;
  const size_t kv_off = (size_t)kvh * hd;
  const int stride_part = hd + 2;

  // K/V of the current position (fused: normalised/rotated here and appended).
  if (a.fuse_norm_rope_append) {
    if (warp == 0) {
      for (int d = lane; d < hd; d += 32) sm.kpos[d] = a.k[kv_off + d];
      __syncwarp();
      norm_rope_row(sm.kpos, sm.sq, hd, a.k_norm, a.k_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base, a.rope_scale,
                    pos, lane);
    } else if (warp == 1) {
      for (int d = lane; d < hd; d += 32) sm.vpos[d] = a.v[kv_off + d];
    }
    __syncthreads();
    if (split == 0) {
      for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        kv_store<T>(a.k_cache, (size_t)pos * kv_dim + kv_off + d, sm.kpos[d]);
        kv_store<T>(a.v_cache, (size_t)pos * kv_dim + kv_off + d, sm.vpos[d]);
      }
    }
  }

  for (int g0 = hb; g0 < he; g0 += kGMax) {
    const int G = min(kGMax, he - g0);
    // q rows of this head batch
    for (int g = warp; g < G; g += kAttnWarps) {
      float* row = sm.q + g * hd;
      for (int d = lane; d < hd; d += 32) row[d] = a.q[(size_t)(g0 + g) * hd + d];
      __syncwarp();
      if (a.fuse_norm_rope_append)
        norm_rope_row(row, sm.sq + warp * 256, hd, a.q_norm, a.q_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base,
                      a.rope_scale, pos, lane);
    }
    __syncthreads();

    float m[kGMax], l[kGMax], acc[kGMax][J];
#pragma unroll
    for (int g = 0; g < kGMax; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.0f;
#pragma unroll
      for (int j = 0; j < J; ++j) acc[g][j] = 0.0f;
    }
    // lane element mapping: d = lane*J + j (hd == 32*J) or d = lane (J == 1, hd <= 32)
    const bool act = (lane * J) < hd;
    float qv[kGMax][J];
#pragma unroll
    for (int g = 0; g < kGMax; ++g)
#pragma unroll
      for (int j = 0; j < J; ++j) qv[g][j] = (g < G && act) ? sm.q[g * hd + lane * J + j] : 0.0f;

    if (split < n_active) {
      for (int t = t0 + warp; t < t1; t += kAttnWarps) {
        float kv[J], vv[J];
        const bool cur = a.fuse_norm_rope_append && t == pos;
        const size_t base = (size_t)t * kv_dim + kv_off + lane * J;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          kv[j] = act ? (cur ? sm.kpos[lane * J + j] : kv_load<T>(a.k_cache, base + j)) : 0.0f;
          vv[j] = act ? (cur ? sm.vpos[lane * J + j] : kv_load<T>(a.v_cache, base + j)) : 0.0f;
        }
#pragma unroll
        for (int g = 0; g < kGMax; ++g) {
          if (g < G) {
            float p = 0.0f;
#pragma unroll
            for (int j = 0; j < J; ++j) p = __fmaf_rn(qv[g][j], kv[j], p);
            const float s = __fmul_rn(__shfl_sync(0xffffffffu, warp_sum(p), 0), a.scale);
            const float mn = fmaxf(m[g], s);
            const float alpha = expf_det(__fsub_rn(m[g], mn));  // m = -inf -> 0
            const float beta = expf_det(__fsub_rn(s, mn));
            l[g] = __fadd_rn(__fmul_rn(l[g], alpha), beta);
            m[g] = mn;
#pragma unroll
            for (int j = 0; j < J; ++j) acc[g][j] = __fadd_rn(__fmul_rn(acc[g][j], alpha), __fmul_rn(beta, vv[j]));
          }
        }
      }
    }
    // merge the warps of this CTA
#pragma unroll
    for (int g = 0; g < kGMax; ++g) {
      if (g < G) {
        if (lane == 0) {
          sm.rm[warp * kGMax + g] = m[g];
          sm.rl[warp * kGMax + g] = l[g];
        }
        if (act)
#pragma unroll
          for (int j = 0; j < J; ++j) sm.racc[(warp * kGMax + g) * hd + lane * J + j] = acc[g][j];
      }
    }
    __syncthreads();
    if (split < n_active) {
      for (int g = warp; g < G; g += kAttnWarps) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm.rm[w * kGMax + g]);
        float L = 0.0f;
        float wt[kAttnWarps];
        for (int w = 0; w < kAttnWarps; ++w) {
          const float mw = sm.rm[w * kGMax + g];
          wt[w] = mw == -INFINITY ? 0.0f : expf_det(__fsub_rn(mw, M));
          L = __fadd_rn(L, __fmul_rn(wt[w], sm.rl[w * kGMax + g]));
        }
        float* dst = a.partial + ((size_t)(g0 + g) * a.n_split + split) * stride_part;
        for (int d = lane; d < hd; d += 32) {
          float s = 0.0f;
          for (int w = 0; w < kAttnWarps; ++w) s = __fadd_rn(s, __fmul_rn(wt[w], sm.racc[(w * kGMax + g) * hd + d]));
          dst[2 + d] = s;
        }
        if (lane == 0) {
          dst[0] = M;
          dst[1] = L;
        }
      }
    }
    __syncthreads();
  }

  // last CTA of this kv head merges the splits
  __shared__ unsigned ticket_s;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) ticket_s = atomicAdd(&a.counters[kvh], 1u);
  __syncthreads();
  if (ticket_s != (unsigned)(a.n_split - 1)) return;
  if (threadIdx.x == 0) atomicExch(&a.counters[kvh], 0u);
  __threadfence();
  for (int h = hb + warp; h < he; h += kAttnWarps) {
    const float* ph = a.partial + (size_t)h * a.n_split * stride_part;
    float M = -INFINITY;
    for (int s = 0; s < n_active; ++s) M = fmaxf(M, __ldcg(ph + (size_t)s * stride_part));
    float L = 0.0f;
    for (int s = 0; s < n_active; ++s) {
      const float ms = __ldcg(ph + (size_t)s * stride_part);
      if (ms != -INFINITY) L = __fadd_rn(L, __fmul_rn(expf_det(__fsub_rn(ms, M)), __ldcg(ph + (size_t)s * stride_part + 1)));
    }
    const float invL = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
    for (int d0 = 0; d0 < hd; d0 += 32) {
      const int d = d0 + lane;
      float o = 0.0f;
      if (d < hd) {
        for (int s = 0; s < n_active; ++s) {
          const float ms = __ldcg(ph + (size_t)s * stride_part);
          if (ms != -INFINITY)
            o = __fadd_rn(o, __fmul_rn(expf_det(__fsub_rn(ms, M)), __ldcg(ph + (size_t)s * stride_part + 2 + d)));
        }
        o = __fmul_rn(o, invL);
        a.out[(size_t)h * hd + d] = o;
      }
      if (a.out_q8 && (hd % 32) == 0) {
        uint16_t dbits;
        bool zero;
        const int q = q8_1_quant_lane(o, &dbits, &zero);
        const float sum = warp_seq_sum(o);
        const uint16_t sbits = zero ? (uint16_t)0 : f32_to_f16_ref(sum);
        uint32_t word = ((uint32_t)(q & 0xff)) << (8 * (lane & 3));
        word |= __shfl_xor_sync(0xffffffffu, word, 1);
        word |= __shfl_xor_sync(0xffffffffu, word, 2);
        uint32_t* ob = reinterpret_cast<uint32_t*>(a.out_q8 + ((size_t)h * hd + d0) / 32 * 36);
        if (lane == 0) ob[0] = (uint32_t)dbits | ((uint32_t)sbits << 16);
        if ((lane & 3) == 0) ob[1 + (lane >> 2)] = word;
      }
    }
  }
}

size_t attn_smem_bytes(int hd) {
  return sizeof(float) * ((size_t)kGMax * hd + 2 * hd + kAttnWarps * 256 + 2 * kAttnWarps * kGMax +
                          (size_t)kAttnWarps * kGMax * hd);
}

template <int J>
cudaError_t launch_j(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const dim3 grid(a.n_kv, a.n_split);
  const size_t smem = attn_smem_bytes(a.head_dim);
  if (a.kv_f16) return launch_k(k_attention<J, __half>, grid, dim3(kAttnWarps * 32), smem, st, pdl, a);
  return launch_k(k_attention<J, float>, grid, dim3(kAttnWarps * 32), smem, st, pdl, a);
}

}  // namespace

size_t attn_partial_floats(int n_head, int n_split, int head_dim) {
  return (size_t)n_head * n_split * (head_dim + 2);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
  switch (a.head_dim) {
    case 64: return launch_j<2>(a, st, pdl);
    case 128: return launch_j<4>(a, st, pdl);
    case 256: return launch_j<8>(a, st, pdl);
    default:
      if (a.head_dim > 0 && a.head_dim <= 32) return launch_j<1>(a, st, pdl);
      return cudaErrorInvalidValue;
  }
}

}  // namespace mcpo
