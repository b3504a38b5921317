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

#include "attn_dev.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "rowops.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kGMax = 8;     // q heads per kv head handled by one CTA (<= 2 per warp)
constexpr int kMaxSplit = 64;

// The split merge reuses the K/V tile area: per q head of the group the
// splits' m, l and weights, 1/L, and (when they fit) a copy of every split's
// partial row; the merged output rows reuse the q area.
constexpr int kMergeStage = 12288;  // floats of staged partial rows (48 KB)

struct AttnSmem {
  float* q;     // [kGMax][hd]; the merged rows after the merge
  float* kpos;  // [hd]
  float* vpos;  // [hd]
  float* sq;    // [kAttnWarps][256]
  float* kt;    // [kSub][attn_tile_stride(hd)]
  float* vt;    // [kSub][attn_tile_stride(hd)]
  float* cm;    // [kGMax][kMaxSplit]   (merge, aliases kt/vt)
  float* cl;    // [kGMax][kMaxSplit]
  float* cw;    // [kGMax][kMaxSplit]
  float* cinv;  // [kGMax]
  float* mp;    // [G][n_active][attn_part_stride(hd)] staged partials, 16-byte aligned
};

// K/V tile row stride: hd + 4 keeps rows 16-byte aligned (async 16-byte
// copies, float4 reads) and lanes reading rows lane*hs conflict-free per
// quarter warp; odd small head sizes use hd + 1 with scalar access.
__host__ __device__ inline int attn_tile_stride(int hd) { return (hd & 3) ? hd + 1 : hd + 4; }

__host__ __device__ inline size_t attn_tile_floats(int hd) {
  const size_t kv = 2 * (size_t)kSub * attn_tile_stride(hd);
  const size_t merge = 3 * (size_t)kGMax * kMaxSplit + kGMax + 4 + kMergeStage;
  return kv > merge ? kv : merge;
}

__host__ __device__ inline size_t attn_smem_floats(int hd) {
  return (size_t)kGMax * hd + 2 * hd + kAttnWarps * 256 + attn_tile_floats(hd) + 4;
}

__device__ __forceinline__ AttnSmem carve(float* base, int hd) {
  AttnSmem s;
  s.q = base;
  s.kpos = s.q + kGMax * hd;
  s.vpos = s.kpos + hd;
  s.sq = s.vpos + hd;
  s.kt = s.sq + kAttnWarps * 256;
  s.vt = s.kt + kSub * attn_tile_stride(hd);
  s.cm = s.kt;
  s.cl = s.cm + kGMax * kMaxSplit;
  s.cw = s.cl + kGMax * kMaxSplit;
  s.cinv = s.cw + kGMax * kMaxSplit;
  const uintptr_t m = reinterpret_cast<uintptr_t>(s.cinv + kGMax);
  s.mp = reinterpret_cast<float*>((m + 15) & ~static_cast<uintptr_t>(15));
  return s;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// f32 cache, hd % 4 == 0: rows [c0, c0 + kSub) of K and V into the tile with
// L2-only 16-byte async copies (one commit group), rows >= t1 zero-filled.
// The current position's row (fused mode) is skipped; the caller writes it
// from kpos/vpos and then waits for the group.  False (nothing issued) when
// the cache is f16 or the head size is not a multiple of 4.
template <typename T>
__device__ __forceinline__ bool stage_tile_async(const AttnArgs& a, const AttnSmem& sm, int c0, int t1, int pos,
                                                 bool fused, int kv_dim, size_t kv_off, int hd, int hs) {
  if constexpr (sizeof(T) != 4) {
    return false;
  } else {
    if (hd & 3) return false;
    const int per = hd >> 2;
    const float* kc = static_cast<const float*>(a.k_cache);
    const float* vc = static_cast<const float*>(a.v_cache);
    for (int e = threadIdx.x; e < kSub * per; e += blockDim.x) {
      const int r = e / per, d = (e - r * per) * 4, t = c0 + r;
      float* kd = sm.kt + r * hs + d;
      float* vd = sm.vt + r * hs + d;
      if (t < t1) {
        if (!(fused && t == pos)) {
          const size_t i = (size_t)t * kv_dim + kv_off + d;
          cp_async16(kd, kc + i);
          cp_async16(vd, vc + i);
        }
      } else {
        *reinterpret_cast<float4*>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    return true;
  }
}

// The current position's row from kpos/vpos into tile row pos - c0 (when it
// falls in [c0, t1)), then the wait for the tile's async copies.
__device__ __forceinline__ void finish_tile_async(const AttnSmem& sm, int c0, int t1, int pos, bool fused, int hd,
                                                  int hs) {
  if (fused && pos >= c0 && pos < t1) {
    const int r = pos - c0;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      sm.kt[r * hs + d] = sm.kpos[d];
      sm.vt[r * hs + d] = sm.vpos[d];
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ void stage_kv(const AttnArgs& a, const AttnSmem& sm, int c0, int t1, int pos, bool fused,
                                         int kv_dim, size_t kv_off, int hd, int hs) {
  stage_kv_tile<T>(a.k_cache, a.v_cache, sm.kpos, sm.vpos, sm.kt, sm.vt, c0, t1, pos, fused, kv_dim, kv_off, hd, hs,
                   threadIdx.x, blockDim.x);
}

// J = output elements per lane in the P.V phase (hd = 32*J), or J = 1 with
// hd <= 32 (masked lanes).
//
// Per q head and KV chunk, in order over sub-chunks of 32 positions
// (lane = position):
//   s_t   = scale * sum_d q_d k_td            (sequential fma over d)
//   m'    = max(m, max_t s_t)
//   alpha = exp(m - m'),  p_t = exp(s_t - m')  (0 beyond the chunk)
//   l     = l*alpha + butterfly_sum(p)
//   acc_d = acc_d*alpha, then acc_d = fma(p_t, v_td, acc_d) for t in order
// and the splits are merged as o_d = (sum_s w_s acc_sd) / (sum_s w_s l_s),
// w_s = exp(m_s - max m), sums in split order with fma.
template <int J, typename T>
__global__ void __launch_bounds__(kAttnWarps * 32) k_attention(const AttnArgs a) {
  extern __shared__ __align__(16) float smem_f[];
  const int hd = a.head_dim;
  const int hs = attn_tile_stride(hd);
  const AttnSmem sm = carve(smem_f, hd);
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hb = (kvh * a.n_head + a.n_kv - 1) / a.n_kv;
  const int he = ((kvh + 1) * a.n_head + a.n_kv - 1) / a.n_kv;
  const int G = he - hb;
  const int pos = a.pos_ptr ? *a.pos_ptr : a.pos_static;
  const int n_pos = pos + 1;
  int chunk = (n_pos + a.n_split - 1) / a.n_split;
  if (chunk < 32) chunk = 32;
  const int n_active = (n_pos + chunk - 1) / chunk;
  const int t0 = split * chunk;
  const int t1 = min(t0 + chunk, n_pos);
  const int kv_dim = a.n_kv * hd;
  const size_t kv_off = (size_t)kvh * hd;
  const int stride_part = attn_part_stride(hd);
  const bool fused = a.fuse_norm_rope_append != 0;
  const bool active = split < n_active;
  const int nt = blockDim.x;

  // Before waiting for the previous kernel (programmatic dependent launch):
  // everything that only depends on earlier steps -- the position, the K/V
  // rows of earlier positions for the first sub-chunk (f32 cache: async
  // copies straight into the tile; f16: into registers; the current position
  // comes from this kernel's prologue), and the norm weight and RoPE lines
  // (into L1).
  const bool tile_async = active && stage_tile_async<T>(a, sm, t0, t1, pos, fused, kv_dim, kv_off, hd, hs);
  const int n4 = kSub * hd / 4;
  const bool early = active && !tile_async && (hd & 3) == 0 && n4 <= 8 * nt;
  float4 pk[8], pv[8];
  if (early) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = threadIdx.x + u * nt;
      pk[u] = pv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < n4) {
        const int r = (e * 4) / hd, d = e * 4 - r * hd, t = t0 + r;
        if (t < t1 && !(fused && t == pos)) {
          const size_t i = (size_t)t * kv_dim + kv_off + d;
          pk[u] = kv_load4<T>(a.k_cache, i);
          pv[u] = kv_load4<T>(a.v_cache, i);
        }
      }
    }
  }
  if (fused && active && threadIdx.x < 12) {
    const uint8_t* line = nullptr;
    const int qb = a.q_norm_dtype == kF32 ? 4 : 2, kb = a.k_norm_dtype == kF32 ? 4 : 2;
    const int t = threadIdx.x;
    if (t < 4 && a.q_norm && t * 128 < hd * qb) line = static_cast<const uint8_t*>(a.q_norm) + t * 128;
    if (t >= 4 && t < 8 && a.k_norm && (t - 4) * 128 < hd * kb) line = static_cast<const uint8_t*>(a.k_norm) + (t - 4) * 128;
    if (t >= 8 && a.rope_cos) {
      const float* tab = (t < 10 ? a.rope_cos : a.rope_sin) + (size_t)pos * (hd / 2);
      if (((t - 8) & 1) * 128 < hd * 2) line = reinterpret_cast<const uint8_t*>(tab) + ((t - 8) & 1) * 128;
    }
    if (line) asm volatile("prefetch.global.L1 [%0];" ::"l"(line));
  }
  pdl_wait();
  pdl_launch_dependents();

  // K/V of the current position (fused: normalised/rotated here; needed by
  // split 0, which appends it, and by the split that holds position pos).
  if (fused && (split == 0 || split == n_active - 1)) {
    if (warp < 2) {
      const float* src = (warp == 0 ? a.k : a.v) + kv_off;
      float* dst = warp == 0 ? sm.kpos : sm.vpos;
      float r[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) r[k] = lane + 32 * k < hd ? src[lane + 32 * k] : 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (lane + 32 * k < hd) dst[lane + 32 * k] = r[k];
      __syncwarp();
      if (warp == 0)
        norm_rope_row(sm.kpos, sm.sq, hd, a.k_norm, a.k_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base,
                      a.rope_scale, pos, lane);
    }
  }
  // q rows of this kv head's group (loads of both rows of a warp first)
  if (active) {
    float qv[2][8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int g = warp + i * kAttnWarps;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int d = lane + 32 * k;
        qv[i][k] = (g < G && d < hd) ? a.q[(size_t)(hb + g) * hd + d] : 0.0f;
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int g = warp + i * kAttnWarps;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int d = lane + 32 * k;
        if (g < G && d < hd) sm.q[g * hd + d] = qv[i][k];
      }
    }
    __syncwarp();
  }
  for (int g = warp; active && g < G; g += kAttnWarps) {
    float* row = sm.q + g * hd;
    if (fused)
      norm_rope_row(row, sm.sq + warp * 256, hd, a.q_norm, a.q_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base,
                    a.rope_scale, pos, lane);
  }
  __syncthreads();
  if (fused && split == 0) {
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      kv_store<T>(a.k_cache, (size_t)pos * kv_dim + kv_off + d, sm.kpos[d]);
      kv_store<T>(a.v_cache, (size_t)pos * kv_dim + kv_off + d, sm.vpos[d]);
    }
  }

  if (active) {
    // up to two heads per warp (G <= 8)
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f}, acc[2][J];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < J; ++j) acc[i][j] = 0.0f;
    const bool act = lane * J < hd;
    for (int c0 = t0; c0 < t1; c0 += kSub) {
      // stage K and V rows of this sub-chunk (the current position from
      // smem): groups of 4 values, all loads of a batch issued before the
      // shared-memory stores
      if (tile_async && c0 == t0) {
        finish_tile_async(sm, c0, t1, pos, fused, hd, hs);
      } else if (tile_async && c0 > t0) {
        stage_tile_async<T>(a, sm, c0, t1, pos, fused, kv_dim, kv_off, hd, hs);
        finish_tile_async(sm, c0, t1, pos, fused, hd, hs);
      } else if (early && c0 == t0) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int e = threadIdx.x + u * nt;
          if (e < n4) {
            const int r = (e * 4) / hd, d = e * 4 - r * hd, t = c0 + r;
            float4 kk = pk[u], vv = pv[u];
            if (fused && t == pos && t < t1) {
              kk = make_float4(sm.kpos[d], sm.kpos[d + 1], sm.kpos[d + 2], sm.kpos[d + 3]);
              vv = make_float4(sm.vpos[d], sm.vpos[d + 1], sm.vpos[d + 2], sm.vpos[d + 3]);
            }
            float* kd = sm.kt + r * hs + d;
            float* vd = sm.vt + r * hs + d;
            kd[0] = kk.x; kd[1] = kk.y; kd[2] = kk.z; kd[3] = kk.w;
            vd[0] = vv.x; vd[1] = vv.y; vd[2] = vv.z; vd[3] = vv.w;
          }
        }
      } else {
        stage_kv<T>(a, sm, c0, t1, pos, fused, kv_dim, kv_off, hd, hs);
      }
      __syncthreads();
      const int t = c0 + lane;
      const bool valid = t < t1;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int g = warp + i * kAttnWarps;
        if (g >= G) break;
        const float* qrow = sm.q + g * hd;
        float sc = 0.0f;
        if ((hs & 3) == 0) {  // 16-byte reads, the same sequential order over d
          const float4* kr = reinterpret_cast<const float4*>(sm.kt + lane * hs);
          const float4* qr = reinterpret_cast<const float4*>(qrow);
          for (int d4 = 0; d4 < (hd >> 2); ++d4) {
            const float4 k4 = kr[d4], q4 = qr[d4];
            sc = __fmaf_rn(q4.x, k4.x, sc);
            sc = __fmaf_rn(q4.y, k4.y, sc);
            sc = __fmaf_rn(q4.z, k4.z, sc);
            sc = __fmaf_rn(q4.w, k4.w, sc);
          }
        } else {
          for (int d = 0; d < hd; ++d) sc = __fmaf_rn(qrow[d], sm.kt[lane * hs + d], sc);
        }
        sc = valid ? __fmul_rn(sc, a.scale) : -INFINITY;
        const float mx = warp_max(sc);
        const float mn = fmaxf(m[i], mx);
        const float alpha = expf_det(__fsub_rn(m[i], mn));
        const float p = valid ? expf_det(__fsub_rn(sc, mn)) : 0.0f;
        const float psum = __shfl_sync(0xffffffffu, warp_sum(p), 0);
        l[i] = __fadd_rn(__fmul_rn(l[i], alpha), psum);
        m[i] = mn;
#pragma unroll
        for (int j = 0; j < J; ++j) acc[i][j] = __fmul_rn(acc[i][j], alpha);
        for (int tt = 0; tt < kSub; ++tt) {
          const float pt = __shfl_sync(0xffffffffu, p, tt);
          if (act) {
            float vv[J];
            const float* vr = sm.vt + tt * hs + lane * J;
            if constexpr (J % 4 == 0) {
              if ((hs & 3) == 0) {
#pragma unroll
                for (int j = 0; j < J; j += 4) {
                  const float4 v4 = *reinterpret_cast<const float4*>(vr + j);
                  vv[j] = v4.x; vv[j + 1] = v4.y; vv[j + 2] = v4.z; vv[j + 3] = v4.w;
                }
              } else {
#pragma unroll
                for (int j = 0; j < J; ++j) vv[j] = vr[j];
              }
            } else if constexpr (J == 2) {
              if ((hs & 3) == 0) {
                const float2 v2 = *reinterpret_cast<const float2*>(vr);
                vv[0] = v2.x; vv[1] = v2.y;
              } else {
                vv[0] = vr[0]; vv[1] = vr[1];
              }
            } else {
#pragma unroll
              for (int j = 0; j < J; ++j) vv[j] = vr[j];
            }
#pragma unroll
            for (int j = 0; j < J; ++j) acc[i][j] = __fmaf_rn(pt, vv[j], acc[i][j]);
          }
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int g = warp + i * kAttnWarps;
      if (g >= G) break;
      float* dst = a.partial + ((size_t)(hb + g) * a.n_split + split) * stride_part;
      if (act)
#pragma unroll
        for (int j = 0; j < J; ++j) dst[4 + lane * J + j] = acc[i][j];
      if (lane == 0) {
        dst[0] = m[i];
        dst[1] = l[i];
      }
    }
  }

  // last CTA of this kv head merges the splits: the CTA barrier orders every
  // thread's partial stores before thread 0's acquire-release ticket
  __shared__ unsigned ticket_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(&a.counters[kvh]) : "memory");
    ticket_s = t;
  }
  __syncthreads();
  if (ticket_s != (unsigned)(a.n_split - 1)) return;
  if (threadIdx.x == 0) atomicExch(&a.counters[kvh], 0u);
  // Merge: (1) m and l of all (head, split) pairs -- with every split's
  // partial row copied into shared memory in one round trip when they fit
  // (L2-only bulk copies); (2) per head M = max m, w_s = exp(m_s - M) and
  // L = sum_s w_s l_s (fma in split order); (3) o_d = sum_s w_s acc_sd (fma in
  // split order) * (1/L) by one thread per (head, d); (4) Q8_1 blocks of the
  // output, one warp per block.
  const bool staged = (size_t)G * n_active * stride_part <= (size_t)kMergeStage;
  if (staged) {
    const int per = stride_part / 4;  // 16-byte pieces per partial row
    for (int i = threadIdx.x; i < G * n_active * per; i += nt) {
      const int row = i / per, c = i - row * per;
      const int g = row / n_active, sp = row - g * n_active;
      cp_async16(sm.mp + (size_t)row * stride_part + c * 4,
                 a.partial + ((size_t)(hb + g) * a.n_split + sp) * stride_part + c * 4);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    for (int i = threadIdx.x; i < G * n_active; i += nt) {
      const int g = i / n_active, sp = i - g * n_active;
      sm.cm[g * kMaxSplit + sp] = sm.mp[(size_t)i * stride_part];
      sm.cl[g * kMaxSplit + sp] = sm.mp[(size_t)i * stride_part + 1];
    }
  } else {
    for (int i = threadIdx.x; i < G * n_active; i += nt) {
      const int g = i / n_active, sp = i - g * n_active;
      const float* ps = a.partial + ((size_t)(hb + g) * a.n_split + sp) * stride_part;
      sm.cm[g * kMaxSplit + sp] = __ldcg(ps);
      sm.cl[g * kMaxSplit + sp] = __ldcg(ps + 1);
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += kAttnWarps) {
    const float* mg = sm.cm + g * kMaxSplit;
    float M = -INFINITY;
    for (int sp = lane; sp < n_active; sp += 32) M = fmaxf(M, mg[sp]);
    M = warp_max(M);
    for (int sp = lane; sp < n_active; sp += 32) sm.cw[g * kMaxSplit + sp] = expf_det(__fsub_rn(mg[sp], M));
    __syncwarp();
    if (lane == 0) {
      float L = 0.0f;
      for (int sp = 0; sp < n_active; ++sp) L = __fmaf_rn(sm.cw[g * kMaxSplit + sp], sm.cl[g * kMaxSplit + sp], L);
      sm.cinv[g] = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
    }
  }
  __syncthreads();
  constexpr int kLd = 16;
  for (int i = threadIdx.x; i < G * hd; i += nt) {
    const int g = i / hd, d = i - g * hd;
    const float* wg = sm.cw + g * kMaxSplit;
    float o = 0.0f;
    if (staged) {
      const float* pg = sm.mp + (size_t)g * n_active * stride_part + 4 + d;
      for (int sp = 0; sp < n_active; ++sp) o = __fmaf_rn(wg[sp], pg[(size_t)sp * stride_part], o);
    } else {
      const float* pg = a.partial + (size_t)(hb + g) * a.n_split * stride_part + 4 + d;
      for (int s0 = 0; s0 < n_active; s0 += kLd) {
        float r[kLd];
#pragma unroll
        for (int u = 0; u < kLd; ++u) r[u] = s0 + u < n_active ? __ldcg(pg + (size_t)(s0 + u) * stride_part) : 0.0f;
#pragma unroll
        for (int u = 0; u < kLd; ++u)
          if (s0 + u < n_active) o = __fmaf_rn(wg[s0 + u], r[u], o);
      }
    }
    o = __fmul_rn(o, sm.cinv[g]);
    a.out[(size_t)(hb + g) * hd + d] = o;
    sm.q[i] = o;
  }
  if (a.out_q8 && (hd % 32) == 0) {
    __syncthreads();
    for (int b = warp; b < G * hd / 32; b += kAttnWarps) {
      const float o = sm.q[b * 32 + lane];
      uint16_t dbits;
      bool zero;
      const int q = q8_1_quant_lane(o, &dbits, &zero);
      uint32_t word = ((uint32_t)(q & 0xff)) << (8 * (lane & 3));
      word |= __shfl_xor_sync(0xffffffffu, word, 1);
      word |= __shfl_xor_sync(0xffffffffu, word, 2);
      uint32_t* ob = reinterpret_cast<uint32_t*>(a.out_q8 + ((size_t)hb * hd + (size_t)b * 32) / 32 * 36);
      if (lane == 0) {
        float sum = 0.0f;  // the sequential f16 s of the reference block
        for (int t = 0; t < 32; ++t) sum = __fadd_rn(sum, sm.q[b * 32 + t]);
        ob[0] = (uint32_t)dbits | ((uint32_t)(zero ? (uint16_t)0 : f32_to_f16_ref(sum)) << 16);
      }
      if ((lane & 3) == 0) ob[1 + (lane >> 2)] = word;
    }
  }
}

size_t attn_smem_bytes(int hd) { return sizeof(float) * attn_smem_floats(hd); }

template <int J>
cudaError_t launch_j(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const dim3 grid(a.n_kv, a.n_split);
  const size_t smem = attn_smem_bytes(a.head_dim);
  if (a.kv_f16) return launch_k(k_attention<J, __half>, grid, dim3(kAttnWarps * 32), smem, st, pdl, a);
  return launch_k(k_attention<J, float>, grid, dim3(kAttnWarps * 32), smem, st, pdl, a);
}

template <int J>
cudaError_t init_j() {
  const int mx = (int)attn_smem_bytes(256);
  cudaError_t e = cudaFuncSetAttribute(k_attention<J, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_attention<J, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  return e;
}

}  // namespace

size_t attn_partial_floats(int n_head, int n_split, int head_dim) {
  return (size_t)n_head * n_split * attn_part_stride(head_dim);
}

cudaError_t attention_init() {
  cudaError_t e = init_j<1>();
  if (e == cudaSuccess) e = init_j<2>();
  if (e == cudaSuccess) e = init_j<4>();
  if (e == cudaSuccess) e = init_j<8>();
  return e;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.n_split > kMaxSplit || a.n_split < 1) return cudaErrorInvalidValue;
  if (a.n_head > kGMax * a.n_kv) return cudaErrorInvalidValue;
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
