// attention.cu -- single-query (decode) causal GQA attention for sm_100a.
//
// Semantics (src/minicpmo/qwen3.uya:1664-1713, gpu_shim.c:926-979): for q
// head h the kv head is (h*n_kv)/n_head; scores = q.k_t * scale for t <= pos,
// softmax over t, out = sum_t p_t v_t.  KV cache layout [layer][pos][kv_dim]
// as the reference (qwen3.uya:1664-1666), f32 (reference) or f16.
//
// B200 design: split-K flash decoding.  grid = (n_kv, n_split, batch); a CTA
// owns one kv head of one sequence and a contiguous range of positions,
// serves every q head of its GQA group from one pass over K and V (each K/V
// row is read once per token), keeps an online softmax per head in
// registers and produces one partial (m, l, acc) per head.  The partials of
// a kv head are merged either inside a thread-block cluster through
// distributed shared memory (the default of the decode graph) or by the
// last-arriving CTA through global memory (atomic ticket); both merge in
// split order with the same operations, so they give the same bits.  The
// merge writes the f32 output and, optionally, its Q8_1 blocks for the
// o-projection -- no separate combine launch.
//
// K/V rows reach shared memory by 16-byte asynchronous copies (L2 only) in
// the cache's own type, into a ring of 32-position tiles: the first tiles
// are requested before the kernel waits for its predecessor (programmatic
// dependent launch), and each later tile is requested while the tile before
// it is being used.
//
// Fused mode also performs, for the current position, the per-head
// QK-RMSNorm (qwen3.uya:1543-1558, eps 1e-6, reduction order of
// gpu_shim.c:719-745 with an exact 1/sqrtf), NeoX RoPE from the host-built
// cos/sin table (qwen3.uya:1605-1662) and the KV append
// (qwen3.uya:1668-1675), so q/k never round-trip through separate kernels.
// The current position is attended as the cache stores it (f16: rounded).
#include "attention.cuh"

#include <cuda_fp16.h>
#include <math.h>
#include <string.h>

#include <type_traits>

#include "attn_dev.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "rowops.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kGMax = 8;  // q heads per kv head handled by one CTA (<= 2 per warp)
constexpr int kMaxSplit = 64;

// The global-memory merge reuses the tile area: per q head of the group the
// splits' m, l and weights, 1/L, and (when they fit) a copy of every split's
// partial row.
constexpr int kMergeStage = 12288;  // floats of staged partial rows (48 KB)

// Small odd head sizes (J = 1, head_dim <= 32) stage f32 tiles through
// registers with this row stride; the async tiles use head_dim + 16 bytes.
__host__ __device__ inline int attn_tile_stride(int hd) { return (hd & 3) ? hd + 1 : hd + 4; }

// Tile geometry of one instantiation.  J >= 2 (head_dim 64/128/256): tiles
// in the cache type TT, rows of head_dim + 16 bytes (16-byte aligned, and
// lanes reading rows lane*stride hit distinct banks per quarter warp), a
// ring of kRing tiles.  J = 1: one f32 tile staged through registers.
template <int J, typename T>
struct TileCfg {
  static constexpr bool kAsync = J >= 2;
  using TT = std::conditional_t<kAsync, T, float>;
  static constexpr int kRing = kAsync ? (J >= 8 ? 2 : 3) : 1;
  __host__ __device__ static int stride(int hd) { return kAsync ? hd + 16 / (int)sizeof(TT) : attn_tile_stride(hd); }
  __host__ __device__ static size_t buf_bytes(int hd) { return 2 * (size_t)kSub * stride(hd) * sizeof(TT); }
};

__host__ __device__ inline size_t round16(size_t b) { return (b + 15) & ~(size_t)15; }

// Shared memory: q [kGMax][hd], kpos [hd], vpos [hd], norm scratch
// [kAttnWarps][256] (f32), then at tiles_offset the tile ring, which the
// merge reuses (cluster: this split's partial rows [G][hd + 4]; global:
// m/l/w [kGMax][kMaxSplit] x3, 1/L [kGMax], staged partial rows).
__host__ __device__ inline size_t attn_tiles_offset(int hd) {
  return round16(sizeof(float) * ((size_t)kGMax * hd + 2 * (size_t)hd + kAttnWarps * 256));
}

__host__ __device__ inline size_t attn_merge_stage_offset() {
  return round16(sizeof(float) * (3 * (size_t)kGMax * kMaxSplit + kGMax));
}

// The tile ring's mbarriers (one per buffer) follow the tile / merge area.
template <int J, typename T, bool kCluster>
__host__ __device__ inline size_t attn_bars_offset(int hd) {
  using C = TileCfg<J, T>;
  const size_t tiles = C::kRing * C::buf_bytes(hd);
  const size_t merge = kCluster ? sizeof(float) * (size_t)kGMax * attn_part_stride(hd)
                                : attn_merge_stage_offset() + sizeof(float) * (size_t)kMergeStage;
  return round16(attn_tiles_offset(hd) + (tiles > merge ? tiles : merge));
}

template <int J, typename T, bool kCluster>
__host__ __device__ inline size_t attn_smem_bytes_t(int hd) {
  return attn_bars_offset<J, T, kCluster>(hd) + 8 * TileCfg<J, T>::kRing;
}

// Distributed shared memory: the address of `p` in the shared memory of
// cluster CTA `rank`, a load from it, and a full cluster barrier (release /
// acquire: shared-memory writes before it are visible to every CTA of the
// cluster after it).
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, int rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
  return a;
}

__device__ __forceinline__ float dsmem_ld(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename TT>
__device__ __forceinline__ TT to_tile(float v) {
  if constexpr (sizeof(TT) == 2)
    return __float2half_rn(v);
  else
    return v;
}

__device__ __forceinline__ float2 h2f2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return __half22float2(h);
}

// Requests K/V rows [c0, c0 + kSub) of a cache in its own type into tile
// buffer `buf` ([K rows][V rows], row stride hs elements): warp 0, one bulk
// copy per row and matrix (lane = row), completing on `bar`.  Rows >= t1
// and the current position's row (fused mode) are not copied (zero_rows /
// put_pos_row fill them).
template <typename TT>
__device__ __forceinline__ void issue_tile(uint8_t* buf, uint64_t* bar, const uint8_t* kc, const uint8_t* vc, int c0,
                                           int t1, int pos, bool fused, int kv_dim, size_t kv_off, int hd, int hs,
                                           int lane) {
  const size_t rowb = (size_t)hs * sizeof(TT);
  const uint32_t bytes = (uint32_t)(hd * sizeof(TT));
  const int t = c0 + lane;
  const bool cp = t < t1 && !(fused && t == pos);
  const unsigned rows = __popc(__ballot_sync(0xffffffffu, cp));
  if (lane == 0) mbar_arrive_expect_tx(bar, rows * 2u * bytes);
  __syncwarp();
  if (cp) {
    const size_t off = ((size_t)t * kv_dim + kv_off) * sizeof(TT);
    bulk_load(buf + (size_t)lane * rowb, kc + off, bytes, bar);
    bulk_load(buf + (size_t)(kSub + lane) * rowb, vc + off, bytes, bar);
  }
}

// Zeroes tile rows [t1 - c0, kSub) (positions past the chunk: their scores
// are masked, but P.V reads them).
template <typename TT>
__device__ __forceinline__ void zero_rows(uint8_t* buf, int c0, int t1, int hd, int hs) {
  const int r0 = t1 - c0;
  if (r0 >= kSub) return;
  const int per = hd * (int)sizeof(TT) / 16;
  const size_t rowb = (size_t)hs * sizeof(TT);
  for (int e = threadIdx.x; e < (kSub - r0) * per; e += blockDim.x) {
    const int r = r0 + e / per, p = e % per;
    *reinterpret_cast<uint4*>(buf + (size_t)r * rowb + p * 16) = make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(buf + (size_t)(kSub + r) * rowb + p * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// The current position's row into the tile of sub-chunk [c0, c0 + kSub)
// when it lies there (rounded to the tile type, as the cache stores it).
template <typename TT>
__device__ __forceinline__ void put_pos_row(uint8_t* buf, const float* kpos, const float* vpos, int c0, int t1,
                                            int pos, bool fused, int hd, int hs) {
  if (fused && pos >= c0 && pos < min(t1, c0 + kSub)) {
    TT* kr = reinterpret_cast<TT*>(buf) + (size_t)(pos - c0) * hs;
    TT* vr = kr + (size_t)kSub * hs;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      kr[d] = to_tile<TT>(kpos[d]);
      vr[d] = to_tile<TT>(vpos[d]);
    }
  }
}

// s = sum_d q_d k_d as one sequential fma chain over d.
template <typename TT>
__device__ __forceinline__ float score_row(const float* q, const TT* k, int hd, int hs) {
  float sc = 0.0f;
  if constexpr (sizeof(TT) == 2) {  // hd % 8 == 0, 16-byte aligned rows
    const uint4* k8 = reinterpret_cast<const uint4*>(k);
    const float4* q4 = reinterpret_cast<const float4*>(q);
    for (int i = 0; i < (hd >> 3); ++i) {
      const uint4 u = k8[i];
      const float4 qa = q4[2 * i], qb = q4[2 * i + 1];
      float2 f = h2f2(u.x);
      sc = __fmaf_rn(qa.x, f.x, sc);
      sc = __fmaf_rn(qa.y, f.y, sc);
      f = h2f2(u.y);
      sc = __fmaf_rn(qa.z, f.x, sc);
      sc = __fmaf_rn(qa.w, f.y, sc);
      f = h2f2(u.z);
      sc = __fmaf_rn(qb.x, f.x, sc);
      sc = __fmaf_rn(qb.y, f.y, sc);
      f = h2f2(u.w);
      sc = __fmaf_rn(qb.z, f.x, sc);
      sc = __fmaf_rn(qb.w, f.y, sc);
    }
  } else {
    if ((hs & 3) == 0 && (hd & 3) == 0) {
      const float4* k4 = reinterpret_cast<const float4*>(k);
      const float4* q4 = reinterpret_cast<const float4*>(q);
      for (int i = 0; i < (hd >> 2); ++i) {
        const float4 kv = k4[i], qv = q4[i];
        sc = __fmaf_rn(qv.x, kv.x, sc);
        sc = __fmaf_rn(qv.y, kv.y, sc);
        sc = __fmaf_rn(qv.z, kv.z, sc);
        sc = __fmaf_rn(qv.w, kv.w, sc);
      }
    } else {
      for (int d = 0; d < hd; ++d) sc = __fmaf_rn(q[d], k[d], sc);
    }
  }
  return sc;
}

// J consecutive values of a V row (as f32).
template <int J, typename TT>
__device__ __forceinline__ void load_v(const TT* vr, float (&v)[J]) {
  if constexpr (sizeof(TT) == 2) {
    if constexpr (J == 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(vr);
      float2 f = h2f2(u.x); v[0] = f.x; v[1] = f.y;
      f = h2f2(u.y); v[2] = f.x; v[3] = f.y;
      f = h2f2(u.z); v[4] = f.x; v[5] = f.y;
      f = h2f2(u.w); v[6] = f.x; v[7] = f.y;
    } else if constexpr (J == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(vr);
      float2 f = h2f2(u.x); v[0] = f.x; v[1] = f.y;
      f = h2f2(u.y); v[2] = f.x; v[3] = f.y;
    } else {
      static_assert(J == 2, "f16 tiles serve J >= 2");
      const float2 f = h2f2(*reinterpret_cast<const uint32_t*>(vr));
      v[0] = f.x; v[1] = f.y;
    }
  } else {
    if constexpr (J % 4 == 0) {
#pragma unroll
      for (int j = 0; j < J; j += 4) {
        const float4 f = *reinterpret_cast<const float4*>(vr + j);
        v[j] = f.x; v[j + 1] = f.y; v[j + 2] = f.z; v[j + 3] = f.w;
      }
    } else if constexpr (J == 2) {
      const float2 f = *reinterpret_cast<const float2*>(vr);
      v[0] = f.x; v[1] = f.y;
    } else {
#pragma unroll
      for (int j = 0; j < J; ++j) v[j] = vr[j];
    }
  }
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
//
// kCluster: the a.n_split CTAs of a kv head are one thread-block cluster;
// each keeps its partial (m, l, acc) in shared memory and, after a cluster
// barrier, merges 32-value units of the kv head's output (unit u on CTA
// u mod n_split) reading every split's partial through distributed shared
// memory -- no global scratch, no atomics, no second pass over global
// memory.  Every thread of every CTA reaches both cluster barriers.
template <int J, typename T, bool kCluster>
__global__ void __launch_bounds__(kAttnWarps * 32) k_attention(const AttnArgs a) {
  using C = TileCfg<J, T>;
  using TT = typename C::TT;
  constexpr int NT = C::kRing;
  extern __shared__ __align__(16) uint8_t smem_b[];
  const int hd = a.head_dim;
  const int hs = C::stride(hd);
  float* s_q = reinterpret_cast<float*>(smem_b);  // [kGMax][hd]; the merged rows after the merge
  float* s_kpos = s_q + kGMax * hd;
  float* s_vpos = s_kpos + hd;
  float* s_sq = s_vpos + hd;  // [kAttnWarps][256]
  uint8_t* s_tiles = smem_b + attn_tiles_offset(hd);
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem_b + attn_bars_offset<J, T, kCluster>(hd));
  const size_t buf_bytes = C::buf_bytes(hd);

  const int kvh = blockIdx.x, split = blockIdx.y, z = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hb = (kvh * a.n_head + a.n_kv - 1) / a.n_kv;
  const int he = ((kvh + 1) * a.n_head + a.n_kv - 1) / a.n_kv;
  const int G = he - hb;
  const float* qp = a.q + (size_t)z * a.qkv_bstride;
  const uint8_t* kc = static_cast<const uint8_t*>(a.k_cache) + (size_t)z * a.cache_bstride * sizeof(T);
  const uint8_t* vc = static_cast<const uint8_t*>(a.v_cache) + (size_t)z * a.cache_bstride * sizeof(T);
  float* outp = a.out + (size_t)z * a.out_bstride;
  uint8_t* oq8 = a.out_q8 ? a.out_q8 + (size_t)z * a.outq8_bstride : nullptr;
  const int pos = a.pos_ptr ? a.pos_ptr[(size_t)z * (a.pos_stride > 0 ? a.pos_stride : 1)] : a.pos_static;
  const int n_pos = pos + 1;
  int chunk = (n_pos + a.n_split - 1) / a.n_split;
  if (chunk < 32) chunk = 32;
  const int n_active = (n_pos + chunk - 1) / chunk;
  const int t0 = split * chunk;
  const int t1 = min(t0 + chunk, n_pos);
  const int nsub = split < n_active ? (t1 - t0 + kSub - 1) / kSub : 0;
  const int kv_dim = a.n_kv * hd;
  const size_t kv_off = (size_t)kvh * hd;
  const int stride_part = attn_part_stride(hd);
  const bool fused = a.fuse_norm_rope_append != 0;
  const bool active = nsub > 0;
  const int nt = blockDim.x;

  // Before waiting for the previous kernel (programmatic dependent launch):
  // everything that only depends on earlier steps -- the position, the K/V
  // rows of earlier positions of the first NT-1 sub-chunks (the current
  // position comes from this kernel's prologue), and the norm weight and
  // RoPE lines (into L1).
  if constexpr (C::kAsync) {
    if (warp == 0) {
      if (lane == 0) {
#pragma unroll
        for (int b = 0; b < NT; ++b) mbar_init(&s_bar[b], 1);
        mbar_fence_init();
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < NT - 1; ++i)
        if (i < nsub)
          issue_tile<TT>(s_tiles + i * buf_bytes, &s_bar[i], kc, vc, t0 + i * kSub, t1, pos, fused, kv_dim, kv_off, hd,
                         hs, lane);
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

  // Every global load of the prologue first: K/V of the current position
  // (fused: normalised/rotated here; needed by split 0, which appends it,
  // and by the split that holds position pos) on warps 0/1, and each warp's
  // q rows of this kv head's group; then the stores and the norms.
  const bool kv_split = fused && (split == 0 || split == n_active - 1) && warp < 2;
  float kvr[8];
  float qv[2][8];
  if (kv_split) {
    const float* src = (warp == 0 ? a.k : a.v) + (size_t)z * a.qkv_bstride + kv_off;
#pragma unroll
    for (int k = 0; k < 8; ++k) kvr[k] = lane + 32 * k < hd ? src[lane + 32 * k] : 0.0f;
  }
  if (active) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int g = warp + i * kAttnWarps;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int d = lane + 32 * k;
        qv[i][k] = (g < G && d < hd) ? qp[(size_t)(hb + g) * hd + d] : 0.0f;
      }
    }
  }
  if (kv_split) {
    float* dst = warp == 0 ? s_kpos : s_vpos;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (lane + 32 * k < hd) dst[lane + 32 * k] = kvr[k];
  }
  if (active) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int g = warp + i * kAttnWarps;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int d = lane + 32 * k;
        if (g < G && d < hd) s_q[g * hd + d] = qv[i][k];
      }
    }
  }
  __syncwarp();
  if (kv_split && warp == 0)
    norm_rope_row(s_kpos, s_sq, hd, a.k_norm, a.k_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base, a.rope_scale,
                  pos, lane);
  for (int g = warp; active && g < G; g += kAttnWarps) {
    float* row = s_q + g * hd;
    if (fused)
      norm_rope_row(row, s_sq + warp * 256, hd, a.q_norm, a.q_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base,
                    a.rope_scale, pos, lane);
  }
  __syncthreads();
  if (fused && split == 0) {
    void* kw = const_cast<uint8_t*>(kc);
    void* vw = const_cast<uint8_t*>(vc);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      kv_store<T>(kw, (size_t)pos * kv_dim + kv_off + d, s_kpos[d]);
      kv_store<T>(vw, (size_t)pos * kv_dim + kv_off + d, s_vpos[d]);
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
    for (int i = 0; i < nsub; ++i) {
      const int c0 = t0 + i * kSub;
      uint8_t* buf = s_tiles + (size_t)(i % NT) * buf_bytes;
      if constexpr (C::kAsync) {
        // request the tile NT-1 ahead into the buffer the previous
        // iteration finished with, then complete this one
        if (warp == 0 && i + NT - 1 < nsub)
          issue_tile<TT>(s_tiles + (size_t)((i + NT - 1) % NT) * buf_bytes, &s_bar[(i + NT - 1) % NT], kc, vc,
                         c0 + (NT - 1) * kSub, t1, pos, fused, kv_dim, kv_off, hd, hs, lane);
        put_pos_row<TT>(buf, s_kpos, s_vpos, c0, t1, pos, fused, hd, hs);
        zero_rows<TT>(buf, c0, t1, hd, hs);
        mbar_wait(&s_bar[i % NT], (uint32_t)(i / NT) & 1u, a.err);
      } else {
        float* kt = reinterpret_cast<float*>(buf);
        stage_kv_tile<T>(kc, vc, s_kpos, s_vpos, kt, kt + (size_t)kSub * hs, c0, t1, pos, fused, kv_dim, kv_off, hd,
                         hs, threadIdx.x, nt);
      }
      __syncthreads();
      const TT* ktile = reinterpret_cast<const TT*>(buf);
      const TT* vtile = ktile + (size_t)kSub * hs;
      const int t = c0 + lane;
      const bool valid = t < t1;
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int g = warp + hi * kAttnWarps;
        if (g >= G) break;
        float sc = score_row<TT>(s_q + g * hd, ktile + (size_t)lane * hs, hd, hs);
        sc = valid ? __fmul_rn(sc, a.scale) : -INFINITY;
        const float mx = warp_max(sc);
        const float mn = fmaxf(m[hi], mx);
        const float alpha = expf_det(__fsub_rn(m[hi], mn));
        const float p = valid ? expf_det(__fsub_rn(sc, mn)) : 0.0f;
        const float psum = __shfl_sync(0xffffffffu, warp_sum(p), 0);
        l[hi] = __fadd_rn(__fmul_rn(l[hi], alpha), psum);
        m[hi] = mn;
#pragma unroll
        for (int j = 0; j < J; ++j) acc[hi][j] = __fmul_rn(acc[hi][j], alpha);
        for (int tt = 0; tt < kSub; ++tt) {
          const float pt = __shfl_sync(0xffffffffu, p, tt);
          if (act) {
            float vv[J];
            load_v<J, TT>(vtile + (size_t)tt * hs + lane * J, vv);
#pragma unroll
            for (int j = 0; j < J; ++j) acc[hi][j] = __fmaf_rn(pt, vv[j], acc[hi][j]);
          }
        }
      }
      __syncthreads();
    }
    float* part_base = kCluster ? reinterpret_cast<float*>(s_tiles)
                                : a.partial + ((size_t)z * a.n_head + hb) * a.n_split * stride_part;
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      const int g = warp + hi * kAttnWarps;
      if (g >= G) break;
      float* dst = kCluster ? part_base + (size_t)g * stride_part
                            : part_base + ((size_t)g * a.n_split + split) * stride_part;
      if (act)
#pragma unroll
        for (int j = 0; j < J; ++j) dst[4 + lane * J + j] = acc[hi][j];
      if (lane == 0) {
        dst[0] = m[hi];
        dst[1] = l[hi];
      }
    }
  }

  if constexpr (kCluster) {
    // Every split's partial rows are in its shared memory (tile area).  Unit
    // u (32 consecutive output values of this kv head's G heads) is merged
    // by warp (u / n_split) mod 4 of CTA u mod n_split, lane = value:
    // M = max_s m_s, w_s = exp(m_s - M), L = sum_s w_s l_s and
    // o = sum_s w_s acc_s (fma chains in split order), o * (1/L).
    cluster_sync_all();
    const int S = a.n_split;
    const int n_units = (G * hd + 31) / 32;
    const float* part_s = reinterpret_cast<const float*>(s_tiles);
    for (int u = split + S * warp; u < n_units; u += S * kAttnWarps) {
      const int e = u * 32 + lane;
      const bool ve = e < G * hd;
      const int g = ve ? e / hd : 0, d = ve ? e - g * hd : 0;
      const float* row = part_s + (size_t)g * stride_part;
      float av[kAttnMaxCluster];
#pragma unroll
      for (int sp = 0; sp < kAttnMaxCluster; ++sp) av[sp] = sp < n_active ? dsmem_ld(dsmem_addr(row + 4 + d, sp)) : 0.0f;
      float L = 0.0f, o = 0.0f;
      if ((hd & 31) == 0) {
        // one head per unit: lane sp holds split sp's (m, l) and weight
        // w_sp = exp(m_sp - M); the sums run in split order via shuffles
        const float* hrow = part_s + (size_t)(u * 32 / hd) * stride_part;
        const float msp = lane < n_active ? dsmem_ld(dsmem_addr(hrow, lane)) : -INFINITY;
        const float lsp = lane < n_active ? dsmem_ld(dsmem_addr(hrow + 1, lane)) : 0.0f;
        const float M = warp_max(msp);
        const float wsp = lane < n_active ? expf_det(__fsub_rn(msp, M)) : 0.0f;
#pragma unroll
        for (int sp = 0; sp < kAttnMaxCluster; ++sp) {
          const float w = __shfl_sync(0xffffffffu, wsp, sp);
          const float ls = __shfl_sync(0xffffffffu, lsp, sp);
          if (sp < n_active) {
            L = __fmaf_rn(w, ls, L);
            o = __fmaf_rn(w, av[sp], o);
          }
        }
      } else {  // small heads: a unit spans several heads, each lane its own
        float ms[kAttnMaxCluster], ls[kAttnMaxCluster];
#pragma unroll
        for (int sp = 0; sp < kAttnMaxCluster; ++sp) {
          ms[sp] = sp < n_active ? dsmem_ld(dsmem_addr(row, sp)) : -INFINITY;
          ls[sp] = sp < n_active ? dsmem_ld(dsmem_addr(row + 1, sp)) : 0.0f;
        }
        float M = -INFINITY;
#pragma unroll
        for (int sp = 0; sp < kAttnMaxCluster; ++sp)
          if (sp < n_active) M = fmaxf(M, ms[sp]);
#pragma unroll
        for (int sp = 0; sp < kAttnMaxCluster; ++sp) {
          if (sp < n_active) {
            const float w = expf_det(__fsub_rn(ms[sp], M));
            L = __fmaf_rn(w, ls[sp], L);
            o = __fmaf_rn(w, av[sp], o);
          }
        }
      }
      o = __fmul_rn(o, L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f);
      if (ve) outp[(size_t)hb * hd + e] = o;
      if (oq8 && (hd % 32) == 0) {
        uint16_t dbits;
        bool zero;
        const int q = q8_1_quant_lane(o, &dbits, &zero);
        uint32_t word = ((uint32_t)(q & 0xff)) << (8 * (lane & 3));
        word |= __shfl_xor_sync(0xffffffffu, word, 1);
        word |= __shfl_xor_sync(0xffffffffu, word, 2);
        float sum = 0.0f;  // the sequential f16 s of the reference block
        for (int t = 0; t < 32; ++t) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, o, t));
        uint32_t* ob = reinterpret_cast<uint32_t*>(oq8 + ((size_t)hb * hd / 32 + u) * 36);
        if (lane == 0) ob[0] = (uint32_t)dbits | ((uint32_t)(zero ? (uint16_t)0 : f32_to_f16_ref(sum)) << 16);
        if ((lane & 3) == 0) ob[1 + (lane >> 2)] = word;
      }
    }
    cluster_sync_all();  // no CTA leaves while another still reads its partials
    return;
  }

  // last CTA of this kv head merges the splits: the CTA barrier orders every
  // thread's partial stores before thread 0's acquire-release ticket
  __shared__ unsigned ticket_s;
  unsigned* counter = a.counters + (size_t)z * a.n_kv + kvh;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(counter) : "memory");
    ticket_s = t;
  }
  __syncthreads();
  if (ticket_s != (unsigned)(a.n_split - 1)) return;
  if (threadIdx.x == 0) atomicExch(counter, 0u);
  // Merge: (1) m and l of all (head, split) pairs -- with every split's
  // partial row copied into shared memory in one round trip when they fit
  // (L2-only async copies); (2) per head M = max m, w_s = exp(m_s - M) and
  // L = sum_s w_s l_s (fma in split order); (3) o_d = sum_s w_s acc_sd (fma in
  // split order) * (1/L) by one thread per (head, d); (4) Q8_1 blocks of the
  // output, one warp per block.
  const float* part_g = a.partial + ((size_t)z * a.n_head + hb) * a.n_split * stride_part;
  float* cm = reinterpret_cast<float*>(s_tiles);
  float* cl = cm + kGMax * kMaxSplit;
  float* cw = cl + kGMax * kMaxSplit;
  float* cinv = cw + kGMax * kMaxSplit;
  float* mp = reinterpret_cast<float*>(s_tiles + attn_merge_stage_offset());
  const bool staged = (size_t)G * n_active * stride_part <= (size_t)kMergeStage;
  if (staged) {
    const int per = stride_part / 4;  // 16-byte pieces per partial row
    for (int i = threadIdx.x; i < G * n_active * per; i += nt) {
      const int row = i / per, c = i - row * per;
      const int g = row / n_active, sp = row - g * n_active;
      cp_async16(mp + (size_t)row * stride_part + c * 4, part_g + ((size_t)g * a.n_split + sp) * stride_part + c * 4);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    for (int i = threadIdx.x; i < G * n_active; i += nt) {
      const int g = i / n_active, sp = i - g * n_active;
      cm[g * kMaxSplit + sp] = mp[(size_t)i * stride_part];
      cl[g * kMaxSplit + sp] = mp[(size_t)i * stride_part + 1];
    }
  } else {
    for (int i = threadIdx.x; i < G * n_active; i += nt) {
      const int g = i / n_active, sp = i - g * n_active;
      const float* ps = part_g + ((size_t)g * a.n_split + sp) * stride_part;
      cm[g * kMaxSplit + sp] = __ldcg(ps);
      cl[g * kMaxSplit + sp] = __ldcg(ps + 1);
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += kAttnWarps) {
    const float* mg = cm + g * kMaxSplit;
    float M = -INFINITY;
    for (int sp = lane; sp < n_active; sp += 32) M = fmaxf(M, mg[sp]);
    M = warp_max(M);
    for (int sp = lane; sp < n_active; sp += 32) cw[g * kMaxSplit + sp] = expf_det(__fsub_rn(mg[sp], M));
    __syncwarp();
    if (lane == 0) {
      float L = 0.0f;
      for (int sp = 0; sp < n_active; ++sp) L = __fmaf_rn(cw[g * kMaxSplit + sp], cl[g * kMaxSplit + sp], L);
      cinv[g] = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
    }
  }
  __syncthreads();
  constexpr int kLd = 16;
  for (int i = threadIdx.x; i < G * hd; i += nt) {
    const int g = i / hd, d = i - g * hd;
    const float* wg = cw + g * kMaxSplit;
    float o = 0.0f;
    if (staged) {
      const float* pg = mp + (size_t)g * n_active * stride_part + 4 + d;
      for (int sp = 0; sp < n_active; ++sp) o = __fmaf_rn(wg[sp], pg[(size_t)sp * stride_part], o);
    } else {
      const float* pg = part_g + (size_t)g * a.n_split * stride_part + 4 + d;
      for (int s0 = 0; s0 < n_active; s0 += kLd) {
        float r[kLd];
#pragma unroll
        for (int u = 0; u < kLd; ++u) r[u] = s0 + u < n_active ? __ldcg(pg + (size_t)(s0 + u) * stride_part) : 0.0f;
#pragma unroll
        for (int u = 0; u < kLd; ++u)
          if (s0 + u < n_active) o = __fmaf_rn(wg[s0 + u], r[u], o);
      }
    }
    o = __fmul_rn(o, cinv[g]);
    outp[(size_t)(hb + g) * hd + d] = o;
    s_q[i] = o;
  }
  if (oq8 && (hd % 32) == 0) {
    __syncthreads();
    for (int b = warp; b < G * hd / 32; b += kAttnWarps) {
      const float o = s_q[b * 32 + lane];
      uint16_t dbits;
      bool zero;
      const int q = q8_1_quant_lane(o, &dbits, &zero);
      uint32_t word = ((uint32_t)(q & 0xff)) << (8 * (lane & 3));
      word |= __shfl_xor_sync(0xffffffffu, word, 1);
      word |= __shfl_xor_sync(0xffffffffu, word, 2);
      uint32_t* ob = reinterpret_cast<uint32_t*>(oq8 + ((size_t)hb * hd + (size_t)b * 32) / 32 * 36);
      if (lane == 0) {
        float sum = 0.0f;  // the sequential f16 s of the reference block
        for (int t = 0; t < 32; ++t) sum = __fadd_rn(sum, s_q[b * 32 + t]);
        ob[0] = (uint32_t)dbits | ((uint32_t)(zero ? (uint16_t)0 : f32_to_f16_ref(sum)) << 16);
      }
      if ((lane & 3) == 0) ob[1 + (lane >> 2)] = word;
    }
  }
}

// Cluster launch: grid (n_kv, n_split, batch) in clusters of (1, n_split, 1),
// with programmatic dependent launch when pdl is set.
template <typename Kern>
cudaError_t launch_cluster(Kern kernel, dim3 grid, int cluster_y, size_t smem, cudaStream_t st, bool pdl,
                           const AttnArgs& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)cluster_y;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

// Whether clusters of n CTAs of a kernel can be resident, queried once at
// set-up per device; the cluster merge is launched only where they can
// (otherwise the global-memory merge, with the same bits, is used).
constexpr int kMaxDevices = 64;
bool g_cluster_ok[kMaxDevices][2][4][kAttnMaxCluster + 1];  // [device][f16][J index][cluster size]

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}

template <typename Kern>
bool query_cluster(Kern kernel, size_t smem, int n) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, n, 1);
  cfg.blockDim = dim3(kAttnWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)n;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return clusters > 0;
}

constexpr int j_index(int J) { return J == 1 ? 0 : J == 2 ? 1 : J == 4 ? 2 : 3; }

template <int J, typename T>
cudaError_t init_jt(int dev) {
  const size_t mx = attn_smem_bytes_t<J, T, false>(32 * J);
  const size_t mc = attn_smem_bytes_t<J, T, true>(32 * J);
  cudaError_t e = cudaFuncSetAttribute(k_attention<J, T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mx);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_attention<J, T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mc);
  if (e != cudaSuccess) return e;
  const bool nonportable =
      cudaFuncSetAttribute(k_attention<J, T, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  if (!nonportable) (void)cudaGetLastError();
  for (int n = 1; n <= kAttnMaxCluster; ++n)
    g_cluster_ok[dev][sizeof(T) == 2][j_index(J)][n] =
        (n <= 8 || nonportable) && query_cluster(k_attention<J, T, true>, mc, n);
  return cudaSuccess;
}

template <int J>
cudaError_t launch_j(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int hd = a.head_dim;
  const dim3 grid(a.n_kv, a.n_split, a.batch > 0 ? a.batch : 1);
  const bool f16 = a.kv_f16 != 0;
  const int dev = a.cluster ? current_device() : -1;
  if (dev >= 0 && g_cluster_ok[dev][f16][j_index(J)][a.n_split]) {
    if (f16)
      return launch_cluster(k_attention<J, __half, true>, grid, a.n_split, attn_smem_bytes_t<J, __half, true>(hd), st,
                            pdl, a);
    return launch_cluster(k_attention<J, float, true>, grid, a.n_split, attn_smem_bytes_t<J, float, true>(hd), st, pdl,
                          a);
  }
  if (!a.partial || !a.counters) return cudaErrorInvalidValue;
  if (f16)
    return launch_k(k_attention<J, __half, false>, grid, dim3(kAttnWarps * 32), attn_smem_bytes_t<J, __half, false>(hd),
                    st, pdl, a);
  return launch_k(k_attention<J, float, false>, grid, dim3(kAttnWarps * 32), attn_smem_bytes_t<J, float, false>(hd), st,
                  pdl, a);
}

template <int J>
cudaError_t init_j(int dev) {
  cudaError_t e = init_jt<J, float>(dev);
  if (e == cudaSuccess) e = init_jt<J, __half>(dev);
  return e;
}

}  // namespace

size_t attn_partial_floats(int n_head, int n_split, int head_dim) {
  return (size_t)n_head * n_split * attn_part_stride(head_dim);
}

cudaError_t attention_init() {
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  cudaError_t e = init_j<1>(dev);
  if (e == cudaSuccess) e = init_j<2>(dev);
  if (e == cudaSuccess) e = init_j<4>(dev);
  if (e == cudaSuccess) e = init_j<8>(dev);
  return e;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.n_split > kMaxSplit || a.n_split < 1) return cudaErrorInvalidValue;
  if (a.cluster && a.n_split > kAttnMaxCluster) return cudaErrorInvalidValue;
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
