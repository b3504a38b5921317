// attention.cu -- single-query (decode) causal GQA attention for sm_100a.
//
// Semantics (src/minicpmo/qwen3.uya:1664-1713, gpu_shim.c:926-979): for q
// head h the kv head is (h*n_kv)/n_head; scores = q.k_t * scale for t <= pos,
// softmax over t, out = sum_t p_t v_t.  KV cache layout [layer][pos][kv_dim]
// as the reference (qwen3.uya:1664-1666), f32 (reference) or f16.
//
// Arithmetic (the device order, restated by the oracle): positions are cut
// into blocks of 32.  For every q head and block c, with lane = position:
//   s_t = scale * sum_d q_d k_td          (one sequential fma chain over d)
//   m_c = max_t s_t,  p_t = exp(s_t - m_c) (0 past the last position)
//   l_c = butterfly_sum(p),  acc_c,d = sum_t p_t v_td  (fma in t order)
// and the blocks merge in block order:
//   M = max_c m_c,  w_c = exp(m_c - M),  L = sum_c w_c l_c,
//   o_d = (sum_c w_c acc_c,d) * (1/L)      (fma chains in c order).
//
// B200 design: grid = (n_kv, n_split, batch); the n_split CTAs of a kv head
// take its blocks round-robin, and inside a CTA eight warps work on (head,
// block) pairs side by side, so a 600-position context is one round of
// work.  K/V tiles reach shared memory in the cache's own type by 2-D TMA
// tensor copies issued by one thread (a layer's cache is a [rows][kv_dim]
// tensor map, boxes of 32 positions x 128 bytes in the 128-byte swizzle), a
// ring of 32-position tiles on mbarriers; the first round's tiles are
// requested before the kernel waits for its predecessor (programmatic
// dependent launch), and no other thread spends issue slots on copies.  The block partials merge either inside a thread-block
// cluster -- each warp stores its block's values straight into the shared
// memory of the CTA that merges each 32-value output unit, so the merge
// reads only local shared memory (the default of the single-sequence
// decode graph) -- or through global memory by the last-arriving CTA
// (atomic ticket; the batched decode); both give the same bits.  The merge
// writes the f32 output and, optionally, its Q8_1 blocks for the
// o-projection.
//
// Fused mode also performs, for the current position, the per-head
// QK-RMSNorm (qwen3.uya:1543-1558, eps 1e-6, reduction order of
// gpu_shim.c:719-745 with an exact 1/sqrtf), NeoX RoPE from the host-built
// cos/sin table (qwen3.uya:1605-1662) and the KV append
// (qwen3.uya:1668-1675), so q/k never round-trip through separate kernels.
// The current position is attended as the cache stores it (f16: rounded).
#include "attention.cuh"

#include <cuda.h>
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

constexpr int kAttnWarps = 8;
constexpr int kGMax = 8;  // q heads per kv head handled by one CTA
constexpr int kMaxSplit = 64;
constexpr int kMaxBlocks = 4096;  // blocks per sequence (131072 positions)

// Small odd head sizes (J = 1, head_dim <= 32) stage f32 tiles through
// registers with this row stride.
__host__ __device__ inline int attn_tile_stride(int hd) { return (hd & 3) ? hd + 1 : hd + 4; }

// Tile geometry of one instantiation.  J >= 2 (head_dim 64/128/256): tiles
// in the cache type TT brought in by TMA tensor copies, each 32-position K
// (or V) tile head_dim*sizeof(TT)/128 boxes of 32 rows x 128 bytes in the
// 128-byte swizzle (16-byte chunk c of row r stored at chunk c ^ (r & 7),
// so lanes reading rows lane hit distinct banks per quarter warp), a ring
// of kRing tiles.  J = 1: one f32 tile staged through registers.
template <int J, typename T>
struct TileCfg {
  static constexpr bool kAsync = J >= 2;
  using TT = std::conditional_t<kAsync, T, float>;
  static constexpr int kRing = (kAsync && (sizeof(T) == 2 || J < 8)) ? 4 : 2;
  __host__ __device__ static int stride(int hd) { return attn_tile_stride(hd); }  // J = 1
  __host__ __device__ static size_t buf_bytes(int hd) {
    return kAsync ? 2 * (size_t)kSub * hd * sizeof(TT) : 2 * (size_t)kSub * attn_tile_stride(hd) * sizeof(float);
  }
};

__host__ __device__ inline size_t round16(size_t b) { return (b + 15) & ~(size_t)15; }

// Blocks a CTA computes per round: one warp per (head, block), at most
// half the tile ring (the next round's tiles load meanwhile).
template <int J, typename T>
__host__ __device__ inline int attn_bpr(int G) {
  const int b = kAttnWarps / G, h = TileCfg<J, T>::kRing / 2;
  return b < 1 ? 1 : (b < h ? b : h);
}

// Tile buffers a CTA uses when the CTAs of a kv head hold at most nb_cta
// blocks each: every block its own buffer when two rounds cover them, else
// two rounds' worth in turn.  The shared-memory carve-up uses the group
// size g_min = n_head / n_kv (the most blocks per round of any kv head).
template <int J, typename T>
__host__ __device__ inline int attn_ring(int g, int nb_cta) {
  const int r = 2 * attn_bpr<J, T>(g);
  return nb_cta < 1 ? 1 : (nb_cta < r ? nb_cta : r);
}

// Cluster merge: the CTA that merges a 32-value output unit receives, for
// every block c of the context, that unit's 32 accumulator values and the
// block's (m, l) in one row of kMergeRow floats (16-byte rows).
constexpr int kMergeRow = 36;

// Shared memory: q [kGMax][hd], kpos [hd], vpos [hd], norm scratch
// [kAttnWarps][256] (f32), `ring` tile buffers, the cluster path's merge
// rows [slots][attn_n_blocks(ctx)][kMergeRow] (f32), one mbarrier per tile
// buffer.
__host__ __device__ inline size_t attn_tiles_offset(int hd) {  // 1024-aligned (swizzle atoms)
  return (sizeof(float) * ((size_t)kGMax * hd + 2 * (size_t)hd + kAttnWarps * 256) + 1023) & ~(size_t)1023;
}

template <int J, typename T>
__host__ __device__ inline size_t attn_parts_offset(int hd, int ring) {
  return attn_tiles_offset(hd) + (size_t)ring * TileCfg<J, T>::buf_bytes(hd);
}

template <int J, typename T>
__host__ __device__ inline size_t attn_bars_offset(int hd, int ring, int merge_rows) {
  return round16(attn_parts_offset<J, T>(hd, ring) + sizeof(float) * (size_t)merge_rows * kMergeRow);
}

template <int J, typename T>
__host__ __device__ inline size_t attn_smem_bytes_t(int hd, int ring, int merge_rows) {
  // + 1024: the kernel aligns its base to 1024 bytes
  return attn_bars_offset<J, T>(hd, ring, merge_rows) + 8 * (size_t)ring + 1024;
}

// The layout of one launch (kernel and host compute it alike): a unit u of
// a kv head's G * hd / 32 is merged by CTA u mod n_split in its slot
// u / n_split.
struct AttnLayout {
  int ring, merge_rows;
};

template <int J, typename T>
__host__ __device__ inline AttnLayout attn_layout(int hd, int n_head, int n_kv, int ctx, int n_split, bool cluster) {
  const int nb_cta = (attn_n_blocks(ctx) + n_split - 1) / n_split;
  const int g_min = n_head / n_kv > 0 ? n_head / n_kv : 1;
  const int g_max = (n_head + n_kv - 1) / n_kv;
  const int slots = (g_max * (hd / 32) + n_split - 1) / n_split;
  AttnLayout l;
  l.ring = attn_ring<J, T>(g_min, nb_cta);
  l.merge_rows = cluster ? slots * attn_n_blocks(ctx) : 0;
  return l;
}

// Distributed shared memory: the address of `p` in the shared memory of
// cluster CTA `rank`, stores to it, and a full cluster barrier (release /
// acquire: shared-memory writes before it are visible to every CTA of the
// cluster after it).
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, int rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
  return a;
}

__device__ __forceinline__ void dsmem_st4(uint32_t a, float x, float y, float z, float w) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}

__device__ __forceinline__ void dsmem_st2(uint32_t a, float x, float y) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(x), "f"(y) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
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

// Byte offset of byte `byte` of row r (0..31) in a swizzled K or V tile.
__device__ __forceinline__ uint32_t sw_off(int r, int byte) {
  return (uint32_t)((byte >> 7) * 4096 + r * 128 + ((((byte >> 4) & 7) ^ (r & 7)) << 4) + (byte & 15));
}

// One 2-D TMA tensor copy (no multicast) of the box at element (x, y) of
// `map` into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Requests the K and V tiles of positions [y, y + 32) of the maps' rows,
// columns [x0, x0 + head_dim), into tile buffer `buf` ([K boxes][V boxes]):
// one thread, 2 * head_dim*sizeof(TT)/128 copies completing on `bar`.  Rows
// past the map read as zero; rows past the current position and the current
// position's row (fused mode) are rewritten after the wait.
template <typename TT>
__device__ __forceinline__ void issue_tile(uint8_t* buf, uint64_t* bar, const CUtensorMap* km, const CUtensorMap* vm,
                                           int x0, int y, int hd) {
  const int nbox = hd * (int)sizeof(TT) / 128, per = 128 / (int)sizeof(TT);
  mbar_arrive_expect_tx(bar, (uint32_t)(2 * nbox * 4096));
  for (int j = 0; j < nbox; ++j) {
    tma_load_2d(buf + j * 4096, km, x0 + j * per, y, bar);
    tma_load_2d(buf + (nbox + j) * 4096, vm, x0 + j * per, y, bar);
  }
}

// Zeroes rows [t1 - c0, kSub) of a landed tile (positions past the current
// one: their scores are masked, but P.V reads them).
template <typename TT>
__device__ __forceinline__ void zero_rows(uint8_t* buf, int c0, int t1, int hd) {
  const int r0 = t1 - c0;
  if (r0 >= kSub) return;
  const int nr = kSub - r0, nbox2 = 2 * hd * (int)sizeof(TT) / 128;
  for (int e = threadIdx.x; e < nbox2 * nr * 8; e += blockDim.x) {
    const int box = e / (nr * 8), rem = e - box * (nr * 8), r = r0 + (rem >> 3), ch = rem & 7;
    *reinterpret_cast<uint4*>(buf + box * 4096 + r * 128 + ch * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// The current position's row into a landed tile of [c0, c0 + kSub) when it
// lies there (rounded to the tile type, as the cache stores it).
template <typename TT>
__device__ __forceinline__ void put_pos_row(uint8_t* buf, const float* kpos, const float* vpos, int c0, int pos,
                                            bool fused, int hd) {
  if (fused && pos >= c0 && pos < c0 + kSub) {
    const int r = pos - c0;
    uint8_t* vb = buf + (size_t)kSub * hd * sizeof(TT);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      const uint32_t o = sw_off(r, d * (int)sizeof(TT));
      *reinterpret_cast<TT*>(buf + o) = to_tile<TT>(kpos[d]);
      *reinterpret_cast<TT*>(vb + o) = to_tile<TT>(vpos[d]);
    }
  }
}

// s = sum_d q_d k_d over row r of a swizzled K tile (head_dim HD), one
// sequential fma chain over d; the loads run two 16-byte chunks ahead of
// the chain.
template <typename TT, int HD>
__device__ __forceinline__ float score_row_sw(const float* q, const uint8_t* kt, int r) {
  constexpr int nch = HD * (int)sizeof(TT) / 16;  // 16-byte chunks of the row
  constexpr int QPC = sizeof(TT) == 2 ? 2 : 1;    // q float4s per chunk
  constexpr int GRP = 2;
  static_assert(nch % GRP == 0, "whole chunk groups");
  const float4* q4 = reinterpret_cast<const float4*>(q);
  uint4 kc[GRP];
  float4 qc[GRP * QPC];
#pragma unroll
  for (int u = 0; u < GRP; ++u) kc[u] = *reinterpret_cast<const uint4*>(kt + sw_off(r, u * 16));
#pragma unroll
  for (int u = 0; u < GRP * QPC; ++u) qc[u] = q4[u];
  float sc = 0.0f;
#pragma unroll
  for (int g = 0; g < nch / GRP; ++g) {
    uint4 kn[GRP];
    float4 qn[GRP * QPC];
    if (g + 1 < nch / GRP) {
#pragma unroll
      for (int u = 0; u < GRP; ++u) kn[u] = *reinterpret_cast<const uint4*>(kt + sw_off(r, ((g + 1) * GRP + u) * 16));
#pragma unroll
      for (int u = 0; u < GRP * QPC; ++u) qn[u] = q4[(g + 1) * GRP * QPC + u];
    }
#pragma unroll
    for (int u = 0; u < GRP; ++u) {
      const uint4 k = kc[u];
      if constexpr (sizeof(TT) == 2) {
        const float4 qa = qc[2 * u], qb = qc[2 * u + 1];
        float2 f = h2f2(k.x);
        sc = __fmaf_rn(qa.x, f.x, sc);
        sc = __fmaf_rn(qa.y, f.y, sc);
        f = h2f2(k.y);
        sc = __fmaf_rn(qa.z, f.x, sc);
        sc = __fmaf_rn(qa.w, f.y, sc);
        f = h2f2(k.z);
        sc = __fmaf_rn(qb.x, f.x, sc);
        sc = __fmaf_rn(qb.y, f.y, sc);
        f = h2f2(k.w);
        sc = __fmaf_rn(qb.z, f.x, sc);
        sc = __fmaf_rn(qb.w, f.y, sc);
      } else {
        const float4 qv = qc[u];
        sc = __fmaf_rn(qv.x, __uint_as_float(k.x), sc);
        sc = __fmaf_rn(qv.y, __uint_as_float(k.y), sc);
        sc = __fmaf_rn(qv.z, __uint_as_float(k.z), sc);
        sc = __fmaf_rn(qv.w, __uint_as_float(k.w), sc);
      }
    }
    if (g + 1 < nch / GRP) {
#pragma unroll
      for (int u = 0; u < GRP; ++u) kc[u] = kn[u];
#pragma unroll
      for (int u = 0; u < GRP * QPC; ++u) qc[u] = qn[u];
    }
  }
  return sc;
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

// J consecutive values (as f32) of row r of a swizzled V tile, starting at
// value lane*J.
template <int J, typename TT>
__device__ __forceinline__ void load_v_sw(const uint8_t* vt, int r, int lane, float (&v)[J]) {
  const int byte = lane * J * (int)sizeof(TT);
  if constexpr (J * sizeof(TT) == 32) {  // f32, J = 8: two chunks
    const float4 a = *reinterpret_cast<const float4*>(vt + sw_off(r, byte));
    const float4 b = *reinterpret_cast<const float4*>(vt + sw_off(r, byte + 16));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    load_v<J, TT>(reinterpret_cast<const TT*>(vt + sw_off(r, byte)), v);
  }
}

// One output value merged over the blocks of a context in block order, the
// accessors giving block c's m, l and this lane's accumulator value (one
// head for the whole warp):
//   M = max_c m_c,  w_c = exp(m_c - M),  L = sum_c w_c l_c,
//   o = (sum_c w_c acc_c) * (1/L)        (fma chains in c order).
// Lane k holds blocks k, k+32, ...: their (m, l) and weights; the sums run
// via shuffles.  Up to 128 blocks every value is requested in one round.
template <typename FM, typename FL, typename FA>
__device__ __forceinline__ float merge_blocks(int nblk, int lane, FM mf, FL lf, FA af) {
  float L = 0.0f, o = 0.0f;
  if (nblk <= 4 * 32) {
    float mr[4], lr[4], av[32];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = 32 * q + lane;
      mr[q] = c < nblk ? mf(c) : -INFINITY;
      lr[q] = c < nblk ? lf(c) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 32; ++k) av[k] = k < nblk ? af(k) : 0.0f;
    const float M = warp_max(fmaxf(fmaxf(mr[0], mr[1]), fmaxf(mr[2], mr[3])));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c0 = 32 * q;
      if (c0 < nblk) {
        if (q > 0) {
#pragma unroll
          for (int k = 0; k < 32; ++k) av[k] = c0 + k < nblk ? af(c0 + k) : 0.0f;
        }
        const float wc = c0 + lane < nblk ? expf_det(__fsub_rn(mr[q], M)) : 0.0f;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float w = __shfl_sync(0xffffffffu, wc, k);
          const float ls = __shfl_sync(0xffffffffu, lr[q], k);
          if (c0 + k < nblk) {
            L = __fmaf_rn(w, ls, L);
            o = __fmaf_rn(w, av[k], o);
          }
        }
      }
    }
  } else {  // longer contexts: the maximum first, then 32 blocks at a time
    float M = -INFINITY;
    for (int c0 = 0; c0 < nblk; c0 += 4 * 32) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (c0 + 32 * q + lane < nblk) M = fmaxf(M, mf(c0 + 32 * q + lane));
    }
    M = warp_max(M);
    for (int c0 = 0; c0 < nblk; c0 += 32) {
      const int c = c0 + lane;
      const float mc = c < nblk ? mf(c) : -INFINITY;
      const float lc = c < nblk ? lf(c) : 0.0f;
      float av[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) av[k] = c0 + k < nblk ? af(c0 + k) : 0.0f;
      const float wc = c < nblk ? expf_det(__fsub_rn(mc, M)) : 0.0f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float w = __shfl_sync(0xffffffffu, wc, k);
        const float ls = __shfl_sync(0xffffffffu, lc, k);
        if (c0 + k < nblk) {
          L = __fmaf_rn(w, ls, L);
          o = __fmaf_rn(w, av[k], o);
        }
      }
    }
  }
  return __fmul_rn(o, L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f);
}

// merge_blocks for accessors that read this CTA's shared memory (cheap
// loads): the same operations in the same order, as short loops (the
// kernel runs once per CTA, so its code is fetched cold).
template <typename FM, typename FL, typename FA>
__device__ __forceinline__ float merge_blocks_local(int nblk, int lane, FM mf, FL lf, FA af) {
  float M = -INFINITY;
  for (int c = lane; c < nblk; c += 32) M = fmaxf(M, mf(c));
  M = warp_max(M);
  float L = 0.0f, o = 0.0f;
  for (int c0 = 0; c0 < nblk; c0 += 32) {
    const int c = c0 + lane;
    const float lc = c < nblk ? lf(c) : 0.0f;
    const float wc = c < nblk ? expf_det(__fsub_rn(mf(c), M)) : 0.0f;
    const int nc = nblk - c0 < 32 ? nblk - c0 : 32;
#pragma unroll 4
    for (int k = 0; k < nc; ++k) {
      const float w = __shfl_sync(0xffffffffu, wc, k);
      L = __fmaf_rn(w, __shfl_sync(0xffffffffu, lc, k), L);
      o = __fmaf_rn(w, af(c0 + k), o);
    }
  }
  return __fmul_rn(o, L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f);
}

// Writes merged unit u (lane = value) of the kv head whose first q head is
// hb: the f32 output and, when requested (head_dim % 32 == 0), its Q8_1
// block for the o-projection.
__device__ __forceinline__ void write_unit(float o, int u, int lane, int hb, int hd, bool ve, float* outp,
                                           uint8_t* oq8) {
  if (ve) outp[(size_t)hb * hd + u * 32 + lane] = o;
  if (oq8 && (hd % 32) == 0) {
    uint16_t dbits;
    bool zero;
    const int q = q8_1_quant_lane(o, &dbits, &zero);
    uint32_t word = ((uint32_t)(q & 0xff)) << (8 * (lane & 3));
    word |= __shfl_xor_sync(0xffffffffu, word, 1);
    word |= __shfl_xor_sync(0xffffffffu, word, 2);
    const float sum = warp_seq_sum(o);  // the sequential f16 s of the reference block
    uint32_t* ob = reinterpret_cast<uint32_t*>(oq8 + ((size_t)hb * hd / 32 + u) * 36);
    if (lane == 0) ob[0] = (uint32_t)dbits | ((uint32_t)(zero ? (uint16_t)0 : f32_to_f16_ref(sum)) << 16);
    if ((lane & 3) == 0) ob[1 + (lane >> 2)] = word;
  }
}

// Per-head RMSNorm + RoPE of a row held in registers, v[k] = row[lane + 32k]
// (head_dim = 32*J, J >= 2, so the rotation pairs k with k + J/2 in the
// same lane), with the weights and the position's (cos, sin) already
// loaded: the operations and their order are those of norm_rope_row with a
// RoPE table.
template <int J>
__device__ __forceinline__ void norm_rope_regs(float (&v)[8], const float (&wr)[8], const float (&cr)[4],
                                               const float (&sr)[4], bool has_w, int hd) {
  static_assert(J >= 2 && J <= 8 && J % 2 == 0, "head_dim 64, 128 or 256");
  if (has_w) {
    float q[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) q[k] = k < J ? __fmul_rn(v[k], v[k]) : 0.0f;
    float c = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[4]), __fadd_rn(q[2], q[6])),
                        __fadd_rn(__fadd_rn(q[1], q[5]), __fadd_rn(q[3], q[7])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c = __fadd_rn(c, __shfl_down_sync(0xffffffffu, c, o));
    c = __shfl_sync(0xffffffffu, c, 0);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(c, (float)hd), 1e-6f)));
#pragma unroll
    for (int k = 0; k < J; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], inv), wr[k]);
  }
  constexpr int H = J / 2;
#pragma unroll
  for (int k = 0; k < H; ++k) {
    const float x0 = v[k], x1 = v[k + H];
    v[k] = __fsub_rn(__fmul_rn(x0, cr[k]), __fmul_rn(x1, sr[k]));
    v[k + H] = __fadd_rn(__fmul_rn(x1, cr[k]), __fmul_rn(x0, sr[k]));
  }
}

// J = output elements per lane in the P.V phase (hd = 32*J), or J = 1 with
// hd <= 32 (masked lanes).  kCluster: the a.n_split CTAs of a kv head are
// one thread-block cluster; block partials stay in shared memory and, after
// a cluster barrier, 32-value units of the kv head's output are merged
// (unit u on CTA u mod n_split) reading the partials through distributed
// shared memory.  Every thread of every CTA reaches both cluster barriers.
template <int J, typename T, bool kCluster>
__global__ void __launch_bounds__(kAttnWarps * 32, 2)
    k_attention(const AttnArgs a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  using C = TileCfg<J, T>;
  using TT = typename C::TT;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // the swizzled tiles need 1024-byte alignment (the launch adds the slack)
  uint8_t* smem_b = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int hd = a.head_dim;
  const int hs = C::stride(hd);  // J = 1 tiles
  const int S = a.n_split;
  const int nbmax_cta = (attn_n_blocks(a.ctx) + S - 1) / S;
  const AttnLayout lay = attn_layout<J, T>(hd, a.n_head, a.n_kv, a.ctx, S, kCluster);
  float* s_q = reinterpret_cast<float*>(smem_b);  // [kGMax][hd]; the merged rows after the merge
  float* s_kpos = s_q + kGMax * hd;
  float* s_vpos = s_kpos + hd;
  float* s_sq = s_vpos + hd;  // [kAttnWarps][256]
  uint8_t* s_tiles = smem_b + attn_tiles_offset(hd);
  float* s_merge = reinterpret_cast<float*>(smem_b + attn_parts_offset<J, T>(hd, lay.ring));
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem_b + attn_bars_offset<J, T>(hd, lay.ring, lay.merge_rows));
  const size_t buf_bytes = C::buf_bytes(hd);

  const int kvh = blockIdx.x, split = blockIdx.y, z = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#if MCPO_TRACE
  unsigned long long* tr =
      a.trace ? a.trace + ((size_t)(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 8 : nullptr;
  if (threadIdx.x == 0) trace_stamp(tr, 0);
#endif
  const int hb = (kvh * a.n_head + a.n_kv - 1) / a.n_kv;
  const int he = ((kvh + 1) * a.n_head + a.n_kv - 1) / a.n_kv;
  const int G = he - hb;
  const float* qp = a.q + (size_t)z * a.qkv_bstride;
  const uint8_t* kc = static_cast<const uint8_t*>(a.k_cache) + (size_t)z * a.cache_bstride * sizeof(T);
  const uint8_t* vc = static_cast<const uint8_t*>(a.v_cache) + (size_t)z * a.cache_bstride * sizeof(T);
  float* outp = a.out + (size_t)z * a.out_bstride;
  uint8_t* oq8 = a.out_q8 ? a.out_q8 + (size_t)z * a.outq8_bstride : nullptr;
  const int pos = a.pos_ptr ? a.pos_ptr[(size_t)z * (a.pos_stride > 0 ? a.pos_stride : 1)] : a.pos_static;
  if (pos < 0 || pos >= a.ctx) {  // every CTA of the sequence (and cluster) leaves here
    if (threadIdx.x == 0 && a.err) atomicExch(a.err, 2);
    return;
  }
  // cluster: shared memory of another CTA is written only once every CTA
  // of the cluster has started (this arrival, the wait before the rounds)
  if constexpr (kCluster) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  const int n_pos = pos + 1;
  const int nblk = attn_n_blocks(n_pos);
  const int nb = split < nblk ? (nblk - 1 - split) / S + 1 : 0;  // this CTA's blocks: split + S*i, i < nb
  const int bpr = attn_bpr<J, T>(G);
  const int NT = attn_ring<J, T>(G, nbmax_cta);  // <= lay.ring (G >= g_min)
  const int kv_dim = a.n_kv * hd;
  const size_t kv_off = (size_t)kvh * hd;
  const int stride_part = attn_part_stride(hd);
  const bool fused = a.fuse_norm_rope_append != 0;
  const int pos_cta = (nblk - 1) % S;  // the CTA holding the current position's block
  const int nt = blockDim.x;

  // Before waiting for the previous kernel (programmatic dependent launch):
  // the position, the K/V rows of earlier positions for the first round's
  // blocks (the current position comes from this kernel's prologue), and
  // the norm weights and RoPE row (into registers, or into L1 for the
  // shared-memory norm).
  const int row0 = a.cache_bstride ? z * a.ctx : 0;  // this sequence's first row in the maps (0: one shared cache)
  if constexpr (C::kAsync) {
    if (threadIdx.x == 0) {
      for (int b = 0; b < NT; ++b) mbar_init(&s_bar[b], 1);
      mbar_fence_init();
      for (int i = 0; i < bpr && i < nb; ++i)
        issue_tile<TT>(s_tiles + (size_t)(i % NT) * buf_bytes, &s_bar[i % NT], &kmap, &vmap, (int)kv_off,
                       row0 + (split + S * i) * kSub, hd);
    }
    __syncthreads();
  }
  if (fused && nb > 0 && threadIdx.x < 12 && !(J >= 2 && a.rope_cos && a.rope_sin)) {
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
  // Prologue roles: warp g < G takes q row g; K/V of the current position
  // (fused: normalised/rotated here; needed by split 0, which appends it,
  // and by the CTA holding the current position's block) the next two
  // warps.  With a RoPE table and head_dim 64/128/256 the norm and rotation
  // run in registers, their weights and table row loaded before the wait.
  const bool kv_cta = fused && (split == 0 || split == pos_cta);
  const int kw = G < kAttnWarps ? G : 0, vw = G + 1 < kAttnWarps ? G + 1 : 1;
  const bool has_q = nb > 0 && warp < G;
  const bool has_kv = kv_cta && (warp == kw || warp == vw);
  const bool reg_norm = J >= 2 && fused && a.rope_cos != nullptr && a.rope_sin != nullptr;
  float wq[8], wk[8], cr[4], sr[4];
  if (reg_norm) {
    const int half = hd / 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = lane + 32 * k;
      wq[k] = has_q && a.q_norm && d < hd ? load_weight(a.q_norm, a.q_norm_dtype, d) : 0.0f;
      wk[k] = has_kv && warp == kw && a.k_norm && d < hd ? load_weight(a.k_norm, a.k_norm_dtype, d) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = lane + 32 * k;
      const bool need = (has_q || (has_kv && warp == kw)) && d < half;
      cr[k] = need ? a.rope_cos[(size_t)pos * half + d] : 0.0f;
      sr[k] = need ? a.rope_sin[(size_t)pos * half + d] : 0.0f;
    }
  }
  pdl_wait();
  pdl_launch_dependents();
#if MCPO_TRACE
  if (threadIdx.x == 0) trace_stamp(tr, 1);
#endif

  // every global load first, then the norms, then the stores
  float qv[8], kvr[8];
  if (has_q) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = lane + 32 * k;
      qv[k] = d < hd ? qp[(size_t)(hb + warp) * hd + d] : 0.0f;
    }
  }
  if (has_kv) {
    const float* src = (warp == kw ? a.k : a.v) + (size_t)z * a.qkv_bstride + kv_off;
#pragma unroll
    for (int k = 0; k < 8; ++k) kvr[k] = lane + 32 * k < hd ? src[lane + 32 * k] : 0.0f;
  }
  if constexpr (J >= 2) {
    if (reg_norm) {
      if (has_q) norm_rope_regs<J>(qv, wq, cr, sr, a.q_norm != nullptr, hd);
      if (has_kv && warp == kw) norm_rope_regs<J>(kvr, wk, cr, sr, a.k_norm != nullptr, hd);
    }
  }
  if (has_q) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (lane + 32 * k < hd) s_q[warp * hd + lane + 32 * k] = qv[k];
  }
  if (has_kv) {
    float* dst = warp == kw ? s_kpos : s_vpos;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (lane + 32 * k < hd) dst[lane + 32 * k] = kvr[k];
  }
  __syncwarp();
  if (fused && !reg_norm && has_q)
    norm_rope_row(s_q + warp * hd, s_sq + warp * 256, hd, a.q_norm, a.q_norm_dtype, true, a.rope_cos, a.rope_sin,
                  a.rope_base, a.rope_scale, pos, lane);
  if (!reg_norm && has_kv && warp == kw)
    norm_rope_row(s_kpos, s_sq + warp * 256, hd, a.k_norm, a.k_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base,
                  a.rope_scale, pos, lane);
  __syncthreads();
  if (fused && split == 0) {
    void* kwp = const_cast<uint8_t*>(kc);
    void* vwp = const_cast<uint8_t*>(vc);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      kv_store<T>(kwp, (size_t)pos * kv_dim + kv_off + d, s_kpos[d]);
      kv_store<T>(vwp, (size_t)pos * kv_dim + kv_off + d, s_vpos[d]);
    }
  }

  if constexpr (kCluster) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
#if MCPO_TRACE
  if (threadIdx.x == 0) trace_stamp(tr, 2);
#endif

  // Rounds of bpr blocks; warp w takes (head w % G, block r*bpr + w / G).
  const int nblk_max = attn_n_blocks(a.ctx);
  const bool act = lane * J < hd;
  for (int r = 0; r * bpr < nb; ++r) {
    if constexpr (C::kAsync) {
      // next round's tiles into the buffers the round before finished with
      // (their generic reads and writes ordered before the copies)
      if (threadIdx.x == 0) {
        fence_proxy_async();
        for (int j = 0; j < bpr; ++j) {
          const int i = (r + 1) * bpr + j;
          if (i < nb)
            issue_tile<TT>(s_tiles + (size_t)(i % NT) * buf_bytes, &s_bar[i % NT], &kmap, &vmap, (int)kv_off,
                           row0 + (split + S * i) * kSub, hd);
        }
      }
      for (int j = 0; j < bpr; ++j) {
        const int i = r * bpr + j;
        if (i >= nb) break;
        mbar_wait(&s_bar[i % NT], (uint32_t)(i / NT) & 1u, a.err);
      }
      for (int j = 0; j < bpr; ++j) {
        const int i = r * bpr + j;
        if (i >= nb) break;
        uint8_t* buf = s_tiles + (size_t)(i % NT) * buf_bytes;
        put_pos_row<TT>(buf, s_kpos, s_vpos, (split + S * i) * kSub, pos, fused, hd);
        zero_rows<TT>(buf, (split + S * i) * kSub, n_pos, hd);
      }
#if MCPO_TRACE
      if (r == 0 && threadIdx.x == 0) trace_stamp(tr, 6);  // the first round's tiles have landed
#endif
    } else {
      for (int j = 0; j < bpr; ++j) {
        const int i = r * bpr + j;
        if (i >= nb) break;
        float* kt = reinterpret_cast<float*>(s_tiles + (size_t)(i % NT) * buf_bytes);
        stage_kv_tile<T>(kc, vc, s_kpos, s_vpos, kt, kt + (size_t)kSub * hs, (split + S * i) * kSub, n_pos, pos, fused,
                         kv_dim, kv_off, hd, hs, threadIdx.x, nt);
      }
    }
    __syncthreads();
    const int g = warp % G, j = warp / G, i = r * bpr + j;
    if (j < bpr && i < nb) {
      const int c = split + S * i;
      const uint8_t* tile = s_tiles + (size_t)(i % NT) * buf_bytes;
      const bool valid = c * kSub + lane < n_pos;
      float sc;
      if constexpr (C::kAsync)
        sc = score_row_sw<TT, 32 * J>(s_q + g * hd, tile, lane);  // head_dim = 32 * J
      else
        sc = score_row<TT>(s_q + g * hd, reinterpret_cast<const TT*>(tile) + (size_t)lane * hs, hd, hs);
      sc = valid ? __fmul_rn(sc, a.scale) : -INFINITY;
      const float m = warp_max(sc);
      const float p = valid ? expf_det(__fsub_rn(sc, m)) : 0.0f;
      const float l = __shfl_sync(0xffffffffu, warp_sum(p), 0);
      float acc[J];
#pragma unroll
      for (int jj = 0; jj < J; ++jj) acc[jj] = 0.0f;
      if constexpr (C::kAsync) {
        // P.V: the probabilities through this warp's shared scratch (free
        // after the prologue) as broadcasts, V rows in groups whose loads
        // are all issued before their fma chains
        float* pw = s_sq + warp * 256;
        pw[lane] = p;
        __syncwarp();
        const uint8_t* vt = tile + (size_t)kSub * 32 * J * sizeof(TT);
        constexpr int PG = J * sizeof(TT) > 16 ? 4 : 8;  // positions per group
#pragma unroll
        for (int t0 = 0; t0 < kSub; t0 += PG) {
          float pt[PG], vv[PG][J];
#pragma unroll
          for (int u = 0; u < PG; ++u) pt[u] = pw[t0 + u];
#pragma unroll
          for (int u = 0; u < PG; ++u) load_v_sw<J, TT>(vt, t0 + u, lane, vv[u]);
#pragma unroll
          for (int u = 0; u < PG; ++u)
#pragma unroll
            for (int jj = 0; jj < J; ++jj) acc[jj] = __fmaf_rn(pt[u], vv[u][jj], acc[jj]);
        }
        __syncwarp();
      } else {
#pragma unroll 8
        for (int tt = 0; tt < kSub; ++tt) {
          const float pt = __shfl_sync(0xffffffffu, p, tt);
          if (act) {
            float vv[J];
            load_v<J, TT>(reinterpret_cast<const TT*>(tile) + (size_t)(kSub + tt) * hs + lane * J, vv);
#pragma unroll
            for (int jj = 0; jj < J; ++jj) acc[jj] = __fmaf_rn(pt, vv[jj], acc[jj]);
          }
        }
      }
      if constexpr (kCluster) {
        // into the merge row of block c at the CTA merging each unit: this
        // lane's J values lie in unit g * hd/32 + lane*J/32; lane k < hd/32
        // sends (m, l) for unit g * hd/32 + k
        static_assert(!kCluster || J >= 2, "the cluster merge serves head_dim 64/128/256");
        const int upw = hd / 32;
        const int U = g * upw + (lane * J) / 32;
        const uint32_t ra = dsmem_addr(s_merge + ((size_t)(U / S) * nblk_max + c) * kMergeRow + (lane * J) % 32, U % S);
        if constexpr (J == 2) {
          dsmem_st2(ra, acc[0], acc[1]);
        } else {
#pragma unroll
          for (int jj = 0; jj < J; jj += 4) dsmem_st4(ra + 4 * jj, acc[jj], acc[jj + 1], acc[jj + 2], acc[jj + 3]);
        }
        if (lane < upw) {
          const int U2 = g * upw + lane;
          dsmem_st2(dsmem_addr(s_merge + ((size_t)(U2 / S) * nblk_max + c) * kMergeRow + 32, U2 % S), m, l);
        }
      } else {
        float* dst = a.partial + (((size_t)z * a.n_head + hb + g) * nblk_max + c) * stride_part;
        if (act)
#pragma unroll
          for (int jj = 0; jj < J; ++jj) dst[4 + lane * J + jj] = acc[jj];
        if (lane == 0) {
          dst[0] = m;
          dst[1] = l;
        }
      }
    }
    __syncthreads();
  }

  // ---- merge over blocks in block order.  Unit u = 32 consecutive output
  // values of this kv head's G heads, lane = value.
  const int n_units = (G * hd + 31) / 32;
#if MCPO_TRACE
  if (threadIdx.x == 0) trace_stamp(tr, 4);
#endif
  if constexpr (kCluster) {
    cluster_sync_all();  // every merge row of this CTA's units has arrived
#if MCPO_TRACE
    if (threadIdx.x == 0) trace_stamp(tr, 5);
#endif
    for (int slot = warp; split + slot * S < n_units; slot += kAttnWarps) {
      const int u = split + slot * S;
      const float* rows = s_merge + (size_t)slot * nblk_max * kMergeRow;
      const float o = merge_blocks_local(
          nblk, lane, [&](int c) { return rows[(size_t)c * kMergeRow + 32]; },
          [&](int c) { return rows[(size_t)c * kMergeRow + 33]; },
          [&](int c) { return rows[(size_t)c * kMergeRow + lane]; });
      write_unit(o, u, lane, hb, hd, true, outp, oq8);
    }
#if MCPO_TRACE
    if (tr) {
      __syncthreads();
      if (threadIdx.x == 0) trace_stamp(tr, 3);
    }
#endif
  } else {
    __shared__ unsigned ticket_s;
    unsigned* counter = a.counters + (size_t)z * a.n_kv + kvh;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned t;
      asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(counter) : "memory");
      ticket_s = t;
    }
    __syncthreads();
#if MCPO_TRACE
    if (threadIdx.x == 0) trace_stamp(tr, 3);
#endif
    if (ticket_s != (unsigned)(S - 1)) return;
    if (threadIdx.x == 0) atomicExch(counter, 0u);
    const float* part = a.partial + ((size_t)z * a.n_head + hb) * nblk_max * stride_part;
    for (int u = warp; u < n_units; u += kAttnWarps) {
      const int e = u * 32 + lane;
      const bool ve = e < G * hd;
      const int g = ve ? e / hd : 0, d = ve ? e - g * hd : 0;
      const float* hp = part + (size_t)g * nblk_max * stride_part;
      float o;
      if ((hd & 31) == 0) {  // one head per unit
        o = merge_blocks(
            nblk, lane, [&](int c) { return __ldcg(hp + (size_t)c * stride_part); },
            [&](int c) { return __ldcg(hp + (size_t)c * stride_part + 1); },
            [&](int c) { return __ldcg(hp + (size_t)c * stride_part + 4 + d); });
      } else {  // small heads: a unit spans several heads, each lane its own
        float M = -INFINITY, L = 0.0f, acc = 0.0f;
        for (int c = 0; c < nblk; ++c) M = fmaxf(M, __ldcg(hp + (size_t)c * stride_part));
        for (int c = 0; c < nblk; ++c) {
          const float w = expf_det(__fsub_rn(__ldcg(hp + (size_t)c * stride_part), M));
          L = __fmaf_rn(w, __ldcg(hp + (size_t)c * stride_part + 1), L);
          acc = __fmaf_rn(w, __ldcg(hp + (size_t)c * stride_part + 4 + d), acc);
        }
        o = __fmul_rn(acc, L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f);
      }
      write_unit(o, u, lane, hb, hd, ve, outp, oq8);
    }
  }
}

// ---------------------------------------------------------------------
// Prompt attention (launch_prompt_attention): grid (n_kv, ceil(T / 8)), 8
// warps; warp w serves token 8*blockIdx.y + w and the kv head's G q heads.
// K/V blocks of 32 positions are staged as f32 rows (stride head_dim + 4
// floats: lanes reading different rows hit different banks) in two
// buffers; the next block's rows are loaded into registers while the
// current one is used.  Per (token, head, block) the decode's arithmetic:
// s = scale * (q . k) as one fma chain in d order, -inf past the token's
// position, m = max, p = exp(s - m), l = butterfly sum, acc_d = sum p_t v_td
// in t order, written as the block's partial; then the blocks merge in
// block order (merge_blocks).
constexpr int kPaTokens = 8;
constexpr int kPaHeads = 4;  // q heads scored together by a warp (they share the K loads)

template <int J>
__host__ __device__ inline int pa_row_stride() {
  return 32 * J + 4;
}

template <int J, typename T>
__host__ __device__ inline size_t pa_smem_bytes(int G) {
  return ((size_t)kPaTokens * G * 32 * J + (size_t)2 * 2 * 32 * pa_row_stride<J>()) * 4;
}

// Loads (vals) or stores (st) this thread's share of one K/V block: rows
// c*32 .. +31 of the kv head, 4 values per chunk; rows at or past `rows`
// are zeros.
template <int J, typename T>
struct PaStage {
  static constexpr int kChunks = 2 * 32 * 32 * J / 4;  // K and V, 4 values each
  static constexpr int kPer = kChunks / (8 * 32);        // per thread (256 threads)
  float4 v[kPer];
  __device__ __forceinline__ void load(const T* kc, const T* vc, int kv_dim, int kv_off, int c, int rows) {
    const int hd = 32 * J;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int ch = threadIdx.x + i * 256;
      const int half = ch / (kChunks / 2), rem = ch % (kChunks / 2);
      const int r = rem / (hd / 4), q4 = rem % (hd / 4);
      const int row = c * 32 + r;
      float4 f = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (row < rows) {
        const T* src = (half ? vc : kc) + (size_t)row * kv_dim + kv_off + q4 * 4;
        if constexpr (sizeof(T) == 2) {
          const uint2 u = *reinterpret_cast<const uint2*>(src);
          const float2 a = h2f2(u.x), b = h2f2(u.y);
          f = make_float4(a.x, a.y, b.x, b.y);
        } else {
          f = *reinterpret_cast<const float4*>(src);
        }
      }
      v[i] = f;
    }
  }
  __device__ __forceinline__ void store(float* buf) const {
    const int hd = 32 * J, rs = pa_row_stride<J>();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int ch = threadIdx.x + i * 256;
      const int half = ch / (kChunks / 2), rem = ch % (kChunks / 2);
      const int r = rem / (hd / 4), q4 = rem % (hd / 4);
      *reinterpret_cast<float4*>(buf + (size_t)half * 32 * rs + (size_t)r * rs + q4 * 4) = v[i];
    }
  }
};

template <int J, typename T>
__global__ void __launch_bounds__(256, 2) k_prompt_attention(const PromptAttnArgs a) {
  extern __shared__ __align__(16) float pa_smem[];
  const int hd = 32 * J, rs = pa_row_stride<J>();
  const int kvh = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hb = (kvh * a.n_head + a.n_kv - 1) / a.n_kv;
  const int he = ((kvh + 1) * a.n_head + a.n_kv - 1) / a.n_kv;
  const int G = he - hb;
  float* sq = pa_smem;                             // [kPaTokens][G][hd]
  float* tiles = pa_smem + (size_t)kPaTokens * G * hd;  // [2 buffers][K, V][32][rs]
  const int t = blockIdx.y * kPaTokens + warp;
  const bool tok = t < a.T;
  const int kv_dim = a.n_kv * hd, kv_off = kvh * hd;
  const int nblk_max = attn_n_blocks(a.ctx), stride_part = attn_part_stride(hd);
  const T* kc = static_cast<const T*>(a.k_cache);
  const T* vc = static_cast<const T*>(a.v_cache);
  pdl_wait();
  // positions: this warp's token and the CTA's last one
  __shared__ int maxpos_s;
  if (threadIdx.x == 0) {
    int mx = -1;
    for (int w = 0; w < kPaTokens; ++w) {
      const int tt = blockIdx.y * kPaTokens + w;
      if (tt < a.T) mx = max(mx, min(a.pos[tt], a.ctx - 1));
    }
    maxpos_s = mx;
  }
  for (int i = threadIdx.x; i < kPaTokens * G * hd; i += 256) {
    const int w = i / (G * hd), rem = i % (G * hd);
    const int tt = blockIdx.y * kPaTokens + w;
    sq[i] = tt < a.T ? a.q[(size_t)tt * a.q_stride + (size_t)hb * hd + rem] : 0.0f;
  }
  __syncthreads();
  const int rows = maxpos_s + 1;
  const int nb_cta = attn_n_blocks(rows);
  const int pos = tok ? min(a.pos[t], a.ctx - 1) : -1;
  const int n_pos = pos + 1, nb = tok ? attn_n_blocks(n_pos) : 0;

  PaStage<J, T> stage;
  if (nb_cta > 0) {
    stage.load(kc, vc, kv_dim, kv_off, 0, rows);
    stage.store(tiles);
  }
  __syncthreads();
  for (int c = 0; c < nb_cta; ++c) {
    const float* kt = tiles + (size_t)(c & 1) * 2 * 32 * rs;
    const float* vt = kt + (size_t)32 * rs;
    if (c + 1 < nb_cta) stage.load(kc, vc, kv_dim, kv_off, c + 1, rows);
    if (c < nb) {
      const bool valid = c * 32 + lane < n_pos;
      for (int g0 = 0; g0 < G; g0 += kPaHeads) {
        float sc[kPaHeads];
#pragma unroll
        for (int g = 0; g < kPaHeads; ++g) sc[g] = 0.0f;
        const float* krow = kt + (size_t)lane * rs;
#pragma unroll 8
        for (int d4 = 0; d4 < hd / 4; ++d4) {
          const float4 k = *reinterpret_cast<const float4*>(krow + d4 * 4);
#pragma unroll
          for (int g = 0; g < kPaHeads; ++g) {
            if (g0 + g < G) {
              const float4 q = *reinterpret_cast<const float4*>(sq + ((size_t)warp * G + g0 + g) * hd + d4 * 4);
              sc[g] = __fmaf_rn(q.x, k.x, sc[g]);
              sc[g] = __fmaf_rn(q.y, k.y, sc[g]);
              sc[g] = __fmaf_rn(q.z, k.z, sc[g]);
              sc[g] = __fmaf_rn(q.w, k.w, sc[g]);
            }
          }
        }
        float p[kPaHeads], acc[kPaHeads][J];
#pragma unroll
        for (int g = 0; g < kPaHeads; ++g) {
          const float s = valid ? __fmul_rn(sc[g], a.scale) : -INFINITY;
          const float m = warp_max(s);
          p[g] = valid ? expf_det(__fsub_rn(s, m)) : 0.0f;
          const float l = __shfl_sync(0xffffffffu, warp_sum(p[g]), 0);
          if (g0 + g < G && lane == 0) {
            float* dst = a.partial + (((size_t)t * a.n_head + hb + g0 + g) * nblk_max + c) * stride_part;
            dst[0] = m;
            dst[1] = l;
          }
#pragma unroll
          for (int jj = 0; jj < J; ++jj) acc[g][jj] = 0.0f;
        }
#pragma unroll 4
        for (int i = 0; i < 32; ++i) {
          float v[J];
          load_v<J, float>(vt + (size_t)i * rs + lane * J, v);
#pragma unroll
          for (int g = 0; g < kPaHeads; ++g) {
            const float pt = __shfl_sync(0xffffffffu, p[g], i);
#pragma unroll
            for (int jj = 0; jj < J; ++jj) acc[g][jj] = __fmaf_rn(pt, v[jj], acc[g][jj]);
          }
        }
#pragma unroll
        for (int g = 0; g < kPaHeads; ++g) {
          if (g0 + g < G) {
            float* dst = a.partial + (((size_t)t * a.n_head + hb + g0 + g) * nblk_max + c) * stride_part + 4 + lane * J;
#pragma unroll
            for (int jj = 0; jj < J; ++jj) dst[jj] = acc[g][jj];
          }
        }
      }
    }
    __syncthreads();  // every warp is done with the buffer the next store overwrites
    if (c + 1 < nb_cta) stage.store(tiles + (size_t)((c + 1) & 1) * 2 * 32 * rs);
    __syncthreads();
  }
  // merge each (token, head) over its blocks in block order
  if (tok) {
    for (int g = 0; g < G; ++g) {
      const float* hp = a.partial + ((size_t)t * a.n_head + hb + g) * nblk_max * stride_part;
      for (int u = 0; u < J; ++u) {
        const int d = u * 32 + lane;
        const float o = merge_blocks(
            nb, lane, [&](int c) { return __ldcg(hp + (size_t)c * stride_part); },
            [&](int c) { return __ldcg(hp + (size_t)c * stride_part + 1); },
            [&](int c) { return __ldcg(hp + (size_t)c * stride_part + 4 + d); });
        a.out[(size_t)t * a.out_stride + (size_t)(hb + g) * hd + d] = o;
      }
    }
  }
  pdl_launch_dependents();
}


// Cluster launch: grid (n_kv, n_split, batch) in clusters of (1, n_split, 1),
// with programmatic dependent launch when pdl is set.
template <typename Kern>
cudaError_t launch_cluster(Kern kernel, dim3 grid, int cluster_y, size_t smem, cudaStream_t st, bool pdl,
                           const AttnArgs& a, const CUtensorMap& km, const CUtensorMap& vm) {
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
  return cudaLaunchKernelEx(&cfg, kernel, a, km, vm);
}

// cuTensorMapEncodeTiled, from the driver (resolved once at set-up).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

// The K or V cache of one layer as a 2-D tensor [rows][kv_dim] in its own
// type (rows = sequences x context), read in boxes of 32 rows x 128 bytes
// with the 128-byte swizzle; rows past the end read as zero.
bool encode_kv_map(CUtensorMap* m, const void* base, bool f16, int kv_dim, unsigned long long rows) {
  const int esz = f16 ? 2 : 4;
  if (!g_encode || !base || (reinterpret_cast<uintptr_t>(base) & 15) || ((size_t)kv_dim * esz) % 16) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kv_dim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kv_dim * esz};
  const cuuint32_t box[2] = {(cuuint32_t)(128 / esz), (cuuint32_t)kSub};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Whether clusters of n CTAs of a kernel can be resident, queried once at
// set-up per device (with the largest cluster-path shared memory); the
// cluster merge is launched only where they can (otherwise the
// global-memory merge, with the same bits, is used).
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
// dynamic shared memory the cluster kernels are set up for (the sm_100
// opt-in maximum per CTA, 232448 bytes, less a margin for static data)
constexpr int kDynSmemMax = 232448 - 256;

template <int J, typename T>
cudaError_t init_jt(int dev) {
  const size_t mx = attn_smem_bytes_t<J, T>(32 * J, TileCfg<J, T>::kRing, 0);  // a full ring
  cudaError_t e = cudaFuncSetAttribute(k_attention<J, T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mx);
  if (e != cudaSuccess) return e;
  if constexpr (J >= 2) {
    e = cudaFuncSetAttribute(k_prompt_attention<J, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmemMax);
    if (e != cudaSuccess) return e;
    // two CTAs per SM (the staging and the per-token work are latency-bound)
    e = cudaFuncSetAttribute(k_prompt_attention<J, T>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_attention<J, T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmemMax);
    if (e != cudaSuccess) return e;
    const bool nonportable =
        cudaFuncSetAttribute(k_attention<J, T, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
        cudaSuccess;
    if (!nonportable) (void)cudaGetLastError();
    // queried at the largest shared memory (one CTA per SM): a cluster that
    // is resident then is resident with any smaller carve-up
    for (int n = 1; n <= kAttnMaxCluster; ++n)
      g_cluster_ok[dev][sizeof(T) == 2][j_index(J)][n] =
          (n <= 8 || nonportable) && query_cluster(k_attention<J, T, true>, kDynSmemMax, n);
  }
  return cudaSuccess;
}

template <int J>
cudaError_t launch_j(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int hd = a.head_dim;
  const dim3 grid(a.n_kv, a.n_split, a.batch > 0 ? a.batch : 1);
  const bool f16 = a.kv_f16 != 0;
  CUtensorMap km, vm;
  memset(&km, 0, sizeof(km));
  memset(&vm, 0, sizeof(vm));
  if constexpr (J >= 2) {
    // the sequences' caches must be consecutive [batch][ctx][kv_dim] blocks,
    // or one cache they all read (cache_bstride 0: the tokens of one prompt)
    const int B = a.batch > 1 && a.cache_bstride ? a.batch : 1;
    const int kv_dim = a.n_kv * hd;
    if (B > 1 && a.cache_bstride != (size_t)a.ctx * kv_dim) return cudaErrorInvalidValue;
    const unsigned long long rows = (unsigned long long)B * a.ctx;
    if (rows > 0x7fffffffull || !encode_kv_map(&km, a.k_cache, f16, kv_dim, rows) ||
        !encode_kv_map(&vm, a.v_cache, f16, kv_dim, rows))
      return cudaErrorInvalidValue;
  }
  auto bytes = [&](auto t, bool cl) {
    using TE = decltype(t);
    const AttnLayout l = attn_layout<J, TE>(hd, a.n_head, a.n_kv, a.ctx, a.n_split, cl);
    return attn_smem_bytes_t<J, TE>(hd, l.ring, l.merge_rows);
  };
  if constexpr (J >= 2) {
    const int nb_cta = (attn_n_blocks(a.ctx) + a.n_split - 1) / a.n_split;
    const int dev = a.cluster ? current_device() : -1;
    if (dev >= 0 && nb_cta <= kAttnMaxBlocksCta && g_cluster_ok[dev][f16][j_index(J)][a.n_split]) {
      const size_t b = f16 ? bytes(__half(), true) : bytes(0.0f, true);
      if (b <= (size_t)kDynSmemMax) {
        if (f16) return launch_cluster(k_attention<J, __half, true>, grid, a.n_split, b, st, pdl, a, km, vm);
        return launch_cluster(k_attention<J, float, true>, grid, a.n_split, b, st, pdl, a, km, vm);
      }
    }
  }
  if (!a.partial || !a.counters) return cudaErrorInvalidValue;
  if (f16)
    return launch_k(k_attention<J, __half, false>, grid, dim3(kAttnWarps * 32), bytes(__half(), false), st, pdl, a, km,
                    vm);
  return launch_k(k_attention<J, float, false>, grid, dim3(kAttnWarps * 32), bytes(0.0f, false), st, pdl, a, km, vm);
}

template <int J>
cudaError_t init_j(int dev) {
  cudaError_t e = init_jt<J, float>(dev);
  if (e == cudaSuccess) e = init_jt<J, __half>(dev);
  return e;
}

}  // namespace

size_t attn_partial_floats(int n_head, int n_blocks, int head_dim) {
  return (size_t)n_head * n_blocks * attn_part_stride(head_dim);
}

namespace {

template <int J, typename T>
cudaError_t launch_prompt_attention_jt(const PromptAttnArgs& a, int G, cudaStream_t st) {
  const size_t smem = pa_smem_bytes<J, T>(G);
  if (smem > (size_t)kDynSmemMax) return cudaErrorInvalidValue;
  return launch_k(k_prompt_attention<J, T>, dim3(a.n_kv, (a.T + kPaTokens - 1) / kPaTokens), dim3(256), smem, st, true,
                  a);
}

}  // namespace

cudaError_t launch_prompt_attention(const PromptAttnArgs& a, cudaStream_t st) {
  if (!a.q || !a.k_cache || !a.v_cache || !a.pos || !a.partial || !a.out || a.T < 1 || a.n_kv < 1 ||
      a.n_head < a.n_kv || a.n_head % a.n_kv || a.n_head / a.n_kv > kGMax || a.ctx < 1 ||
      (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256))
    return cudaErrorInvalidValue;
  const int G = a.n_head / a.n_kv;
  const bool f16 = a.kv_f16 != 0;
  switch (a.head_dim) {
    case 64: return f16 ? launch_prompt_attention_jt<2, __half>(a, G, st) : launch_prompt_attention_jt<2, float>(a, G, st);
    case 128: return f16 ? launch_prompt_attention_jt<4, __half>(a, G, st) : launch_prompt_attention_jt<4, float>(a, G, st);
    default: return f16 ? launch_prompt_attention_jt<8, __half>(a, G, st) : launch_prompt_attention_jt<8, float>(a, G, st);
  }
}

cudaError_t attention_init() {
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return cudaErrorNotSupported;
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  cudaError_t e = init_j<1>(dev);
  if (e == cudaSuccess) e = init_j<2>(dev);
  if (e == cudaSuccess) e = init_j<4>(dev);
  if (e == cudaSuccess) e = init_j<8>(dev);
  return e;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.n_split > kMaxSplit || a.n_split < 1) return cudaErrorInvalidValue;
  if (a.cluster && a.n_split > kAttnMaxCluster) return cudaErrorInvalidValue;
  if (a.n_kv < 1 || a.n_head < a.n_kv || a.n_head > kGMax * a.n_kv || a.ctx < 1 || attn_n_blocks(a.ctx) > kMaxBlocks) return cudaErrorInvalidValue;
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
