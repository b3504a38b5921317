// attn_dev.cuh -- KV-cache access shared by the decode attention kernels.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace mcpo {

constexpr int kSub = 32;  // positions per attention sub-chunk (one per lane)

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

// A value of the current position as the cache holds it (f16: rounded to
// nearest even), so the current position is attended exactly as stored.
template <typename T>
__device__ __forceinline__ float kv_round(float v) {
  if constexpr (sizeof(T) == 2)
    return __half2float(__float2half_rn(v));
  else
    return v;
}

// K/V rows are read once per step: streaming (evict-first) loads.
template <typename T>
__device__ __forceinline__ float4 kv_load4(const void* p, size_t i) {
  if constexpr (sizeof(T) == 2) {
    const uint2 u = __ldcs(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p) + i));
    const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
  } else {
    return __ldcs(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
  }
}

// K/V rows c0 .. c0+31 (zero past t1) into kt/vt, 4 consecutive values of a
// row per item (hd % 4 == 0, rows 16-byte aligned), kBatch items per thread
// per round with every load issued before the stores.
template <typename T, int kBatch = 8>
__device__ __forceinline__ void stage_kv_tile(const void* k_cache, const void* v_cache, const float* kpos,
                                              const float* vpos, float* kt, float* vt, int c0, int t1, int pos,
                                              bool fused, int kv_dim, size_t kv_off, int hd, int hs, int tid, int nt) {
  if (hd & 3) {  // small odd head sizes: one value per item
    for (int e0 = tid; e0 < kSub * hd; e0 += nt * kBatch) {
      float kr[kBatch], vr[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int e = e0 + u * nt;
        kr[u] = vr[u] = 0.0f;
        if (e < kSub * hd) {
          const int r = e / hd, d = e - r * hd, t = c0 + r;
          if (t < t1) {
            if (fused && t == pos) {
              kr[u] = kv_round<T>(kpos[d]);
              vr[u] = kv_round<T>(vpos[d]);
            } else {
              const size_t i = (size_t)t * kv_dim + kv_off + d;
              kr[u] = kv_load<T>(k_cache, i);
              vr[u] = kv_load<T>(v_cache, i);
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int e = e0 + u * nt;
        if (e < kSub * hd) {
          const int r = e / hd, d = e - r * hd;
          kt[r * hs + d] = kr[u];
          vt[r * hs + d] = vr[u];
        }
      }
    }
    return;
  }
  const int n4 = kSub * hd / 4;
  for (int e0 = tid; e0 < n4; e0 += nt * kBatch) {
    float4 kr[kBatch], vr[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int e = e0 + u * nt;
      kr[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      vr[u] = kr[u];
      if (e < n4) {
        const int r = (e * 4) / hd, d = e * 4 - r * hd, t = c0 + r;
        if (t < t1) {
          if (fused && t == pos) {
            kr[u] = make_float4(kv_round<T>(kpos[d]), kv_round<T>(kpos[d + 1]), kv_round<T>(kpos[d + 2]),
                                kv_round<T>(kpos[d + 3]));
            vr[u] = make_float4(kv_round<T>(vpos[d]), kv_round<T>(vpos[d + 1]), kv_round<T>(vpos[d + 2]),
                                kv_round<T>(vpos[d + 3]));
          } else {
            const size_t i = (size_t)t * kv_dim + kv_off + d;
            kr[u] = kv_load4<T>(k_cache, i);
            vr[u] = kv_load4<T>(v_cache, i);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int e = e0 + u * nt;
      if (e < n4) {
        const int r = (e * 4) / hd, d = e * 4 - r * hd;
        float* kd = kt + r * hs + d;
        float* vd = vt + r * hs + d;
        kd[0] = kr[u].x; kd[1] = kr[u].y; kd[2] = kr[u].z; kd[3] = kr[u].w;
        vd[0] = vr[u].x; vd[1] = vr[u].y; vd[2] = vr[u].z; vd[3] = vr[u].w;
      }
    }
  }
}

}  // namespace mcpo
