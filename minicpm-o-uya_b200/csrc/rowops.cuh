// rowops.cuh -- per-head row operations shared by the attention kernel and
// the standalone slot kernels: QK-RMSNorm and NeoX RoPE on one row held in
// shared memory, computed by one warp with only round-to-nearest IEEE
// operations (no FMA contraction), so the result is bit-identical to the
// CPU restatement of the reference.
#pragma once

#include "common.cuh"

namespace mcpo {

// Warp-level per-head RMSNorm + RoPE of row[0..hd) in shared memory.
// Sum of squares in the order of a 256-thread halving tree (virtual thread
// t holds row[t]^2, zero beyond hd).
__device__ inline void norm_rope_row(float* row, float* sq, int hd, const void* w, int w_dtype, bool rope,
                                     const float* cos_t, const float* sin_t, float base, float fscale, int pos,
                                     int lane) {
  // every global load (weights, rope table) is issued up front: hd <= 256
  // gives at most 8 weights and 4 (cos, sin) pairs per lane
  const int half = hd / 2;
  float wr[8], cr[4], sr[4];
  if (w) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = lane + 32 * k;
      wr[k] = d < hd ? load_weight(w, w_dtype, d) : 0.0f;
    }
  }
  if (rope && cos_t) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = lane + 32 * k;
      cr[k] = d < half ? cos_t[(size_t)pos * half + d] : 0.0f;
      sr[k] = d < half ? sin_t[(size_t)pos * half + d] : 0.0f;
    }
  }
  if (w) {
    for (int t = lane; t < 256; t += 32) sq[t] = t < hd ? __fmul_rn(row[t], row[t]) : 0.0f;
    __syncwarp();
    float c = __fadd_rn(__fadd_rn(__fadd_rn(sq[lane], sq[lane + 128]), __fadd_rn(sq[lane + 64], sq[lane + 192])),
                        __fadd_rn(__fadd_rn(sq[lane + 32], sq[lane + 160]), __fadd_rn(sq[lane + 96], sq[lane + 224])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c = __fadd_rn(c, __shfl_down_sync(0xffffffffu, c, o));
    c = __shfl_sync(0xffffffffu, c, 0);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(c, (float)hd), 1e-6f)));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = lane + 32 * k;
      if (d < hd) row[d] = __fmul_rn(__fmul_rn(row[d], inv), wr[k]);
    }
    __syncwarp();
  }
  if (!rope) return;
  float r0[4], r1[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    if (d < half) {
      float c, s;
      if (cos_t) {
        c = cr[k];
        s = sr[k];
      } else {
        // qwen3.uya:1620-1623 without a table
        const float theta = __fdiv_rn(__fmul_rn((float)pos, fscale), powf(base, __fdiv_rn((float)(2 * d), (float)hd)));
        c = cosf(theta);
        s = sinf(theta);
      }
      const float x0 = row[d], x1 = row[d + half];
      r0[k] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      r1[k] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    }
  }
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    if (d < half) {
      row[d] = r0[k];
      row[d + half] = r1[k];
    }
  }
  __syncwarp();
}

}  // namespace mcpo
