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
  if (w) {
    for (int t = lane; t < 256; t += 32) sq[t] = t < hd ? __fmul_rn(row[t], row[t]) : 0.0f;
    __syncwarp();
    float c = __fadd_rn(__fadd_rn(__fadd_rn(sq[lane], sq[lane + 128]), __fadd_rn(sq[lane + 64], sq[lane + 192])),
                        __fadd_rn(__fadd_rn(sq[lane + 32], sq[lane + 160]), __fadd_rn(sq[lane + 96], sq[lane + 224])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c = __fadd_rn(c, __shfl_down_sync(0xffffffffu, c, o));
    c = __shfl_sync(0xffffffffu, c, 0);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(c, (float)hd), 1e-6f)));
    for (int d = lane; d < hd; d += 32) row[d] = __fmul_rn(__fmul_rn(row[d], inv), load_weight(w, w_dtype, d));
    __syncwarp();
  }
  if (!rope) return;
  const int half = hd / 2;
  float r0[4], r1[4];
  int cnt = 0;
  for (int d = lane; d < half && cnt < 4; d += 32, ++cnt) {
    float c, s;
    if (cos_t) {
      c = cos_t[(size_t)pos * half + d];
      s = sin_t[(size_t)pos * half + d];
    } else {
      // qwen3.uya:1620-1623 without a table
      const float theta = __fdiv_rn(__fmul_rn((float)pos, fscale), powf(base, __fdiv_rn((float)(2 * d), (float)hd)));
      c = cosf(theta);
      s = sinf(theta);
    }
    const float x0 = row[d], x1 = row[d + half];
    r0[cnt] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    r1[cnt] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
  }
  __syncwarp();
  cnt = 0;
  for (int d = lane; d < half && cnt < 4; d += 32, ++cnt) {
    row[d] = r0[cnt];
    row[d + half] = r1[cnt];
  }
  __syncwarp();
}

}  // namespace mcpo
