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
//  * weights are pre-tiled at upload (layout.cuh) so that every warp load is
//    a coalesced 512-byte 128-bit access with L1 bypass;
//  * the Q8_1 activation vector lives in shared memory, transposed to
//    [16-byte chunk][super-block] so lanes of a row read consecutive 16-byte
//    words without bank conflicts;
//  * up to three matrices sharing one input (q/k/v, gate/up) are one launch
//    over a common tile space, dtype chosen per CTA tile;
//  * epilogues: store, residual add, SwiGLU pairing of gate and up rows.
#include "gemv.cuh"

#include <math.h>

namespace mcpo {

namespace {

struct XShared {
  const uint4* xs;    // [16][nb] 16-byte chunks of q8
  const float* xd;    // [cols/32] d8 (f32 of the f16 d)
  const float* xds;   // [cols/32] d8 * sum(q8)
  const int* xs16;    // [cols/16] sum(q8) over 16 values
  int nb;
};

__device__ __forceinline__ int dot4(uint4 w, uint4 x, int acc) {
  acc = dp4a((int)w.x, (int)x.x, acc);
  acc = dp4a((int)w.y, (int)x.y, acc);
  acc = dp4a((int)w.z, (int)x.z, acc);
  acc = dp4a((int)w.w, (int)x.w, acc);
  return acc;
}

__device__ __forceinline__ uint4 and4(uint4 v, uint32_t m) { return make_uint4(v.x & m, v.y & m, v.z & m, v.w & m); }
__device__ __forceinline__ uint4 shr4(uint4 v, int s) { return make_uint4(v.x >> s, v.y >> s, v.z >> s, v.w >> s); }
__device__ __forceinline__ uint4 or4(uint4 a, uint4 b) { return make_uint4(a.x | b.x, a.y | b.y, a.z | b.z, a.w | b.w); }
__device__ __forceinline__ uint4 shl4(uint4 v, int s) { return make_uint4(v.x << s, v.y << s, v.z << s, v.w << s); }

// ---- Q4_K super-block: c[0] = {d, dmin, scales}, c[1..8] = qs ----
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
    int dlo = dot4(and4(q0, 0x0f0f0f0fu), x0, 0);
    dlo = dot4(and4(q1, 0x0f0f0f0fu), x1, dlo);
    int dhi = dot4(and4(shr4(q0, 4), 0x0f0f0f0fu), x2, 0);
    dhi = dot4(and4(shr4(q1, 4), 0x0f0f0f0fu), x3, dhi);
    const int j0 = 2 * g, j1 = 2 * g + 1;
    const uint32_t scw = j0 < 4 ? sc_lo : sc_hi, mnw = j0 < 4 ? mn_lo : mn_hi;
    const int s0 = (scw >> (8 * (j0 & 3))) & 0xff, s1 = (scw >> (8 * (j1 & 3))) & 0xff;
    const int m0 = (mnw >> (8 * (j0 & 3))) & 0xff, m1 = (mnw >> (8 * (j1 & 3))) & 0xff;
    const int xb = sb * 8;
    const float t0 = __fmul_rn(__fmul_rn((float)s0, x.xd[xb + j0]), (float)dlo);
    const float t1 = __fmul_rn(__fmul_rn((float)s1, x.xd[xb + j1]), (float)dhi);
    sum_d = __fadd_rn(sum_d, __fadd_rn(t0, t1));
    sum_m = __fadd_rn(sum_m, __fadd_rn(__fmul_rn((float)m0, x.xds[xb + j0]), __fmul_rn((float)m1, x.xds[xb + j1])));
    if (kDots && dots) {
      dots[sb * 8 + j0] = dlo;
      dots[sb * 8 + j1] = dhi;
    }
  }
  return __fsub_rn(__fmul_rn(d, sum_d), __fmul_rn(dmin, sum_m));
}

// ---- Q6_K super-block: c[0..7] = ql, c[8..11] = qh, c[12] = sc, d separate ----
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
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int g = 8 * n + 2 * qq + h;
        const uint4 qlw = c[4 * n + ((qq & 1) ? 2 : 0) + h];
        const uint4 qhw = c[8 + 2 * n + h];
        const uint4 lo = and4(shr4(qlw, (qq >= 2) ? 4 : 0), 0x0f0f0f0fu);
        const uint4 hi = shl4(and4(shr4(qhw, 2 * qq), 0x03030303u), 4);
        const int raw = dot4(or4(lo, hi), x.xs[g * x.nb + sb], 0);
        const int dotg = raw - 32 * x.xs16[sb * 16 + g];
        const int scale = (int)(int8_t)((scw[g >> 2] >> (8 * (g & 3))) & 0xff);
        sum = __fadd_rn(sum, __fmul_rn(x.xd[sb * 8 + (g >> 1)], __fmul_rn((float)dotg, (float)scale)));
        if (kDots && dots) dots[sb * 16 + g] = dotg;
      }
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
    sum = __fadd_rn(sum, __fmul_rn(__fmul_rn(dwf, x.xd[sb * 8 + b]), (float)acc));
    if (kDots && dots) dots[sb * 8 + b] = acc;
  }
  return sum;
}

// Dot of one lane tile row segment: the lane's super-blocks of one row.
template <int kDtype, bool kDots>
__device__ __forceinline__ float lane_row_dot(const uint8_t* tile_base, const GemvSeg& s, int warp, int lane,
                                              int lane_in_row, const XShared& x, int* dots) {
  constexpr int kChunks = kDtype == kQ4_K ? 9 : kDtype == kQ6_K ? 13 : 17;
  float acc = 0.0f;
  for (int k = 0; k < s.ks; ++k) {
    const uint8_t* blk = tile_base + ((size_t)k * kGemvWarps + warp) * s.step_bytes;
    uint4 c[kChunks];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) c[i] = ldg_stream(blk + i * 512 + lane * 16);
    const int sb = k * s.lpr + lane_in_row;
    if (kDtype == kQ4_K) {
      acc = __fadd_rn(acc, sb_dot_q4k<kDots>(c, x, sb, dots));
    } else if (kDtype == kQ6_K) {
      const uint16_t db = *reinterpret_cast<const uint16_t*>(blk + 13 * 512 + lane * 2);
      acc = __fadd_rn(acc, sb_dot_q6k<kDots>(c, db, x, sb, dots));
    } else {
      acc = __fadd_rn(acc, sb_dot_q80<kDots>(c, x, sb, dots));
    }
  }
  return acc;
}

template <bool kDots>
__device__ __forceinline__ float seg_row_dot(const uint8_t* tile_base, const GemvSeg& s, int warp, int lane,
                                             int lane_in_row, const XShared& x, int* dots) {
  if (s.dtype == kQ4_K) return lane_row_dot<kQ4_K, kDots>(tile_base, s, warp, lane, lane_in_row, x, dots);
  if (s.dtype == kQ6_K) return lane_row_dot<kQ6_K, kDots>(tile_base, s, warp, lane, lane_in_row, x, dots);
  return lane_row_dot<kQ8_0, kDots>(tile_base, s, warp, lane, lane_in_row, x, dots);
}

// Butterfly over the lpr lanes of a row (xor lpr/2 .. 1); the row's value is
// the one of its first lane.
__device__ __forceinline__ float reduce_row(float v, int lpr) {
  for (int o = lpr >> 1; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <bool kDots>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int cols = a.cols;
  const int nb = cols / 256;
  const int nblk = cols / 32;
  uint4* xs = reinterpret_cast<uint4*>(smem);
  float* xd = reinterpret_cast<float*>(smem + cols);
  float* xds = xd + nblk;
  int* xs16 = reinterpret_cast<int*>(xds + nblk);

  // Prologue: Q8_1 blocks -> shared, transposed to [chunk][super-block].
  for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.xq + (size_t)b * 36);
    const uint32_t hdr = __ldg(src);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __ldg(src + 1 + i);
    int s_lo = 0, s_hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) s_lo = dp4a((int)q[i], 0x01010101, s_lo);
#pragma unroll
    for (int i = 4; i < 8; ++i) s_hi = dp4a((int)q[i], 0x01010101, s_hi);
    const float d8 = f16_to_f32((uint16_t)(hdr & 0xffffu));
    xd[b] = d8;
    xds[b] = __fmul_rn(d8, (float)(s_lo + s_hi));
    xs16[2 * b] = s_lo;
    xs16[2 * b + 1] = s_hi;
    const int sb = b >> 3, c = (b & 7) * 2;
    xs[c * nb + sb] = make_uint4(q[0], q[1], q[2], q[3]);
    xs[(c + 1) * nb + sb] = make_uint4(q[4], q[5], q[6], q[7]);
  }
  __syncthreads();
  const XShared x{xs, xd, xds, xs16, nb};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x) {
    GemvSeg s = a.seg[0];
    if (a.nseg > 1 && tile >= a.seg[1].tile_begin) s = a.seg[1];
    if (a.nseg > 2 && tile >= a.seg[2].tile_begin) s = a.seg[2];
    const int lt = tile - s.tile_begin;
    const int row_in_warp = lane / s.lpr, lane_in_row = lane % s.lpr;
    const int row = lt * (kGemvWarps * s.rpw) + warp * s.rpw + row_in_warp;
    int* dots = nullptr;
    if (kDots) {
      // only meaningful for single-segment launches (parity tests)
      const int per_row = s.dtype == kQ6_K ? cols / 16 : cols / 32;
      dots = a.dots + (size_t)(row < s.rows ? row : 0) * per_row;
    }
    const uint8_t* tb = s.w + (size_t)lt * s.cta_tile_bytes;
    float acc = seg_row_dot<kDots>(tb, s, warp, lane, lane_in_row, x, (kDots && row < s.rows) ? dots : nullptr);
    acc = reduce_row(acc, s.lpr);
    if (s.epi == kEpiSwiglu) {
      const uint8_t* tb2 = s.w2 + (size_t)lt * s.cta_tile_bytes;
      float up = seg_row_dot<false>(tb2, s, warp, lane, lane_in_row, x, nullptr);
      up = reduce_row(up, s.lpr);
      if (lane_in_row == 0 && row < s.rows) s.y[row] = silu_mul_det(acc, up);
    } else if (lane_in_row == 0 && row < s.rows) {
      if (s.epi == kEpiAdd)
        s.y[row] = __fadd_rn(s.y[row], acc);
      else
        s.y[row] = acc;
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

size_t gemv_smem_bytes(int cols) { return (size_t)cols + (size_t)(cols / 32) * 8 + (size_t)(cols / 16) * 4; }

cudaError_t launch_gemv(GemvArgs& a, int grid, cudaStream_t st) {
  int tiles = 0;
  for (int i = 0; i < a.nseg; ++i) {
    a.seg[i].tile_begin = tiles;
    tiles += a.seg[i].n_tiles;
  }
  a.total_tiles = tiles;
  if (tiles == 0) return cudaSuccess;
  const size_t smem = gemv_smem_bytes(a.cols);
  if (grid <= 0 || grid > tiles) grid = tiles;
  if (a.dots)
    k_gemv<true><<<grid, kGemvThreads, smem, st>>>(a);
  else
    k_gemv<false><<<grid, kGemvThreads, smem, st>>>(a);
  return cudaGetLastError();
}

int gemv_occupancy(int cols) {
  const size_t smem = gemv_smem_bytes(cols);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(k_gemv<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(k_gemv<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv<false>, kGemvThreads, smem) != cudaSuccess) n = 1;
  return n > 0 ? n : 1;
}

cudaError_t launch_quantize_q8_1(const float* x, int n, uint8_t* xq, cudaStream_t st) {
  const int blocks = n / 32;
  const int grid = (blocks + 7) / 8;
  k_quantize_q8_1<<<grid, 256, 0, st>>>(x, n, xq);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_q8_1(const float* x, const void* w, int w_dtype, int n, float eps, float* out, uint8_t* xq,
                                cudaStream_t st) {
  const int blocks = (n + 31) / 32;
  int grid = (blocks + 7) / 8;
  if (grid > 32) grid = 32;
  k_rmsnorm_q8_1<<<grid, 256, 0, st>>>(x, w, w_dtype, n, eps, out, xq);
  return cudaGetLastError();
}

cudaError_t launch_dense_gemv(const void* w, int dtype, int rows, int cols, const float* x, float* y, cudaStream_t st) {
  const int grid = (rows * 32 + 255) / 256;
  k_dense_gemv<<<grid, 256, 0, st>>>(w, dtype, rows, cols, x, y);
  return cudaGetLastError();
}

}  // namespace mcpo
