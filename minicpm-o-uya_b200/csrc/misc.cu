// misc.cu -- small kernels of the decode step: weight re-layout at upload,
// token-embedding dequant lookup, greedy sampler, and the elementwise slot
// operations of the reference ABI.
#include "misc.cuh"

#include <math.h>

#include "attn_dev.cuh"
#include "gemv.cuh"
#include "rowops.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

// ---------------------------------------------------------------------
// upload re-layout: GGUF rows -> warp tiles (layout.cuh).  One thread per
// 16-byte destination chunk (plus one per Q6_K d).  Bytes are moved, never
// changed.
// ---------------------------------------------------------------------
__global__ void k_relayout(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, TileGeom g, size_t row_bytes) {
  const int per_sb = g.chunks + (g.dtype == kQ6_K ? 1 : 0);
  const size_t total = (size_t)g.rows * g.nb * per_sb;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(idx % per_sb);
    const size_t rs = idx / per_sb;
    const int sb = (int)(rs % g.nb);
    const int row = (int)(rs / g.nb);
    const uint8_t* s = src + (size_t)row * row_bytes;
    if (g.dtype == kQ6_K && c == g.chunks) {
      const uint8_t* b = s + (size_t)sb * 210 + 208;
      uint8_t* o = dst + tiled_byte_offset(g, row, sb, 208);
      o[0] = b[0];
      o[1] = b[1];
      continue;
    }
    uint8_t tmp[16];
    if (g.dtype == kQ8_0) {
      const uint8_t* grp = s + (size_t)sb * 8 * 34;  // 8 GGUF blocks of 34 B
      if (c == 0) {
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          tmp[2 * b] = grp[b * 34];
          tmp[2 * b + 1] = grp[b * 34 + 1];
        }
      } else {
        const int b = (c - 1) / 2, half = (c - 1) % 2;
#pragma unroll
        for (int i = 0; i < 16; ++i) tmp[i] = grp[b * 34 + 2 + half * 16 + i];
      }
    } else {
      const uint8_t* blk = s + (size_t)sb * g.sb_bytes + c * 16;
#pragma unroll
      for (int i = 0; i < 16; ++i) tmp[i] = blk[i];
    }
    uint4 v;
    memcpy(&v, tmp, 16);
    *reinterpret_cast<uint4*>(dst + tiled_byte_offset(g, row, sb, c * 16)) = v;
  }
}

// ---------------------------------------------------------------------
// token embedding lookup (qwen3.uya:1164-1174 and the row dequantisers
// qwen3.uya:1069-1149 / 836-856), one thread per value, the reference's
// float operation sequence with round-to-nearest intrinsics.
// ---------------------------------------------------------------------
__device__ __forceinline__ uint8_t tb(const uint8_t* w, const TileGeom& g, int row, int sb, int o) {
  return w[tiled_byte_offset(g, row, sb, o)];
}

// Sequence blockIdx.y reads its token at tok_ptr[y * tok_stride] and
// writes out + y * hidden.
__global__ void k_embed(const uint8_t* __restrict__ w, TileGeom g, int dtype, int rows, int hidden, const int* tok_ptr,
                        int tok_static, float* __restrict__ out, int tok_stride, const float* __restrict__ in_row,
                        const int* in_flag) {
  pdl_wait();
  pdl_launch_dependents();
  if (in_flag && *in_flag) {  // the caller's input row (qwen3_append_prompt_embeddings)
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < hidden; e += gridDim.x * blockDim.x) out[e] = in_row[e];
    return;
  }
  const int token = tok_ptr ? tok_ptr[(size_t)blockIdx.y * tok_stride] : tok_static;
  out += (size_t)blockIdx.y * hidden;
  if (token < 0 || token >= rows) {  // never index outside the table; the host validates ids
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < hidden; e += gridDim.x * blockDim.x) out[e] = 0.0f;
    return;
  }
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < hidden; e += gridDim.x * blockDim.x) {
    float v;
    if (dtype == kF32) {
      v = reinterpret_cast<const float*>(w)[(size_t)token * hidden + e];
    } else if (dtype == kF16 || dtype == kBF16) {
      v = load_weight(w + (size_t)token * hidden * 2, dtype, e);
    } else {
      const int sb = e / 256, i = e % 256;
      if (dtype == kQ4_K) {
        const float d = f16_to_f32((uint16_t)(tb(w, g, token, sb, 0) | (tb(w, g, token, sb, 1) << 8)));
        const float dmin = f16_to_f32((uint16_t)(tb(w, g, token, sb, 2) | (tb(w, g, token, sb, 3) << 8)));
        const int grp = i / 64, within = i % 64, hi = within >= 32, l = within % 32;
        const int j = 2 * grp + hi;
        uint8_t s8[12];
#pragma unroll
        for (int k = 0; k < 12; ++k) s8[k] = tb(w, g, token, sb, 4 + k);
        int sc, mn;
        if (j < 4) {
          sc = s8[j] & 63;
          mn = s8[j + 4] & 63;
        } else {
          sc = (s8[j + 4] & 15) | ((s8[j - 4] >> 6) << 4);
          mn = (s8[j + 4] >> 4) | ((s8[j] >> 6) << 4);
        }
        const uint8_t qb = tb(w, g, token, sb, 16 + grp * 32 + l);
        const int q = hi ? (qb >> 4) : (qb & 15);
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
        v = __fsub_rn(__fmul_rn(d1, (float)q), m1);
      } else if (dtype == kQ6_K) {
        const float d = f16_to_f32((uint16_t)(tb(w, g, token, sb, 208) | (tb(w, g, token, sb, 209) << 8)));
        const int n = i / 128 * 128, r = i - n, quarter = r / 32, l = r % 32;
        int lo, hh;
        if (quarter == 0) { lo = tb(w, g, token, sb, n / 2 + l) & 15; hh = (tb(w, g, token, sb, 128 + n / 4 + l) >> 0) & 3; }
        else if (quarter == 1) { lo = tb(w, g, token, sb, n / 2 + l + 32) & 15; hh = (tb(w, g, token, sb, 128 + n / 4 + l) >> 2) & 3; }
        else if (quarter == 2) { lo = tb(w, g, token, sb, n / 2 + l) >> 4; hh = (tb(w, g, token, sb, 128 + n / 4 + l) >> 4) & 3; }
        else { lo = tb(w, g, token, sb, n / 2 + l + 32) >> 4; hh = (tb(w, g, token, sb, 128 + n / 4 + l) >> 6) & 3; }
        const int q = (lo | (hh << 4)) - 32;
        const int sc = (int8_t)tb(w, g, token, sb, 192 + i / 16);
        v = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
      } else {  // Q8_0 (tiled order: 0..15 = d's, 16.. = quants)
        const int b = i / 32, l = i % 32;
        const float d = f16_to_f32((uint16_t)(tb(w, g, token, sb, 2 * b) | (tb(w, g, token, sb, 2 * b + 1) << 8)));
        const int q = (int8_t)tb(w, g, token, sb, 16 + b * 32 + l);
        v = __fmul_rn(d, (float)q);
      }
    }
    out[e] = v;
  }
}

// ---------------------------------------------------------------------
// greedy sampler (qwen3.uya:1734-1752): first maximum of the penalised
// logits, plus the gap to the second-best value.  Per-CTA partials, merged
// by the last CTA to finish.
// ---------------------------------------------------------------------
struct Top2 {
  float b;
  int i;
  float s;
};

__device__ __forceinline__ Top2 merge(Top2 x, Top2 y) {
  const bool ywins = (y.b > x.b) || (y.b == x.b && y.i < x.i);
  const Top2 w = ywins ? y : x, l = ywins ? x : y;
  Top2 r;
  r.b = w.b;
  r.i = w.i;
  r.s = fmaxf(fmaxf(w.s, l.s), l.b);
  return r;
}

__device__ __forceinline__ Top2 warp_merge(Top2 t) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Top2 u;
    u.b = __shfl_xor_sync(0xffffffffu, t.b, o);
    u.i = __shfl_xor_sync(0xffffffffu, t.i, o);
    u.s = __shfl_xor_sync(0xffffffffu, t.s, o);
    t = merge(t, u);
  }
  return t;
}

__global__ void __launch_bounds__(256) k_argmax(const float* __restrict__ logits, int n, const uint32_t* seen_bits,
                                                float* scratch, unsigned* counter, StepState* st, int* history,
                                                int history_cap, int vocab_base, float* tp_top) {
  pdl_wait();
  pdl_launch_dependents();
  // independent sequences along grid y: logits, scratch, counter, state and
  // history of sequence y
  logits += (size_t)blockIdx.y * n;
  scratch += (size_t)blockIdx.y * gridDim.x * 3;
  counter += blockIdx.y;
  st += blockIdx.y;
  if (history) history += (size_t)blockIdx.y * history_cap;
  const float penalty = st->penalty;
  Top2 t{-INFINITY, 0x7fffffff, -INFINITY};
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float v = logits[i];
    const int gi = i + vocab_base;  // global vocab index (a tensor-parallel slice starts at vocab_base)
    if (penalty > 1.0f && seen_bits && ((seen_bits[gi >> 5] >> (gi & 31)) & 1u)) {
      if (v > 0.0f) v = __fdiv_rn(v, penalty);
      if (v < 0.0f) v = __fmul_rn(v, penalty);
    }
    Top2 u{v, gi, -INFINITY};
    t = merge(t, u);
  }
  t = warp_merge(t);
  __shared__ Top2 ws[8];
  __shared__ unsigned ticket;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) ws[warp] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    Top2 r = ws[0];
    for (int w = 1; w < 8; ++w) r = merge(r, ws[w]);
    scratch[blockIdx.x * 3 + 0] = r.b;
    scratch[blockIdx.x * 3 + 1] = __int_as_float(r.i);
    scratch[blockIdx.x * 3 + 2] = r.s;
    __threadfence();
    ticket = atomicAdd(counter, 1u);
  }
  __syncthreads();
  if (ticket != gridDim.x - 1) return;
  __threadfence();
  Top2 r{-INFINITY, 0x7fffffff, -INFINITY};
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    Top2 u{__ldcg(scratch + b * 3), __float_as_int(__ldcg(scratch + b * 3 + 1)), __ldcg(scratch + b * 3 + 2)};
    r = merge(r, u);
  }
  r = warp_merge(r);
  if (lane == 0) ws[warp] = r;
  __syncthreads();
  if (threadIdx.x == 0) {
    Top2 f = ws[0];
    for (int w = 1; w < 8; ++w) f = merge(f, ws[w]);
    *counter = 0u;
    if (tp_top) {  // a slice of the vocab: the cross-rank merge finishes the step
      tp_top[0] = f.b;
      tp_top[1] = __int_as_float(f.i);
      tp_top[2] = f.s;
      return;
    }
    if (f.i < 0 || f.i >= n) {  // every value NaN: report token 0 and flag it
      f.i = 0;
      st->err = 1;
    }
    st->next_token = f.i;
    st->best = f.b;
    st->gap = f.b - f.s;
    if (st->auto_advance) {
      if (history && st->history_len < history_cap) history[st->history_len] = f.i;
      st->history_len = st->history_len + 1;
      st->token = f.i;
      st->pos = st->pos + 1;
    }
  }
}

__global__ void k_mark_seen(uint32_t* bits, const StepState* st, int vocab) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = st->token;
  if (t >= 0 && t < vocab) atomicOr(&bits[t >> 5], 1u << (t & 31));
}

// qwen3_sample (qwen3.uya:2073-2138) for vocab <= 256, one CTA of 256
// threads: greedy (argmax, the penalty once per seen token) unless
// temperature > 1e-6 and top_k > 1; then the penalty per seen-list entry in
// list order, logits / temperature, softmax (kernels.uya:149-160: max
// scan, expf, sequential sum, divisions), the reference's swap selection
// sort (descending, not stable), top-k, top-p, min-p, renormalisation and
// one xorshift32 draw (qwen3.uya:2046-2057).  The steps the reference runs
// in sequence run on one thread, in the same order; the element-wise ones
// on all.  io[0] = xorshift32 state (in/out), io[1] = the token.
__global__ void __launch_bounds__(256) k_sample_small(const float* __restrict__ logits, int vocab,
                                                      const uint32_t* __restrict__ seen, int seen_count, float temp,
                                                      uint32_t top_k, float top_p, float min_p, float penalty,
                                                      uint32_t* io) {
  __shared__ float local[256], probs[256];
  __shared__ uint32_t order[256];
  __shared__ unsigned char flag[256];
  __shared__ float s_max, s_sum;
  const int t = threadIdx.x;
  if (t < vocab) {
    local[t] = logits[t];
    order[t] = (uint32_t)t;
    flag[t] = 0;
  }
  __syncthreads();
  if (temp <= 0.000001f || top_k <= 1) {
    for (int i = t; i < seen_count; i += blockDim.x)
      if (seen[i] < (uint32_t)vocab) flag[seen[i]] = 1;
    __syncthreads();
    if (t == 0) {
      int best = 0;
      float bv = local[0];
      if (penalty > 1.0f && flag[0]) {
        if (bv > 0.0f) bv = __fdiv_rn(bv, penalty);
        if (bv < 0.0f) bv = __fmul_rn(bv, penalty);
      }
      for (int i = 1; i < vocab; ++i) {
        float v = local[i];
        if (penalty > 1.0f && flag[i]) {
          if (v > 0.0f) v = __fdiv_rn(v, penalty);
          if (v < 0.0f) v = __fmul_rn(v, penalty);
        }
        if (v > bv) {
          best = i;
          bv = v;
        }
      }
      io[1] = (uint32_t)best;
    }
    return;
  }
  if (t == 0 && penalty > 1.0f) {
    for (int i = 0; i < seen_count; ++i) {
      const uint32_t s = seen[i];
      if (s < (uint32_t)vocab) {
        if (local[s] > 0.0f) local[s] = __fdiv_rn(local[s], penalty);
        if (local[s] < 0.0f) local[s] = __fmul_rn(local[s], penalty);
      }
    }
  }
  __syncthreads();
  if (t < vocab) local[t] = __fdiv_rn(local[t], temp);
  __syncthreads();
  if (t == 0) {
    float m = local[0];
    for (int i = 1; i < vocab; ++i)
      if (local[i] > m) m = local[i];
    s_max = m;
  }
  __syncthreads();
  if (t < vocab) probs[t] = expf(__fsub_rn(local[t], s_max));
  __syncthreads();
  if (t == 0) {
    float sum = 0.0f;
    for (int i = 0; i < vocab; ++i) sum = __fadd_rn(sum, probs[i]);
    s_sum = sum;
  }
  __syncthreads();
  if (t < vocab && s_sum != 0.0f) probs[t] = __fdiv_rn(probs[t], s_sum);
  __syncthreads();
  if (t != 0) return;
  for (int a = 0; a < vocab; ++a)
    for (int b = a + 1; b < vocab; ++b)
      if (probs[b] > probs[a]) {
        const float tp = probs[a];
        const uint32_t ti = order[a];
        probs[a] = probs[b];
        probs[b] = tp;
        order[a] = order[b];
        order[b] = ti;
      }
  int limit = vocab;
  if (top_k > 0 && top_k < (uint32_t)limit) limit = (int)top_k;
  float cumulative = 0.0f;
  int kept = 0;
  while (kept < limit) {
    if (kept >= vocab || kept >= 256) break;
    cumulative = __fadd_rn(cumulative, probs[kept]);
    kept = kept + 1;
    if (cumulative >= top_p && top_p < 0.999999f) break;
  }
  const float max_prob = probs[0];
  if (min_p > 0.0f)
    while (kept > 1) {
      const int tail = kept - 1;
      if (tail >= 256 || probs[tail] >= __fmul_rn(max_prob, min_p)) break;
      kept = kept - 1;
    }
  float norm = 0.0f;
  for (int i = 0; i < kept; ++i) norm = __fadd_rn(norm, probs[i]);
  uint32_t x = io[0];
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  io[0] = x;
  const float r = __fdiv_rn(__uint2float_rn(x), 4294967295.0f);
  float acc = 0.0f;
  uint32_t pick = order[0];
  for (int i = 0; i < kept; ++i) {
    acc = __fadd_rn(acc, __fdiv_rn(probs[i], norm));
    if (r <= acc || i + 1 == kept) {
      pick = order[i];
      break;
    }
  }
  io[1] = pick;
}

// Seen bits of a token list (tokens >= vocab ignored).
__global__ void k_seen_bits(uint32_t* bits, const uint32_t* list, int n, int vocab) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    if (list[i] < (uint32_t)vocab) atomicOr(&bits[list[i] >> 5], 1u << (list[i] & 31));
}

// ---------------------------------------------------------------------
// elementwise slot kernels (gpu_shim.c:649-745)
// ---------------------------------------------------------------------
__global__ void k_add_inplace(float* dst, const float* src, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = __fadd_rn(dst[i], src[i]);
}

__global__ void k_silu_mul(float* dst, const float* gate, const float* up, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = silu_mul_det(gate[i], up[i]);
}

// In-place per-head RMSNorm and/or RoPE, one warp per head.
__global__ void k_head_norm_rope(float* vec, int n_head, int hd, const void* w, int w_dtype, int do_rope,
                                 const float* cos_t, const float* sin_t, float base, float fscale, int pos) {
  __shared__ float row_s[4][256];
  __shared__ float sq_s[4][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x * 4 + warp;
  if (h >= n_head) return;
  float* row = row_s[warp];
  for (int d = lane; d < hd; d += 32) row[d] = vec[(size_t)h * hd + d];
  __syncwarp();
  norm_rope_row(row, sq_s[warp], hd, w, w_dtype, do_rope != 0, cos_t, sin_t, base, fscale, pos, lane);
  for (int d = lane; d < hd; d += 32) vec[(size_t)h * hd + d] = row[d];
}

// Prompt prefill: for token t of a chunk (position pos[t]), the per-head
// QK-RMSNorm + RoPE of its q and k heads in place (norm_rope_row, as the
// decode step's attention prologue) and the append of its k and v rows to
// the cache (the value the cache stores: f16-rounded for an f16 cache).
// One warp per head, q heads first; rows of q/k/v `stride` floats apart.
template <typename T>
__global__ void k_prompt_qk(float* q, float* k, const float* v, int stride, int n_head, int n_kv, int hd,
                            const void* qn, int qndt, const void* kn, int kndt, const float* cos_t,
                            const float* sin_t, float base, float fscale, const int* pos, void* kc, void* vc) {
  __shared__ float row_s[4][256];
  __shared__ float sq_s[4][256];
  pdl_wait();  // q/k/v come from the q/k/v GEMV
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x, hh = blockIdx.y * 4 + warp;
  if (hh >= n_head + n_kv) return;
  const int p = pos[t];
  const bool isq = hh < n_head;
  const int h = isq ? hh : hh - n_head;
  float* vec = (isq ? q : k) + (size_t)t * stride + (size_t)h * hd;
  float* row = row_s[warp];
  for (int d = lane; d < hd; d += 32) row[d] = vec[d];
  __syncwarp();
  norm_rope_row(row, sq_s[warp], hd, isq ? qn : kn, isq ? qndt : kndt, true, cos_t, sin_t, base, fscale, p, lane);
  for (int d = lane; d < hd; d += 32) vec[d] = row[d];
  if (!isq) {
    const size_t at = (size_t)p * n_kv * hd + (size_t)h * hd;
    const float* vr = v + (size_t)t * stride + (size_t)h * hd;
    for (int d = lane; d < hd; d += 32) {
      kv_store<T>(kc, at + d, row[d]);
      kv_store<T>(vc, at + d, vr[d]);
    }
  }
}

}  // namespace

cudaError_t launch_prompt_qk(float* q, float* k, const float* v, int stride, int n_tok, int n_head, int n_kv, int hd,
                             const void* qn, int qndt, const void* kn, int kndt, const float* cos_t, const float* sin_t,
                             float base, float fscale, const int* pos, void* kc, void* vc, int kv_f16,
                             cudaStream_t st) {
  if (hd > 256 || n_tok < 1) return cudaErrorInvalidValue;
  const dim3 grid(n_tok, (n_head + n_kv + 3) / 4);
  // programmatic dependent launch: the CTAs wait for the q/k/v GEMV in the
  // kernel (the kernel never triggers its dependents early)
  if (kv_f16)
    return launch_k(k_prompt_qk<__half>, grid, dim3(128), 0, st, true, q, k, v, stride, n_head, n_kv, hd, qn, qndt, kn,
                    kndt, cos_t, sin_t, base, fscale, pos, kc, vc);
  return launch_k(k_prompt_qk<float>, grid, dim3(128), 0, st, true, q, k, v, stride, n_head, n_kv, hd, qn, qndt, kn,
                  kndt, cos_t, sin_t, base, fscale, pos, kc, vc);
}

cudaError_t launch_relayout(const uint8_t* src, uint8_t* dst, const TileGeom& g, size_t row_bytes, cudaStream_t st) {
  const int per_sb = g.chunks + (g.dtype == kQ6_K ? 1 : 0);
  const size_t total = (size_t)g.rows * g.nb * per_sb;
  size_t grid = (total + 255) / 256;
  if (grid > 65535u * 8u) grid = 65535u * 8u;
  k_relayout<<<(unsigned)grid, 256, 0, st>>>(src, dst, g, row_bytes);
  return cudaGetLastError();
}

cudaError_t launch_embed(const uint8_t* w, const TileGeom& g, int dtype, int rows, int hidden, const int* tok_ptr, int tok,
                         float* out, cudaStream_t st, bool pdl, int batch, int tok_stride, const float* in_row,
                         const int* in_flag) {
  const int grid = (hidden + 255) / 256;
  if (in_flag && (!in_row || batch > 1)) return cudaErrorInvalidValue;
  return launch_k(k_embed, dim3(grid, batch < 1 ? 1 : batch), dim3(256), 0, st, pdl, w, g, dtype, rows, hidden, tok_ptr,
                  tok, out, tok_stride, in_row, in_flag);
}

cudaError_t launch_argmax(const float* logits, int n, const uint32_t* seen_bits, float* scratch, unsigned* counter,
                          StepState* st, int* history, int history_cap, int grid, cudaStream_t s, bool pdl,
                          int vocab_base, float* tp_top, int batch) {
  if (grid <= 0) grid = 1;
  if (batch > 1 && (seen_bits || tp_top)) return cudaErrorInvalidValue;
  return launch_k(k_argmax, dim3(grid, batch < 1 ? 1 : batch), dim3(256), 0, s, pdl, logits, n, seen_bits, scratch,
                  counter, st, history, history_cap, vocab_base, tp_top);
}

cudaError_t launch_sample_small(const float* logits, int vocab, const uint32_t* seen, int seen_count, float temp,
                                uint32_t top_k, float top_p, float min_p, float penalty, uint32_t* io, cudaStream_t st) {
  if (vocab < 1 || vocab > 256) return cudaErrorInvalidValue;
  k_sample_small<<<1, 256, 0, st>>>(logits, vocab, seen, seen_count, temp, top_k, top_p, min_p, penalty, io);
  return cudaGetLastError();
}

cudaError_t launch_seen_bits(uint32_t* bits, const uint32_t* list, int n, int vocab, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_seen_bits<<<(n + 255) / 256, 256, 0, st>>>(bits, list, n, vocab);
  return cudaGetLastError();
}

cudaError_t launch_mark_seen(uint32_t* bits, const StepState* st, int vocab, cudaStream_t s, bool pdl) {
  return launch_k(k_mark_seen, dim3(1), dim3(32), 0, s, pdl, bits, st, vocab);
}

cudaError_t launch_add_inplace(float* dst, const float* src, int n, cudaStream_t st) {
  k_add_inplace<<<(n + 255) / 256, 256, 0, st>>>(dst, src, n);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(float* dst, const float* gate, const float* up, int n, cudaStream_t st) {
  k_silu_mul<<<(n + 255) / 256, 256, 0, st>>>(dst, gate, up, n);
  return cudaGetLastError();
}

cudaError_t launch_head_norm_rope(float* vec, int n_head, int hd, const void* w, int w_dtype, int do_rope,
                                  const float* cos_t, const float* sin_t, float base, float fscale, int pos,
                                  cudaStream_t st) {
  k_head_norm_rope<<<(n_head + 3) / 4, 128, 0, st>>>(vec, n_head, hd, w, w_dtype, do_rope, cos_t, sin_t, base, fscale,
                                                     pos);
  return cudaGetLastError();
}

}  // namespace mcpo
