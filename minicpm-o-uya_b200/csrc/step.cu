// step.cu -- the persistent decode-step kernel for sm_100a.
//
// One cooperative launch of one CTA per SM runs a whole token: per layer
//   GEMV q/k/v   (RMSNorm -> Q8_1 prologue, three segments)
//   attention    (QK-RMSNorm + RoPE + KV append, split-K flash decoding,
//                 last-arriving CTA merges and quantises the output)
//   GEMV o       (Q8_1 input, residual add)
//   GEMV gate/up (RMSNorm -> Q8_1 prologue, SwiGLU epilogue)
//   GEMV down    (f32 -> Q8_1 prologue, residual add)
// then the final RMSNorm -> lm_head GEMV.  The order and arithmetic are
// those of the per-kernel step (gemv.cu, attention.cu), so the logits are
// bit-identical to it.
//
// Why one kernel: batch-1 decode is a weight stream (4.9 GB per token for
// the 8B shape) cut into ~180 dependent pieces.  As separate launches each
// piece pays launch latency, a cold instruction cache and a pipeline ramp
// and drain.  Here the weight stream never stops: the producer warp of each
// CTA knows the whole step's schedule (which step blocks of which matrix
// its consumers will need, in order) and keeps its ring of shared-memory
// slots full across stage boundaries, while the consumer warps wait at the
// grid barrier for the activations of the previous stage.
//
// Synchronisation:
//  * stages are separated by a grid barrier: a monotonically increasing
//    arrival counter in global memory (zeroed before each launch), release
//    by __threadfence + atomicAdd, acquire by ld.acquire polling;
//  * every wait is bounded (1 s of globaltimer, or an iteration cap); a CTA
//    that gives up raises the error word and a global abort flag, the other
//    CTAs see the flag at their next wait and leave; the producer leaves
//    only after the copies it issued into shared memory have landed;
//  * the launch is cooperative, so all CTAs are co-resident.
#include "step.cuh"

#include <math.h>
#include <stdlib.h>

#include "attn_dev.cuh"
#include "common.cuh"
#include "gemv_dev.cuh"
#include "rowops.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr int kGMax = 8;          // q heads per kv head
constexpr int kMaxSplitS = 64;    // splits per kv head
constexpr int kMaxPairs = 8;      // (head, dim) pairs per thread: kGMax*256 / (8 warps * 32)
constexpr int kSmemMax = 232448;  // opt-in shared memory per CTA on sm_100
constexpr int kMinConsumers = 8;
constexpr int kStepMaxConsumers = 11;  // 12 warps, 3 per SM sub-partition: up to 168 registers

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Named barrier 1 over the consumer warps (the producer warp never joins).
__device__ __forceinline__ void cbar(int nthr) { asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory"); }

__device__ __forceinline__ void raise_abort(const StepPlan& p, volatile int* abort_s, bool error) {
  *abort_s = 1;
  if (error) atomicExch(p.err, 1);
  atomicExch(p.abort, 1);
}

// Arrive for the stages done so far and wait until all CTAs have (arrival
// count >= target).  Called by all consumer threads; false on abort.
__device__ bool grid_sync(const StepPlan& p, unsigned target, int nthr, volatile int* abort_s) {
  cbar(nthr);
  if (threadIdx.x == 0 && !*abort_s) {
    __threadfence();
    atomicAdd(p.bar, 1u);
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 0;; ++it) {
      if (ld_acquire_gpu(p.bar) >= target) break;
      if (*reinterpret_cast<volatile int*>(p.abort)) {
        *abort_s = 1;
        break;
      }
      if ((it & 255u) == 255u && (globaltimer_ns() - t0 > 1000000000ull || it > (1u << 23))) {
        raise_abort(p, abort_s, true);
        break;
      }
    }
    __threadfence();
  }
  cbar(nthr);
  return *abort_s == 0;
}

// ---------------------------------------------------------------------
// attention stage
// ---------------------------------------------------------------------
struct AttnStageSmem {
  float* q;      // [kGMax][hd]; the merged rows after the merge
  float* kpos;   // [hd]
  float* vpos;   // [hd]
  float* sq;     // [kGMax + 1][256] norm scratch (row g; the k row last)
  float* ps;     // [kGMax][kSub] probabilities of the sub-chunk
  float* alpha;  // [kGMax]
  float* kt;     // [kSub][hd + 1]
  float* vt;     // [kSub][hd + 1]
  float* cm;     // merge: [kGMax][kMaxSplitS] (aliases kt/vt)
  float* cl;
  float* cw;
  float* cinv;   // [kGMax]
};

__host__ __device__ inline size_t attn_stage_floats(int hd) {
  const size_t tile = 2 * (size_t)kSub * (hd + 1);
  const size_t merge = 3 * (size_t)kGMax * kMaxSplitS + kGMax;  // aliases the tile
  return (size_t)kGMax * hd + 2 * (size_t)hd + (kGMax + 1) * 256 + kGMax * kSub + kGMax + (tile > merge ? tile : merge);
}

__device__ __forceinline__ AttnStageSmem carve_stage(float* base, int hd) {
  AttnStageSmem s;
  s.q = base;
  s.kpos = s.q + kGMax * hd;
  s.vpos = s.kpos + hd;
  s.sq = s.vpos + hd;
  s.ps = s.sq + (kGMax + 1) * 256;
  s.alpha = s.ps + kGMax * kSub;
  s.kt = s.alpha + kGMax;
  s.vt = s.kt + kSub * (hd + 1);
  s.cm = s.kt;
  s.cl = s.cm + kGMax * kMaxSplitS;
  s.cw = s.cl + kGMax * kMaxSplitS;
  s.cinv = s.cw + kGMax * kMaxSplitS;
  return s;
}

// One warp loads row[0..hd) from global memory (all loads first).
__device__ __forceinline__ void load_row(float* dst, const float* src, int hd, int lane) {
  float r[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) r[k] = lane + 32 * k < hd ? src[lane + 32 * k] : 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    if (lane + 32 * k < hd) dst[lane + 32 * k] = r[k];
  __syncwarp();
}

// One (kv head, split) item on all NC consumer warps.  Arithmetic per
// element is that of k_attention: scores by a sequential fma over d (warp g
// = q head g, lane = position), the online-softmax update per 32-position
// sub-chunk, acc_d = acc_d*alpha then fma(p_t, v_td, acc_d) in t order (one
// thread per (head, d)), and the last arriving item of a kv head merges the
// splits in split order.
template <typename T>
__device__ void attn_item(const AttnArgs& a, const AttnStageSmem& sm, int kvh, int split, int n_active, int chunk,
                          int pos, int NC, int warp, int lane, unsigned* ticket_s) {
  const int nthr = NC * 32, tid = warp * 32 + lane;
  const int hd = a.head_dim, hs = hd + 1;
  const int hb = (kvh * a.n_head + a.n_kv - 1) / a.n_kv;
  const int he = ((kvh + 1) * a.n_head + a.n_kv - 1) / a.n_kv;
  const int G = he - hb;
  const int n_pos = pos + 1;
  const int t0 = split * chunk;
  const int t1 = min(t0 + chunk, n_pos);
  const int kv_dim = a.n_kv * hd;
  const size_t kv_off = (size_t)kvh * hd;
  const int stride_part = attn_part_stride(hd);
  const bool fused = a.fuse_norm_rope_append != 0;

  // Everything the item reads that does not depend on its own prologue is
  // requested first: the norm weights and RoPE row (into L1), and the first
  // sub-chunk's K/V rows (into registers; the current position comes from
  // the prologue and is filled in when the tile is stored).
  if (fused && tid < 12) {
    const uint8_t* line = nullptr;
    const int qb = a.q_norm_dtype == kF32 ? 4 : 2, kb = a.k_norm_dtype == kF32 ? 4 : 2;
    if (tid < 4 && a.q_norm && tid * 128 < hd * qb) line = static_cast<const uint8_t*>(a.q_norm) + tid * 128;
    if (tid >= 4 && tid < 8 && a.k_norm && (tid - 4) * 128 < hd * kb)
      line = static_cast<const uint8_t*>(a.k_norm) + (tid - 4) * 128;
    if (tid >= 8 && a.rope_cos) {
      const float* tab = (tid < 10 ? a.rope_cos : a.rope_sin) + (size_t)pos * (hd / 2);
      if (((tid - 8) & 1) * 128 < hd * 2) line = reinterpret_cast<const uint8_t*>(tab) + ((tid - 8) & 1) * 128;
    }
    if (line) asm volatile("prefetch.global.L1 [%0];" ::"l"(line));
  }
  const int n4 = kSub * hd / 4;
  const bool early = (hd & 3) == 0 && n4 <= 4 * nthr;
  float4 pk[4], pv[4];
  if (early) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = tid + u * nthr;
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
  // prologue: current-position K/V (split 0 appends them; the last split
  // reads them), the q rows of the group
  if (fused && (split == 0 || split == n_active - 1)) {
    if (warp == NC - 1) {
      load_row(sm.kpos, a.k + kv_off, hd, lane);
      norm_rope_row(sm.kpos, sm.sq + kGMax * 256, hd, a.k_norm, a.k_norm_dtype, true, a.rope_cos, a.rope_sin,
                    a.rope_base, a.rope_scale, pos, lane);
    } else if (warp == NC - 2) {
      load_row(sm.vpos, a.v + kv_off, hd, lane);
    }
  }
  for (int g = warp; g < G; g += NC) {
    float* row = sm.q + g * hd;
    load_row(row, a.q + (size_t)(hb + g) * hd, hd, lane);
    if (fused)
      norm_rope_row(row, sm.sq + g * 256, hd, a.q_norm, a.q_norm_dtype, true, a.rope_cos, a.rope_sin, a.rope_base,
                    a.rope_scale, pos, lane);
  }
  cbar(nthr);
  if (fused && split == 0) {
    for (int d = tid; d < hd; d += nthr) {
      kv_store<T>(a.k_cache, (size_t)pos * kv_dim + kv_off + d, sm.kpos[d]);
      kv_store<T>(a.v_cache, (size_t)pos * kv_dim + kv_off + d, sm.vpos[d]);
    }
  }

  float m = -INFINITY, l = 0.0f;  // warp g < G: head g's running max / sum
  float acc[kMaxPairs];
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j) acc[j] = 0.0f;
  const int pairs = G * hd;
  for (int c0 = t0; c0 < t1; c0 += kSub) {
    if (early && c0 == t0) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = tid + u * nthr;
        if (e < n4) {
          const int r = (e * 4) / hd, d = e * 4 - r * hd, t = c0 + r;
          float4 kk = pk[u], vv = pv[u];
          if (fused && t == pos && t < t1) {
            kk = make_float4(kv_round<T>(sm.kpos[d]), kv_round<T>(sm.kpos[d + 1]), kv_round<T>(sm.kpos[d + 2]),
                             kv_round<T>(sm.kpos[d + 3]));
            vv = make_float4(kv_round<T>(sm.vpos[d]), kv_round<T>(sm.vpos[d + 1]), kv_round<T>(sm.vpos[d + 2]),
                             kv_round<T>(sm.vpos[d + 3]));
          }
          float* kd = sm.kt + r * hs + d;
          float* vd = sm.vt + r * hs + d;
          kd[0] = kk.x; kd[1] = kk.y; kd[2] = kk.z; kd[3] = kk.w;
          vd[0] = vv.x; vd[1] = vv.y; vd[2] = vv.z; vd[3] = vv.w;
        }
      }
    } else {
      stage_kv_tile<T, 4>(a.k_cache, a.v_cache, sm.kpos, sm.vpos, sm.kt, sm.vt, c0, t1, pos, fused, kv_dim, kv_off, hd,
                          hs, tid, nthr);
    }
    cbar(nthr);
    if (warp < G) {
      const float* qrow = sm.q + warp * hd;
      const bool valid = c0 + lane < t1;
      float sc = 0.0f;
      for (int d = 0; d < hd; ++d) sc = __fmaf_rn(qrow[d], sm.kt[lane * hs + d], sc);
      sc = valid ? __fmul_rn(sc, a.scale) : -INFINITY;
      const float mx = warp_max(sc);
      const float mn = fmaxf(m, mx);
      const float al = expf_det(__fsub_rn(m, mn));
      const float p = valid ? expf_det(__fsub_rn(sc, mn)) : 0.0f;
      const float psum = __shfl_sync(0xffffffffu, warp_sum(p), 0);
      l = __fadd_rn(__fmul_rn(l, al), psum);
      m = mn;
      sm.ps[warp * kSub + lane] = p;
      if (lane == 0) sm.alpha[warp] = al;
    }
    cbar(nthr);
#pragma unroll
    for (int j = 0; j < kMaxPairs; ++j) {
      const int i = tid + j * nthr;
      if (i < pairs) {
        const int g = i / hd, d = i - g * hd;
        const float* pg = sm.ps + g * kSub;
        float v = __fmul_rn(acc[j], sm.alpha[g]);
        for (int tt = 0; tt < kSub; ++tt) v = __fmaf_rn(pg[tt], sm.vt[tt * hs + d], v);
        acc[j] = v;
      }
    }
    cbar(nthr);
  }
  // partials [head][split][m, l, acc...]
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j) {
    const int i = tid + j * nthr;
    if (i < pairs) {
      const int g = i / hd, d = i - g * hd;
      a.partial[((size_t)(hb + g) * a.n_split + split) * stride_part + 4 + d] = acc[j];
    }
  }
  if (warp < G && lane == 0) {
    float* dst = a.partial + ((size_t)(hb + warp) * a.n_split + split) * stride_part;
    dst[0] = m;
    dst[1] = l;
  }

  // the last item of this kv head to finish merges the splits: the CTA
  // barrier orders every thread's partial stores before thread 0's
  // acquire-release ticket at gpu scope
  cbar(nthr);
  if (tid == 0) {
    unsigned t;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(&a.counters[kvh]) : "memory");
    *ticket_s = t;
  }
  cbar(nthr);
  if (*ticket_s != (unsigned)(n_active - 1)) return;
  if (tid == 0) atomicExch(&a.counters[kvh], 0u);
  // every partial this thread needs is requested together with m and l
  constexpr int kFastSplits = 8;
  const bool fast = n_active <= kFastSplits && pairs <= 2 * nthr;
  float pacc[2][kFastSplits];
  if (fast) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = tid + j * nthr;
      const int g = i / hd, d = i - g * hd;
#pragma unroll
      for (int sp = 0; sp < kFastSplits; ++sp)
        pacc[j][sp] = (i < pairs && sp < n_active)
                          ? __ldcg(a.partial + ((size_t)(hb + g) * a.n_split + sp) * stride_part + 4 + d)
                          : 0.0f;
    }
  }
  for (int i = tid; i < G * n_active; i += nthr) {
    const int g = i / n_active, sp = i - g * n_active;
    const float* ps = a.partial + ((size_t)(hb + g) * a.n_split + sp) * stride_part;
    sm.cm[g * kMaxSplitS + sp] = __ldcg(ps);
    sm.cl[g * kMaxSplitS + sp] = __ldcg(ps + 1);
  }
  cbar(nthr);
  for (int g = warp; g < G; g += NC) {
    const float* mg = sm.cm + g * kMaxSplitS;
    float M = -INFINITY;
    for (int sp = lane; sp < n_active; sp += 32) M = fmaxf(M, mg[sp]);
    M = warp_max(M);
    for (int sp = lane; sp < n_active; sp += 32) sm.cw[g * kMaxSplitS + sp] = expf_det(__fsub_rn(mg[sp], M));
    __syncwarp();
    if (lane == 0) {
      float L = 0.0f;
      for (int sp = 0; sp < n_active; ++sp) L = __fmaf_rn(sm.cw[g * kMaxSplitS + sp], sm.cl[g * kMaxSplitS + sp], L);
      sm.cinv[g] = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
    }
  }
  cbar(nthr);
  if (fast) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = tid + j * nthr;
      if (i < pairs) {
        const int g = i / hd, d = i - g * hd;
        const float* wg = sm.cw + g * kMaxSplitS;
        float o = 0.0f;
#pragma unroll
        for (int sp = 0; sp < kFastSplits; ++sp)
          if (sp < n_active) o = __fmaf_rn(wg[sp], pacc[j][sp], o);
        o = __fmul_rn(o, sm.cinv[g]);
        a.out[(size_t)(hb + g) * hd + d] = o;
        sm.q[i] = o;
      }
    }
  }
  constexpr int kLd = 8;
  for (int i = fast ? pairs : tid; i < pairs; i += nthr) {
    const int g = i / hd, d = i - g * hd;
    const float* pg = a.partial + (size_t)(hb + g) * a.n_split * stride_part + 4 + d;
    const float* wg = sm.cw + g * kMaxSplitS;
    float o = 0.0f;
    for (int s0 = 0; s0 < n_active; s0 += kLd) {
      float r[kLd];
#pragma unroll
      for (int u = 0; u < kLd; ++u) r[u] = s0 + u < n_active ? __ldcg(pg + (size_t)(s0 + u) * stride_part) : 0.0f;
#pragma unroll
      for (int u = 0; u < kLd; ++u)
        if (s0 + u < n_active) o = __fmaf_rn(wg[s0 + u], r[u], o);
    }
    o = __fmul_rn(o, sm.cinv[g]);
    a.out[(size_t)(hb + g) * hd + d] = o;
    sm.q[i] = o;
  }
  if (a.out_q8 && (hd % 32) == 0) {
    cbar(nthr);
    for (int b = warp; b < pairs / 32; b += NC) {
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

template <typename T>
__device__ void attn_stage(const AttnArgs& a, uint8_t* base, int NC, int warp, int lane, unsigned* ticket_s) {
  const AttnStageSmem sm = carve_stage(reinterpret_cast<float*>(base), a.head_dim);
  const int pos = a.pos_ptr ? *a.pos_ptr : a.pos_static;
  const int n_pos = pos + 1;
  int chunk = (n_pos + a.n_split - 1) / a.n_split;
  if (chunk < kSub) chunk = kSub;
  const int n_active = (n_pos + chunk - 1) / chunk;
  const int items = a.n_kv * n_active;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    attn_item<T>(a, sm, item % a.n_kv, item / a.n_kv, n_active, chunk, pos, NC, warp, lane, ticket_s);
    cbar(NC * 32);  // the next item reuses the shared memory
  }
}

// ---------------------------------------------------------------------
// the step kernel
// ---------------------------------------------------------------------
template <int kClass, typename T>
__global__ void __launch_bounds__((kStepMaxConsumers + 1) * 32, 1) k_decode_step(const StepPlan p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int abort_s;
  __shared__ unsigned ticket_s;
  // the consumers read their stage's descriptor from shared memory; the next
  // stage's is copied in (cp.async.bulk) while this one runs
  __shared__ StageDesc sdesc[2];
  __shared__ __align__(8) uint64_t dbar[2];
  // index of the last stage whose activations are in shared memory: the
  // producer holds back all but p.preissue of a stage's copies per warp until
  // then, so the prologue's loads do not queue behind a ring's worth of
  // weight copies
  __shared__ int open_s;
  const int NC = p.nc, S = p.S, slot = p.slot;
  uint8_t* ubase = smem;
  uint8_t* ring = smem + p.x_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)NC * S * slot);
  uint64_t* empty = full + NC * S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, b = blockIdx.x;

  if (threadIdx.x == 0) {
    abort_s = 0;
    open_s = -1;
    for (int i = 0; i < NC * S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&dbar[0], 1);
    mbar_init(&dbar[1], 1);
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == NC) {
    // ---- producer: lane w feeds consumer warp w's ring for the whole step
    const int w = lane;
    if (w >= NC) return;
    const uint64_t policy = l2_evict_first_policy();
    int n = 0;
    bool ok = true;
    for (int si = 0; si < p.n_stages && ok; ++si) {
      const StageDesc& sd = p.stages[si];
      if (sd.kind != kStageGemv) continue;
      const GemvArgs& g = sd.g;
      const int T_ = g.total_wr;
      const int wr0 = (int)((long long)b * T_ / G), wr1 = (int)((long long)(b + 1) * T_ / G);
      const int nwr = wr1 - wr0;
      const bool swiglu = g.seg[0].epi == kEpiSwiglu;
      const int ks = g.seg[0].ks;
      const int items = nwr > w ? (nwr - w + NC - 1) / NC : 0;
      int j = 0;  // copies of this stage issued by this lane
      for (int it = 0; it < items && ok; ++it) {
        const int wr = wr0 + w + NC * it;
        const GemvSeg& s = seg_of(g, wr);
        const size_t base = (size_t)(wr - s.wr_begin) * s.wr_bytes;
        for (int part = 0; part < (swiglu ? 2 : 1) && ok; ++part) {
          const uint8_t* wsrc = (part ? s.w2 : s.w) + base;
          for (int k = 0; k < ks; ++k, ++j) {
            if (j == p.preissue && g.input != kInQ8_1) {
              // bounded wait for the consumers' prologue of this stage
              const volatile int* op = &open_s;
              unsigned it2 = 0;
              while (*op < si && !abort_s && ++it2 < (1u << 24)) __nanosleep(64);
              if (*op < si) {
                ok = false;
                break;
              }
            }
            const int sidx = n % S;
            if (n >= S &&
                !mbar_wait_abort(&empty[w * S + sidx], (uint32_t)((n / S) - 1) & 1u, p.err, &abort_s)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[w * S + sidx], (uint32_t)s.step_bytes);
            bulk_load_hint(ring + (size_t)(w * S + sidx) * slot, wsrc + (size_t)k * s.step_bytes,
                           (uint32_t)s.step_bytes, &full[w * S + sidx], policy);
            ++n;
          }
        }
      }
    }
    if (!ok) atomicExch(p.abort, 1);
    // leave only once every copy issued into shared memory has landed
    for (int m = n - S > 0 ? n - S : 0; m < n; ++m) mbar_wait(&full[w * S + m % S], (uint32_t)(m / S) & 1u, p.err);
    return;
  }

  // ---- consumers
  const int nthr = NC * 32;
  int n = 0;
  int issued = -1, waited = -1;  // last stage whose descriptor copy was issued / awaited
  auto issue_desc = [&](int si) {
    mbar_arrive_expect_tx(&dbar[si & 1], (uint32_t)sizeof(StageDesc));
    bulk_load(&sdesc[si & 1], p.stages + si, (uint32_t)sizeof(StageDesc), &dbar[si & 1]);
    issued = si;
  };
  if (threadIdx.x == 0 && p.n_stages > 0) issue_desc(0);
  for (int si = 0; si < p.n_stages; ++si) {
    if (si > 0) {
      if (p.trace) {
        cbar(nthr);
        if (threadIdx.x == 0) p.trace[((size_t)(si - 1) * G + b) * 3 + 2] = globaltimer_ns();
      }
      if (!grid_sync(p, (unsigned)(si * G), nthr, &abort_s)) break;
    }
    if (p.trace && threadIdx.x == 0) p.trace[((size_t)si * G + b) * 3] = globaltimer_ns();
    if (!mbar_wait_abort(&dbar[si & 1], (uint32_t)(si >> 1) & 1u, p.err, &abort_s)) {
      raise_abort(p, &abort_s, !abort_s);
      break;
    }
    waited = si;
    // every consumer has left stage si-1 (the grid barrier's CTA barrier), so
    // its descriptor buffer is free for stage si+1
    if (threadIdx.x == 0 && si + 1 < p.n_stages) issue_desc(si + 1);
    const StageDesc& sd = sdesc[si & 1];
    if (sd.kind == kStageGemv) {
      const GemvArgs& g = sd.g;
      gemv_build_x<false>(g, ubase, NC, warp, lane);
      cbar(nthr);
      if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(&open_s) = si;
      if (p.trace && threadIdx.x == 0) p.trace[((size_t)si * G + b) * 3 + 1] = globaltimer_ns();
      const XShared x = gemv_x_view(ubase, g.cols);
      const int T_ = g.total_wr;
      const int wr0 = (int)((long long)b * T_ / G), wr1 = (int)((long long)(b + 1) * T_ / G);
      if (!gemv_items<kClass, false>(g, x, ring, full, empty, S, slot, wr0, wr1 - wr0, NC, warp, lane, n, &abort_s))
        raise_abort(p, &abort_s, false);
    } else {
      attn_stage<T>(sd.at, ubase, NC, warp, lane, &ticket_s);
    }
  }
  if (p.trace && p.n_stages > 0 && !abort_s) {
    cbar(nthr);
    if (threadIdx.x == 0) p.trace[((size_t)(p.n_stages - 1) * G + b) * 3 + 2] = globaltimer_ns();
  }
  // a descriptor copy still in flight (after an abort) must land before exit
  if (threadIdx.x == 0 && issued > waited) mbar_wait(&dbar[issued & 1], (uint32_t)(issued >> 1) & 1u, p.err);
}

template <int kClass, typename T>
cudaError_t set_attr() {
  return cudaFuncSetAttribute(k_decode_step<kClass, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax - 2048);
}

template <int kClass, typename T>
cudaError_t launch_t(const StepPlan& p, int grid, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((p.nc + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_decode_step<kClass, T>, p);
}

}  // namespace

size_t step_attn_bytes(int hd) { return (attn_stage_floats(hd) * 4 + 127) / 128 * 128; }

int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : fallback;
}

bool step_layout(int slot, size_t x_bytes, int* nc, int* S, size_t* smem) {
  // tuning overrides: MCPO_STEP_CONSUMERS, MCPO_STEP_STAGES
  const int want_nc = env_int("MCPO_STEP_CONSUMERS", kStepMaxConsumers);
  const int want_s = env_int("MCPO_STEP_STAGES", 0);
  // static shared memory (stage descriptors, flags) ~1 KB is reserved
  if ((size_t)kSmemMax - 2048 < x_bytes) return false;
  const size_t budget = (size_t)kSmemMax - 2048 - x_bytes;
  for (int s = want_s > 0 ? want_s : 2; s >= 1; --s) {
    const size_t per_warp = (size_t)s * ((size_t)slot + 16);
    int n = (int)(budget / per_warp);
    if (n > kStepMaxConsumers) n = kStepMaxConsumers;
    if (n > want_nc) n = want_nc;
    if (n >= kMinConsumers) {
      *nc = n;
      *S = s;
      *smem = x_bytes + (size_t)n * s * slot + (size_t)2 * n * s * 8;
      return true;
    }
  }
  return false;
}

cudaError_t decode_step_init() {
  const cudaError_t r[] = {set_attr<kClassQ4K6K, float>(), set_attr<kClassQ4K6K, __half>(),
                           set_attr<kClassQ80, float>(), set_attr<kClassQ80, __half>()};
  for (cudaError_t e : r)
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

cudaError_t launch_decode_step(const StepPlan& p, int grid, size_t smem, bool q80, bool kv_f16, cudaStream_t st) {
  if (p.nc < kMinConsumers || p.nc > kStepMaxConsumers || p.S < 1 || grid < 1) return cudaErrorInvalidValue;
  if (q80) return kv_f16 ? launch_t<kClassQ80, __half>(p, grid, smem, st) : launch_t<kClassQ80, float>(p, grid, smem, st);
  return kv_f16 ? launch_t<kClassQ4K6K, __half>(p, grid, smem, st) : launch_t<kClassQ4K6K, float>(p, grid, smem, st);
}

}  // namespace mcpo
