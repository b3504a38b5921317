// pgemm.cu -- prompt-prefill projections on the tensor cores (see pgemm.cuh).
//
// One CTA per (128-row tile, 32-token tile), 18 warps:
//   warp 0      producer: per super-block, bulk copies of its A, S, B (Bm for
//               Q6_K) and X tiles into a shared-memory ring (3 stages, 2
//               for Q6_K);
//   warp 1      one thread issues the MMAs: per unit (a super-block, half of
//               one for Q6_K) eight tcgen05.mma kind::i8 (M 128, N 32, K 32),
//               one per 32-value block (Q6_K: per 16-value group, through
//               the masked B), each into its own 32-column s32 region of
//               tensor memory; two buffers of eight regions, so the MMAs of
//               one unit run while the epilogue reads the previous one;
//   warps 2-17  epilogue: warp w reads rows 32*(w%4) .. +31 (the tensor-
//               memory lane quarter it may access) for tokens
//               8*((w-2)/4) .. +7 and combines the dots as the decode GEMV
//               does (gemv_dev.cuh sb_dot_q4k / sb_dot_q6k / sb_dot_q80,
//               gemv_items, reduce_row).
// Super-blocks are visited in the order of the decode's reduction tree: the
// GEMV's lanes i of a row (lane_in_row, lpr of them) in bit-reversed order,
// each lane's super-blocks k*lpr + i in k order.  A lane's sequential sum
// over k is pushed onto a binary-counter stack; its merges add the earlier
// partial and the later one, which is the butterfly's xor tree as the row's
// first lane computes it.
//
// Every wait is bounded; a wait that gives up raises the error word and the
// CTA's abort flag, the other roles leave at their next wait, and the CTA
// waits (bounded) for its copies and MMAs in flight before it frees tensor
// memory.
#include "pgemm.cuh"

#include <cuda_fp16.h>
#include <stdlib.h>

#include "common.cuh"
#include "gemv.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr int kPgEpiWarps = 16;
constexpr int kPgThreads = (2 + kPgEpiWarps) * 32;
constexpr uint32_t kPgTmemCols = 512;  // two buffers x eight 32-column regions
constexpr int kPgLevels = 6;           // reduction-tree levels for lpr <= 32
constexpr int kPgMaxSplit = 16;        // CTAs per row tile at most (the roots fit a tree-stack column)
// Tree levels 1 .. kPgLevels-1 live in shared memory ([level][token][thread]
// floats, each thread its own column); level 0 and the lane sums in
// registers.
constexpr size_t kPgStackBytes = (size_t)(kPgLevels - 1) * 8 * kPgEpiWarps * 32 * 4;

// Ring stages and their operand bytes (Q6_K: two masked B halves, so one
// stage fewer fits).
template <int kDtype>
struct PgSmem {
  static constexpr int kStages = kDtype == kQ6_K ? 2 : 3;
  static constexpr int kBStage = kDtype == kQ6_K ? 2 * kPgBBytes : kPgBBytes;
  __host__ __device__ static constexpr size_t a(int s) { return (size_t)s * kPgABytes; }
  __host__ __device__ static constexpr size_t b(int s) { return (size_t)kStages * kPgABytes + (size_t)s * kBStage; }
  __host__ __device__ static constexpr size_t sc(int s) { return b(kStages) + (size_t)s * kPgSBytes; }
  __host__ __device__ static constexpr size_t x(int s) { return sc(kStages) + (size_t)s * kPgXFloats * 4; }
  __host__ __device__ static constexpr size_t stack() { return x(kStages); }
  __host__ __device__ static constexpr size_t bars() { return stack() + kPgStackBytes; }
  __host__ __device__ static constexpr size_t bytes() { return bars() + 8 * (2 * kStages + 4 + 1) + 16 + 1024; }
};

struct PgArgs {
  const uint8_t* a;
  const uint8_t* s;
  const uint8_t* b;  // B, or Bm for Q6_K
  const float* xs;
  int nb, lpr, ks, levels;
  int tiles, rows, T;
  int epi;
  float* y;
  int ldy;
  const float* gate;
  int ldg;
  int* err;
  // split over the GEMV lanes (ksplit > 1): CTA z takes the lanes' subtree
  // z of the reduction tree and writes its root to part; the last CTA of a
  // (row tile, token tile) adds the roots in tree order (cnt: arrivals,
  // zero at rest)
  int ksplit, lsplit;
  float* part;
  unsigned* cnt;
};

// Instruction descriptor of kind::i8: s8 A and B (K-major), s32
// accumulator, M = 128, N = 32.
constexpr uint32_t kPgIdesc =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPgTok >> 3) << 17) | ((uint32_t)(kPgRows >> 4) << 24);

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// Eight consecutive s32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld8_s32(uint32_t taddr, int (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = (int)r[i];
}

// The super-block visited at position it: lane i = bitrev(it / ks) of
// `levels` bits, then k = it % ks.
__device__ __forceinline__ int pg_sb_at(int it, int ks, int levels) {
  const int li = it / ks, k = it - li * ks;
  const int i = levels ? (int)(__brev((unsigned)li) >> (32 - levels)) : 0;
  return k * (1 << levels) + i;
}

// A lane sum lands on level kTop of the tree stack: the partials of the
// levels below (earlier leaves) are added in front of it, level by level.
// lvl0: level 0 in registers; sst: this thread's column of levels 1.. in
// shared memory (stride kPgEpiWarps * 32 floats per (level, token)).
template <int kTop>
__device__ __forceinline__ void pg_push(float (&lvl0)[8], float* sst, const float (&acc)[8]) {
  constexpr int kStride = kPgEpiWarps * 32;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float c = acc[e];
    if constexpr (kTop == 0) {
      lvl0[e] = c;
    } else {
      c = __fadd_rn(lvl0[e], c);
#pragma unroll
      for (int l = 1; l < kTop; ++l) c = __fadd_rn(sst[((l - 1) * 8 + e) * kStride], c);
      sst[((kTop - 1) * 8 + e) * kStride] = c;
    }
  }
}

template <int kDtype>
__global__ void __launch_bounds__(kPgThreads, 1) k_pgemm(const PgArgs p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  using L = PgSmem<kDtype>;
  constexpr int kPgStages = L::kStages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bars());
  uint64_t* empty = full + kPgStages;
  uint64_t* acc_full = empty + kPgStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_s = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_s + 1);

  constexpr bool kQ6 = kDtype == kQ6_K;
  constexpr int kUnits = kQ6 ? 2 : 1;  // MMA units per super-block
  constexpr int kBBytes = kQ6 ? 2 * kPgBBytes : kPgBBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, ttile = blockIdx.y, z = blockIdx.z;
  const int nsb = p.nb;
  const int n_it = nsb >> p.lsplit, it0 = z * n_it, it1 = it0 + n_it;  // this CTA's super-blocks

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPgStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + kPgEpiWarps);  // the MMAs' commit and every epilogue warp
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kPgEpiWarps);
    }
    mbar_init(done, 1);
    *abort_s = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_s, kPgTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_s;

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      pdl_wait();  // the activation operands come from the previous kernel
      const uint64_t policy = l2_evict_first_policy();
      const uint32_t tx = (uint32_t)(kPgABytes + kPgSBytes + kBBytes + kPgXFloats * 4);
      int issued = 0;
      for (int j = 0; j < n_it; ++j) {
        const int sb = pg_sb_at(it0 + j, p.ks, p.levels);
        const int s = j % kPgStages;
        if (j >= kPgStages && !gwait(&empty[s], (uint32_t)((j / kPgStages) - 1) & 1u, p.err, abort_s)) break;
        const size_t wt = (size_t)tile * nsb + sb, xt = (size_t)ttile * nsb + sb;
        mbar_arrive_expect_tx(&full[s], tx);
        bulk_load_hint(smem + L::a(s), p.a + wt * kPgABytes, kPgABytes, &full[s], policy);
        bulk_load(smem + L::sc(s), p.s + wt * kPgSBytes, kPgSBytes, &full[s]);
        bulk_load(smem + L::b(s), p.b + xt * kBBytes, kBBytes, &full[s]);
        bulk_load(smem + L::x(s), p.xs + xt * kPgXFloats, kPgXFloats * 4, &full[s]);
        issued = j + 1;
      }
      for (int j = issued > kPgStages ? issued - kPgStages : 0; j < issued; ++j)
        if (!mbar_wait(&full[j % kPgStages], (uint32_t)(j / kPgStages) & 1u, p.err)) break;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int u = 0;
      bool ok = true;
      for (int j = 0; j < n_it && ok; ++j) {
        const int s = j % kPgStages;
        if (!gwait(&full[s], (uint32_t)(j / kPgStages) & 1u, p.err, abort_s)) break;
        tc_fence_after();
        const uint32_t a0 = smem_addr(smem + L::a(s)), b0 = smem_addr(smem + L::b(s));
        for (int h = 0; h < kUnits; ++h, ++u) {
          const int buf = u & 1;
          if (u >= 2 && !gwait(&acc_empty[buf], (uint32_t)((u >> 1) - 1) & 1u, p.err, abort_s)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            // A: block blk's two 16-value chunks (core matrices 2048 B apart,
            // row groups 128 B apart); B: the same chunks of the 32 tokens
            // (512 B apart), Q6_K: the half that keeps group 2*blk + (r & 1)
            const int blk = kQ6 ? 4 * h + (r >> 1) : r;
            const uint32_t boff = (uint32_t)((kQ6 ? (r & 1) * kPgBBytes : 0) + blk * 1024);
            umma_i8(tmem + (uint32_t)((buf * 8 + r) * 32), umma_desc(a0 + (uint32_t)blk * 4096u, 2048, 128),
                    umma_desc(b0 + boff, 512, 128), kPgIdesc);
          }
          umma_commit(&acc_full[buf]);
        }
        if (ok) umma_commit(&empty[s]);
      }
      // every MMA issued has completed before tensor memory is freed
      umma_commit(done);
      mbar_wait(done, 0u, p.err);
    }
    __syncwarp();
  } else {
    // ---- epilogue ----
    // a warp reaches only tensor-memory lanes 32*(warp % 4) .. +31
    const int qtr = warp & 3, tg = (warp - 2) >> 2;
    const int rl = qtr * 32 + lane;
    const uint32_t tbase = tmem + ((uint32_t)(qtr * 32) << 16) + (uint32_t)(tg * 8);
    float lvl0[8], acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = lvl0[e] = 0.0f;
    float* sst = reinterpret_cast<float*>(smem + L::stack()) + (threadIdx.x - 64);
    int cnt = 0, u = 0;
    bool go = true;
    for (int it = it0; it < it1; ++it) {
      const int s = (it - it0) % kPgStages;
      if (!__all_sync(0xffffffffu, gwait(&full[s], (uint32_t)((it - it0) / kPgStages) & 1u, p.err, abort_s))) {
        go = false;
        break;
      }
      const uint4* srow = reinterpret_cast<const uint4*>(smem + L::sc(s) + (size_t)rl * 32);
      const float* X = reinterpret_cast<const float*>(smem + L::x(s)) + tg * 8;  // xd [j*32], xds [256 + j*32]
      float v[8];
      if constexpr (kDtype == kQ4_K) {
        const uint4 h = srow[0];
        const float d = f16_to_f32((uint16_t)(h.x & 0xffffu));
        const float dmin = f16_to_f32((uint16_t)(h.x >> 16));
        const uint32_t sc_lo = h.y & 0x3f3f3f3fu, mn_lo = h.z & 0x3f3f3f3fu;
        const uint32_t sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
        const uint32_t mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
        const int buf = u & 1;
        if (!__all_sync(0xffffffffu, gwait(&acc_full[buf], (uint32_t)(u >> 1) & 1u, p.err, abort_s))) {
          go = false;
          break;
        }
        tc_fence_after();
        float sd[8], sm[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) sd[e] = sm[e] = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int dt[8];
          tmem_ld8_s32(tbase + (uint32_t)((buf * 8 + j) * 32), dt);
          const uint32_t scw = j < 4 ? sc_lo : sc_hi, mnw = j < 4 ? mn_lo : mn_hi;
          const int sj = (int)((scw >> (8 * (j & 3))) & 0xffu), mj = (int)((mnw >> (8 * (j & 3))) & 0xffu);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            sd[e] = __fmaf_rn(X[j * 32 + e], (float)(sj * dt[e]), sd[e]);
            sm[e] = __fmaf_rn(X[256 + j * 32 + e], (float)mj, sm[e]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        ++u;
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fmaf_rn(d, sd[e], -__fmul_rn(dmin, sm[e]));
      } else if constexpr (kDtype == kQ8_0) {
        const uint4 h = srow[0];
        const uint32_t dw[4] = {h.x, h.y, h.z, h.w};
        const int buf = u & 1;
        if (!__all_sync(0xffffffffu, gwait(&acc_full[buf], (uint32_t)(u >> 1) & 1u, p.err, abort_s))) {
          go = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.0f;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          int dt[8];
          tmem_ld8_s32(tbase + (uint32_t)((buf * 8 + b) * 32), dt);
          const float dwf = f16_to_f32((uint16_t)((dw[b >> 1] >> (16 * (b & 1))) & 0xffffu));
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = __fmaf_rn(__fmul_rn(dwf, X[b * 32 + e]), (float)dt[e], v[e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        ++u;
      } else {
        const uint4 scv = srow[0];
        const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
        const float d = f16_to_f32((uint16_t)(srow[1].x & 0xffffu));
        float sum[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) sum[e] = 0.0f;
        bool ok = true;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int buf = u & 1;
          if (!__all_sync(0xffffffffu, gwait(&acc_full[buf], (uint32_t)(u >> 1) & 1u, p.err, abort_s))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int b = 4 * h + qq, g0 = 2 * b;
            int dg0[8], dg1[8];
            tmem_ld8_s32(tbase + (uint32_t)((buf * 8 + 2 * qq) * 32), dg0);
            tmem_ld8_s32(tbase + (uint32_t)((buf * 8 + 2 * qq + 1) * 32), dg1);
            const int sc0 = (int)(int8_t)((scw[g0 >> 2] >> (8 * (g0 & 3))) & 0xffu);
            const int sc1 = (int)(int8_t)((scw[(g0 + 1) >> 2] >> (8 * ((g0 + 1) & 3))) & 0xffu);
#pragma unroll
            for (int e = 0; e < 8; ++e) sum[e] = __fmaf_rn(X[b * 32 + e], (float)(sc0 * dg0[e] + sc1 * dg1[e]), sum[e]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
          ++u;
        }
        if (!ok) {
          go = false;
          break;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(d, sum[e]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      // the GEMV lane's sum over its steps (acc starts at 0 there too), then
      // the row's butterfly as a binary-counter stack
      const int k = it % p.ks;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(k == 0 ? 0.0f : acc[e], v[e]);
      if (k == p.ks - 1) {
        // the level the merged value lands on (the same for every thread:
        // one branch, then straight-line code on fixed registers)
        switch (__ffs(~cnt) - 1) {
          case 0: pg_push<0>(lvl0, sst, acc); break;
          case 1: pg_push<1>(lvl0, sst, acc); break;
          case 2: pg_push<2>(lvl0, sst, acc); break;
          case 3: pg_push<3>(lvl0, sst, acc); break;
          case 4: pg_push<4>(lvl0, sst, acc); break;
          default: pg_push<5>(lvl0, sst, acc); break;
        }
        ++cnt;
      }
    }
    const int top = p.levels - p.lsplit;  // the level of this CTA's subtree root
    float val[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) val[e] = top == 0 ? lvl0[e] : sst[((top - 1) * 8 + e) * (kPgEpiWarps * 32)];
    bool store = go && !*abort_s;
    if (p.ksplit > 1) {
      // roots of the subtrees: [z][tile][ttile][token][row]; every CTA
      // arrives (also after an abort, so the count returns to zero)
      __shared__ unsigned ticket_s;
      const size_t tt_idx = (size_t)tile * gridDim.y + ttile, ntt = (size_t)gridDim.x * gridDim.y;
      float* mine = p.part + (((size_t)z * ntt + tt_idx) * kPgTok + tg * 8) * kPgRows + rl;
#pragma unroll
      for (int e = 0; e < 8; ++e) mine[(size_t)e * kPgRows] = val[e];
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kPgEpiWarps * 32) : "memory");
      if (threadIdx.x == 64) ticket_s = atomicAdd(p.cnt + tt_idx, 1u);
      asm volatile("bar.sync 1, %0;" ::"n"(kPgEpiWarps * 32) : "memory");
      const bool last = ticket_s == (unsigned)(p.ksplit - 1);
      if (last) {
        __threadfence();
        if (threadIdx.x == 64) p.cnt[tt_idx] = 0u;
        // the upper levels of the butterfly: adjacent roots pairwise, the
        // earlier one in front (in this thread's column of the tree stack,
        // which the loop above no longer needs)
        constexpr int kStride = kPgEpiWarps * 32;
        for (int e = 0; e < 8; ++e) {
          for (int q = 0; q < p.ksplit; ++q)
            sst[q * kStride] = __ldcg(p.part + (((size_t)q * ntt + tt_idx) * kPgTok + tg * 8 + e) * kPgRows + rl);
          for (int w = 1; w < p.ksplit; w <<= 1)
            for (int q = 0; q + w < p.ksplit; q += 2 * w) sst[q * kStride] = __fadd_rn(sst[q * kStride], sst[(q + w) * kStride]);
          val[e] = sst[0];
        }
      }
      store = store && last;
    }
    if (store) {
      pdl_wait();  // y and gate come from earlier kernels
      const int row = tile * kPgRows + rl;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int t = ttile * kPgTok + tg * 8 + e;
        if (t < p.T && row < p.rows) {
          float* yp = p.y + (size_t)t * p.ldy + row;
          if (p.epi == kPgStore)
            *yp = val[e];
          else if (p.epi == kPgAdd)
            *yp = __fadd_rn(*yp, val[e]);
          else
            *yp = silu_mul_det(p.gate[(size_t)t * p.ldg + row], val[e]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPgTmemCols);
  }
}

// One CTA per (row tile, super-block), one thread per row: the row's
// super-block from the tiled GEMV copy (layout.cuh) as 256 int8 values in
// natural order plus its scales; rows past the matrix are zeros.
__global__ void __launch_bounds__(kPgRows) k_pgemm_relayout(const uint8_t* src, TileGeom g, uint8_t* A, uint8_t* S) {
  const int tile = blockIdx.x, sb = blockIdx.y, t = threadIdx.x;
  const int row = tile * kPgRows + t;
  const bool valid = row < g.rows;
  uint4 ch[17];
  uint16_t d6 = 0;
#pragma unroll
  for (int c = 0; c < 17; ++c) ch[c] = make_uint4(0, 0, 0, 0);
  if (valid) {
    const int wr = row / g.rpw, ri = row % g.rpw, k = sb / g.lpr, li = sb % g.lpr, ln = ri * g.lpr + li;
    const uint8_t* blk = src + (size_t)wr * g.wr_bytes + (size_t)k * g.step_bytes;
    for (int c = 0; c < g.chunks; ++c) ch[c] = *reinterpret_cast<const uint4*>(blk + (size_t)c * 512 + ln * 16);
    if (g.dtype == kQ6_K) d6 = *reinterpret_cast<const uint16_t*>(blk + (size_t)g.chunks * 512 + ln * 2);
  }
  const uint8_t* cb = reinterpret_cast<const uint8_t*>(ch);
  uint8_t* at = A + ((size_t)tile * g.nb + sb) * kPgABytes;
  for (int c = 0; c < 16; ++c) {
    uint32_t wv[4];
    for (int q = 0; q < 4; ++q) {
      uint32_t word = 0;
      for (int e = 0; e < 4; ++e) {
        const int v = c * 16 + q * 4 + e;
        int val = 0;
        if (valid) {
          if (g.dtype == kQ4_K) {
            const int grp = v >> 6, within = v & 63, l = within & 31;
            const int byte = cb[16 + 32 * grp + l];
            val = within >= 32 ? byte >> 4 : byte & 15;
          } else if (g.dtype == kQ6_K) {
            const int n = v >> 7, w = v & 127, qtr = w >> 5, l = w & 31;
            const int qlb = cb[64 * n + l + (qtr & 1) * 32], qhb = cb[128 + 32 * n + l];
            const int lo = qtr < 2 ? (qlb & 15) : (qlb >> 4), hi = (qhb >> (2 * qtr)) & 3;
            val = (lo | (hi << 4)) - 32;
          } else {
            val = (int)(int8_t)cb[16 + v];
          }
        }
        word |= (uint32_t)(val & 0xff) << (8 * e);
      }
      wv[q] = word;
    }
    *reinterpret_cast<uint4*>(at + ((size_t)c * 16 + (t >> 3)) * 128 + (t & 7) * 16) =
        make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
  uint4 s0 = make_uint4(0, 0, 0, 0), s1 = make_uint4(0, 0, 0, 0);
  if (valid) {
    if (g.dtype == kQ6_K) {
      s0 = ch[12];
      s1.x = d6;
    } else {
      s0 = ch[0];
    }
  }
  uint4* st = reinterpret_cast<uint4*>(S + ((size_t)tile * g.nb + sb) * kPgSBytes + (size_t)t * 32);
  st[0] = s0;
  st[1] = s1;
}

// One CTA per token slot of the padded token tiles and 64 blocks of 32
// values: RMSNorm (optional; every CTA of a token computes the row's scale)
// and Q8_1 quantisation in the decode GEMV's arithmetic (gemv_build_x: 256
// strided partial sums, halving and warp trees, exact 1/sqrt; per block the
// reference's variant-B quantiser), written as the B, Bm and X operands.
// Slots past T are zeros.
constexpr int kPgActBlocks = 64;

__global__ void __launch_bounds__(256) k_pgemm_act(const float* x, int ldx, int T, int K, const void* nw, int ndt,
                                                   float eps, uint8_t* B, uint8_t* Bm, float* XS) {
  __shared__ float red[256];
  __shared__ float inv_s;
  pdl_wait();
  const int n = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nb = K / 256, tt = n / kPgTok, nn = n % kPgTok;
  const int b0 = blockIdx.y * kPgActBlocks;  // this CTA's 32-value blocks
  const bool valid = n < T;
  const float* xr = x + (size_t)(valid ? n : 0) * ldx;
  float inv = 1.0f;
  if (nw && valid) {
    float pr = 0.0f;
    for (int k = 0; k < nb; ++k) {
      const float r = xr[t + 256 * k];
      pr = __fadd_rn(pr, __fmul_rn(r, r));
    }
    red[t] = pr;
    __syncthreads();
    if (warp == 0) {
      float q[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = red[lane + 32 * k];
      float r = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[4]), __fadd_rn(q[2], q[6])),
                          __fadd_rn(__fadd_rn(q[1], q[5]), __fadd_rn(q[3], q[7])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) r = __fadd_rn(r, __shfl_down_sync(0xffffffffu, r, o));
      if (lane == 0) inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(r, (float)K), eps)));
    }
    __syncthreads();
    inv = inv_s;
  }
  const int nblk = min(K / 32, b0 + kPgActBlocks);
  for (int bi = b0 + warp; bi < nblk; bi += 8) {
    int q = 0;
    uint16_t dbits = 0;
    if (valid) {
      float v = xr[bi * 32 + lane];
      if (nw) v = __fmul_rn(__fmul_rn(v, inv), load_weight(nw, ndt, bi * 32 + lane));
      bool zero;
      q = q8_1_quant_lane(v, &dbits, &zero);
    }
    const int sum = __reduce_add_sync(0xffffffffu, q);
    uint32_t word = (uint32_t)(q & 0xff) << (8 * (lane & 3));
    word |= __shfl_xor_sync(0xffffffffu, word, 1);
    word |= __shfl_xor_sync(0xffffffffu, word, 2);
    const int sb = bi >> 3, j = bi & 7, c = 2 * j + (lane >> 4);
    const size_t xt = (size_t)tt * nb + sb;
    const size_t off = ((size_t)c * 4 + (nn >> 3)) * 128 + (size_t)(nn & 7) * 16 + (size_t)((lane & 15) & ~3);
    if ((lane & 3) == 0) {
      *reinterpret_cast<uint32_t*>(B + xt * kPgBBytes + off) = word;
      uint8_t* bm = Bm + xt * 2 * kPgBBytes;
      *reinterpret_cast<uint32_t*>(bm + off) = lane < 16 ? word : 0u;
      *reinterpret_cast<uint32_t*>(bm + kPgBBytes + off) = lane < 16 ? 0u : word;
    }
    if (lane == 0) {
      const float d8 = f16_to_f32(dbits);
      XS[xt * kPgXFloats + j * 32 + nn] = d8;
      XS[xt * kPgXFloats + 256 + j * 32 + nn] = __fmul_rn(d8, (float)sum);
    }
  }
  pdl_launch_dependents();
}

template <int kDtype>
cudaError_t set_pgemm_attr() {
  static_assert(PgSmem<kDtype>::bytes() <= 232448, "shared memory per CTA");
  return cudaFuncSetAttribute(k_pgemm<kDtype>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)PgSmem<kDtype>::bytes());
}

}  // namespace

cudaError_t pgemm_init() {
  const cudaError_t r[] = {set_pgemm_attr<kQ4_K>(), set_pgemm_attr<kQ6_K>(), set_pgemm_attr<kQ8_0>()};
  for (cudaError_t e : r)
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

size_t pgemm_mat_bytes(const TileGeom& g) {
  const size_t tiles = ((size_t)g.rows + kPgRows - 1) / kPgRows;
  return tiles * (size_t)g.nb * (kPgABytes + kPgSBytes);
}

cudaError_t pgemm_build(const TileGeom& g, const uint8_t* tiled, PgemmMat* out, cudaStream_t st) {
  if (!tiled || !out || !is_quant(g.dtype) || g.nb < 1 || g.lpr < 1 || g.lpr > 32 || (g.lpr & (g.lpr - 1)) ||
      g.lpr * g.ks != g.nb)
    return cudaErrorInvalidValue;
  PgemmMat m;
  m.dtype = g.dtype;
  m.rows = g.rows;
  m.cols = g.cols;
  m.nb = g.nb;
  m.tiles = (g.rows + kPgRows - 1) / kPgRows;
  m.lpr = g.lpr;
  m.ks = g.ks;
  cudaError_t e = cudaMalloc((void**)&m.a, (size_t)m.tiles * m.nb * kPgABytes);
  if (e == cudaSuccess) e = cudaMalloc((void**)&m.s, (size_t)m.tiles * m.nb * kPgSBytes);
  if (e == cudaSuccess) e = launch_k(k_pgemm_relayout, dim3(m.tiles, m.nb), dim3(kPgRows), 0, st, false, tiled, g, m.a, m.s);
  if (e != cudaSuccess) {
    pgemm_free(&m);
    return e;
  }
  *out = m;
  return cudaSuccess;
}

void pgemm_free(PgemmMat* m) {
  if (!m) return;
  if (m->a) cudaFree(m->a);
  if (m->s) cudaFree(m->s);
  m->a = m->s = nullptr;
}

cudaError_t pgemm_act_alloc(int tmax, int K, PgemmAct* a) {
  if (!a || tmax < 1 || K < 256 || K % 256) return cudaErrorInvalidValue;
  const size_t tt = ((size_t)tmax + kPgTok - 1) / kPgTok, nb = (size_t)K / 256;
  PgemmAct x;
  x.tmax = (int)(tt * kPgTok);
  x.K = K;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  x.split_ctas = sms;
  if (e == cudaSuccess) e = cudaMalloc((void**)&x.b, tt * nb * kPgBBytes);
  if (e == cudaSuccess) e = cudaMalloc((void**)&x.bm, tt * nb * 2 * kPgBBytes);
  if (e == cudaSuccess) e = cudaMalloc((void**)&x.xs, tt * nb * kPgXFloats * 4);
  if (e == cudaSuccess) e = cudaMalloc((void**)&x.part, (size_t)sms * kPgTok * kPgRows * 4);
  if (e == cudaSuccess) e = cudaMalloc((void**)&x.cnt, (size_t)sms * 4);
  if (e == cudaSuccess) e = cudaMemset(x.cnt, 0, (size_t)sms * 4);
  if (e != cudaSuccess) {
    pgemm_act_free(&x);
    return e;
  }
  *a = x;
  return cudaSuccess;
}

void pgemm_act_free(PgemmAct* a) {
  if (!a) return;
  if (a->b) cudaFree(a->b);
  if (a->bm) cudaFree(a->bm);
  if (a->xs) cudaFree(a->xs);
  if (a->part) cudaFree(a->part);
  if (a->cnt) cudaFree(a->cnt);
  a->b = a->bm = nullptr;
  a->xs = a->part = nullptr;
  a->cnt = nullptr;
}

cudaError_t launch_pgemm_act(const float* x, int ldx, int T, const void* norm_w, int norm_dtype, float eps,
                             const PgemmAct& a, cudaStream_t st) {
  if (!x || T < 1 || T > a.tmax || !a.b || !a.bm || !a.xs || ldx < a.K) return cudaErrorInvalidValue;
  const int slots = (T + kPgTok - 1) / kPgTok * kPgTok;
  const int chunks = (a.K / 32 + kPgActBlocks - 1) / kPgActBlocks;
  return launch_k(k_pgemm_act, dim3(slots, chunks), dim3(256), 0, st, true, x, ldx, T, a.K, norm_w, norm_dtype, eps,
                  a.b, a.bm, a.xs);
}

namespace {
int pgemm_split_cfg() {
  static const int v = [] {
    const char* e = getenv("MCPO_PG_SPLIT");
    return (e && *e) ? (atoi(e) != 0 ? 1 : 0) : 1;
  }();
  return v;
}
}  // namespace

cudaError_t launch_pgemm(const PgemmMat& w, const PgemmAct& x, int T, int epi, float* y, int ldy, const float* gate,
                         int ldg, int* err, cudaStream_t st) {
  if (!w.a || !w.s || !x.b || !x.bm || !x.xs || T < 1 || T > x.tmax || x.K != w.cols || !y || ldy < w.rows ||
      epi < kPgStore || epi > kPgSwiglu || (epi == kPgSwiglu && (!gate || ldg < w.rows)) || w.lpr < 1 ||
      w.lpr > 32 || (w.lpr & (w.lpr - 1)) || w.lpr * w.ks != w.nb)
    return cudaErrorInvalidValue;
  PgArgs p{};
  p.a = w.a;
  p.s = w.s;
  p.b = w.dtype == kQ6_K ? x.bm : x.b;
  p.xs = x.xs;
  p.nb = w.nb;
  p.lpr = w.lpr;
  p.ks = w.ks;
  p.levels = __builtin_ctz((unsigned)w.lpr);
  p.tiles = w.tiles;
  p.rows = w.rows;
  p.T = T;
  p.epi = epi;
  p.y = y;
  p.ldy = ldy;
  p.gate = gate;
  p.ldg = ldg;
  p.err = err;
  // fewer CTAs than SMs: split each row tile over its lanes (bits do not
  // change: the subtrees' roots are added in the tree's order)
  const int ttiles = (T + kPgTok - 1) / kPgTok, ctas = w.tiles * ttiles;
  int ks = 1;
  while (pgemm_split_cfg() && x.part && ks * 2 <= w.lpr && ks * 2 <= kPgMaxSplit && ctas * ks * 2 <= x.split_ctas)
    ks *= 2;
  p.ksplit = ks;
  p.lsplit = __builtin_ctz((unsigned)ks);
  p.part = x.part;
  p.cnt = x.cnt;
  const dim3 grid(w.tiles, ttiles, ks);
  switch (w.dtype) {
    case kQ4_K: return launch_k(k_pgemm<kQ4_K>, grid, dim3(kPgThreads), PgSmem<kQ4_K>::bytes(), st, true, p);
    case kQ6_K: return launch_k(k_pgemm<kQ6_K>, grid, dim3(kPgThreads), PgSmem<kQ6_K>::bytes(), st, true, p);
    case kQ8_0: return launch_k(k_pgemm<kQ8_0>, grid, dim3(kPgThreads), PgSmem<kQ8_0>::bytes(), st, true, p);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mcpo
