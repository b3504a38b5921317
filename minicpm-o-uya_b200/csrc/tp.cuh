// tp.cuh -- tensor-parallel exchanges between the ranks of one node, over
// CUDA IPC mappings of each rank's exchange buffer (tagged 64-bit stores
// over NVLink, local loads; no multicast, no TMA on peer memory).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "misc.cuh"
#include "tp_proto.h"

namespace mcpo {

// One rank's exchange buffer (allocated by that rank, IPC-exported; every
// 64-bit word a value and its tag, tp_proto.h):
//   part[2][kTpMaxWorld][hidden]  partial hidden vectors of the
//                    row-parallel GEMVs (o, down), written by each source
//                    rank into its own slot, two parities;
//   top[4]           this rank's sampler result (f32 best, index, second;
//                    written by its own k_argmax);
//   merge[kTpMaxWorld][4]  every rank's sampler result, tagged with the
//                    sampler-merge epoch.
struct TpLayout {
  static size_t part_offset(int parity, int src, size_t hidden) {
    return ((size_t)parity * kTpMaxWorld + (size_t)src) * hidden * 8;
  }
  static size_t top_offset(size_t hidden) { return 2 * (size_t)kTpMaxWorld * hidden * 8; }
  static size_t merge_offset(size_t hidden) { return top_offset(hidden) + 16; }
  static size_t bytes(size_t hidden) { return (merge_offset(hidden) + (size_t)kTpMaxWorld * 4 * 8 + 255) / 256 * 256; }
};

// Device view of all ranks' buffers (own and peer-mapped).
struct TpPeers {
  uint8_t* base[kTpMaxWorld];
  float* top[kTpMaxWorld];
  uint64_t* merge[kTpMaxWorld];
  int rank, world;
};

// One exchange as a GEMV sees it (gemv.cuh: kEpiTpPush produces it,
// kInRmsNormTp consumes it).
struct TpXchg {
  // producer: output row r of this rank's partial goes, tagged, to
  // dst[d][r] on every rank d
  uint64_t* dst[kTpMaxWorld];
  // consumer: base[i] + (src[0][i] + ... + src[world-1][i]) once every
  // src[r][i] carries the exchange's tag; the sum also goes to sum_out
  // (each CTA its share)
  const uint64_t* src[kTpMaxWorld];
  float* sum_out;
  const unsigned* step;  // the step counter (advanced by k_tp_step at each step's start)
  int world;
  int nx;    // exchanges per step
  int x;     // this exchange's index within the step
  int rows;  // values per exchange (hidden)
};

__host__ __device__ inline uint32_t tp_xchg_tag(const TpXchg& t, uint32_t step) {
  return tp_tag(tp_exchange_index(step, (uint32_t)t.nx, (uint32_t)t.x));
}

// Single-copy-atomic 64-bit accesses of the tagged words, strong at system
// scope (the writer and the reader are on different GPUs).
__device__ __forceinline__ void tp_st_word(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t tp_ld_word(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t tp_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// For every element i = tid + j * nthr (i < n) of an exchange with `tag`:
// out(i, rank-order sum of the partials) (tp_rank_sum without the base).
// The (element, rank) words are requested 16 at a time, whole elements per
// batch (world, a power of two <= 8, divides 16), so a thread waits about
// one load latency per 16 words; a word without the tag is polled until it
// has it (bounded by `deadline`, clearing *ok).
template <typename Out>
__device__ __forceinline__ void tp_gather_sums(const TpXchg& t, uint32_t tag, int tid, int nthr, int n,
                                               uint64_t deadline, bool* ok, Out out) {
  const int lw = t.world >= 8 ? 3 : t.world >= 4 ? 2 : t.world >= 2 ? 1 : 0;
  const int wm = (1 << lw) - 1;
  const int total = (n > tid ? (n - tid + nthr - 1) / nthr : 0) << lw;
  for (int q0 = 0; q0 < total; q0 += 16) {
    uint64_t w[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int q = q0 + u;
      w[u] = q < total ? tp_ld_word(t.src[q & wm] + tid + (q >> lw) * nthr) : 0ull;
    }
    float s = 0.0f;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int q = q0 + u;
      if (q < total) {
        const int r = q & wm, i = tid + (q >> lw) * nthr;
        const uint32_t bits =
            tp_ll_tag(w[u]) == tag
                ? tp_ll_bits(w[u])
                : tp_ll_wait(t.src[r] + i, tag, [](const uint64_t* p) { return tp_ld_word(p); },
                             [] { return tp_now_ns(); }, deadline, ok);
        const float f = __uint_as_float(bits);
        s = r == 0 ? f : s + f;
        if (r == wm) out(i, s);
      }
    }
  }
}

// Fills the producer or consumer view of exchange x (parity x & 1: a step
// has an even number of exchanges, so the parity of every exchange of a
// step is fixed) of hidden-size vectors.
void tp_xchg(const TpPeers& p, int nx, int x, int rows, const unsigned* step, float* sum_out, TpXchg* out);

// sum_out = base + rank-order sum of exchange t's partials, after waiting
// for them (one CTA; for a step whose last exchange no GEMV consumes).
cudaError_t launch_tp_finalize(const TpXchg& t, const float* base, int* err, cudaStream_t st);
// *step += 1 (the first kernel of a tensor-parallel step).
cudaError_t launch_tp_step(unsigned* step, cudaStream_t st);
// Merges the ranks' sampler results (each rank's k_argmax over its vocab
// slice wrote its own `top`): global first max (ties to the lowest index),
// top-2 gap, then the StepState update of k_argmax.
cudaError_t launch_tp_sample_merge(const TpPeers& p, StepState* st, int* history, int history_cap, unsigned* epoch,
                                   int* err, cudaStream_t st_);

}  // namespace mcpo
