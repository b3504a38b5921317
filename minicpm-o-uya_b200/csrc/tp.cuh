// tp.cuh -- tensor-parallel exchanges between the ranks of one node, over
// CUDA IPC mappings of each rank's exchange buffer (stores and loads over
// NVLink; no multicast, no TMA on peer memory).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "misc.cuh"
#include "tp_proto.h"

namespace mcpo {

// One rank's exchange buffer (allocated by that rank, IPC-exported):
//   part[2][kTpMaxWorld][hidden]  f32 partial hidden vectors of the
//                    row-parallel GEMVs (o, down), written by each source
//                    rank into its own slot, two parities (tp_proto.h);
//   arrive[kTpMaxWorld]  values received from each source (monotonic);
//   top[4]           this rank's sampler result (best, index, second, pad);
//   flag             the last sampler-merge epoch this rank has published.
struct TpLayout {
  static size_t part_offset(int parity, int src, size_t hidden) {
    return ((size_t)parity * kTpMaxWorld + (size_t)src) * hidden * 4;
  }
  static size_t arrive_offset(size_t hidden) { return 2 * (size_t)kTpMaxWorld * hidden * 4; }
  static size_t top_offset(size_t hidden) { return arrive_offset(hidden) + kTpMaxWorld * 4; }
  static size_t flag_offset(size_t hidden) { return top_offset(hidden) + 16; }
  static size_t bytes(size_t hidden) { return (flag_offset(hidden) + 16 + 255) / 256 * 256; }
};

// Device view of all ranks' buffers (own and peer-mapped).
struct TpPeers {
  uint8_t* base[kTpMaxWorld];
  float* top[kTpMaxWorld];
  unsigned* flag[kTpMaxWorld];
  int rank, world;
};

// One exchange as a GEMV sees it (gemv.cuh: kEpiTpPush produces it,
// kInRmsNormTp consumes it).
struct TpXchg {
  // producer: output row r of this rank's partial goes to dst[d][r] on every
  // rank d, then each dst_arrive[d] (rank d's counter for this rank) grows by
  // the rows a CTA stored
  float* dst[kTpMaxWorld];
  unsigned* dst_arrive[kTpMaxWorld];
  // consumer: base[i] + (src[0][i] + ... + src[world-1][i]) once every
  // arrive[r] reaches the exchange's target; the sum also goes to sum_out
  // (each CTA its share)
  const float* src[kTpMaxWorld];
  const unsigned* arrive;
  float* sum_out;
  const unsigned* step;  // the step counter (advanced by k_tp_step at each step's start)
  int world;
  int nx;    // exchanges per step
  int x;     // this exchange's index within the step
  int rows;  // values per exchange (hidden)
};

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
