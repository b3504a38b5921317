// tp.cuh -- tensor-parallel exchanges between the ranks of one node, over
// CUDA IPC mappings of each rank's exchange buffer (peer loads over NVLink;
// no multicast, no TMA on peer memory).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "misc.cuh"

namespace mcpo {

constexpr int kTpMaxWorld = 8;

// One rank's exchange buffer (allocated by that rank, IPC-exported):
//   part[2][hidden]  f32 partial sums of the row-parallel GEMVs (o, down),
//                    alternating per exchange so a buffer is never rewritten
//                    while a slower peer still reads it;
//   top[4]           this rank's sampler result (best, index, second, pad);
//   flag             the last exchange epoch this rank has published.
struct TpLayout {
  static size_t part_offset(int buf, size_t hidden) { return (size_t)buf * hidden * 4; }
  static size_t top_offset(size_t hidden) { return 2 * hidden * 4; }
  static size_t flag_offset(size_t hidden) { return 2 * hidden * 4 + 16; }
  static size_t bytes(size_t hidden) { return (2 * hidden * 4 + 16 + 16 + 255) / 256 * 256; }
};

// Device view of all ranks' buffers (own and peer-mapped).
struct TpPeers {
  float* part[kTpMaxWorld][2];
  float* top[kTpMaxWorld];
  unsigned* flag[kTpMaxWorld];
  int rank, world;
};

// hidden[i] += part_0[i] + part_1[i] + ... + part_{W-1}[i] (rank order, so
// every rank computes identical bits), after publishing this rank's epoch
// and waiting (bounded, 1 s) for every peer's.  epoch is this rank's counter
// (advanced by the kernel); err is raised on a timeout.
cudaError_t launch_tp_reduce_add(const TpPeers& p, int buf, float* hidden, int n, unsigned* epoch, int* err,
                                 cudaStream_t st);
// Merges the ranks' sampler results (each rank's k_argmax over its vocab
// slice wrote its own `top`): global first max (ties to the lowest index),
// top-2 gap, then the StepState update of k_argmax.
cudaError_t launch_tp_sample_merge(const TpPeers& p, StepState* st, int* history, int history_cap, unsigned* epoch,
                                   int* err, cudaStream_t st_);

}  // namespace mcpo
