// tp_proto.h -- the tensor-parallel exchange protocol, shared by the CUDA
// kernels (tp.cu, gemv_dev.cuh) and the host-thread harness of its CPU test.
//
// Every rank of a tensor-parallel decode runs the same sequence of steps,
// and every step the same number `nx` of exchanges (two per layer: after the
// row-parallel o and down projections).  In exchange x of step s (the step
// counter counts from 1) every source rank pushes its partial vector of
// `rows` values into a slot of every rank's exchange buffer (remote stores
// over NVLink), then adds the number of values it stored to that rank's
// arrival counter for it.  The consumer of the exchange waits (bounded)
// until every source's counter reaches the exchange's target, then sums the
// partials in rank order, so every rank computes identical bits.
//
// Counters are monotonic 32-bit and compared with wraparound arithmetic,
// so they are never reset while ranks run.  Slots alternate between two
// parities by the exchange's global index: a source can only write an
// exchange's slot again two exchanges later, after every rank has consumed
// the exchange in between, which it cannot do before this rank has
// contributed to it, i.e. before this rank finished reading the slot.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define TP_HD __host__ __device__ __forceinline__
#else
#define TP_HD inline
#endif

namespace mcpo {

constexpr int kTpMaxWorld = 8;

// Global index of exchange x of step `step` (step >= 1).
TP_HD uint32_t tp_exchange_index(uint32_t step, uint32_t nx, uint32_t x) { return (step - 1u) * nx + x; }

// Arrival count at which all `rows` values of exchange `index` have arrived
// from one source.
TP_HD uint32_t tp_target(uint32_t index, uint32_t rows) { return (index + 1u) * rows; }

TP_HD bool tp_arrived(uint32_t count, uint32_t target) { return (int32_t)(count - target) >= 0; }

// The slot parity of exchange `index`.
TP_HD int tp_parity(uint32_t index) { return (int)(index & 1u); }

// Waits until arrive[0..world) all reach `target`.  load(p) is an acquire
// load of counter p, now() a clock in nanoseconds; gives up (false) once
// limit_ns have passed or after a fixed number of polls.
template <typename Load, typename Now>
TP_HD bool tp_wait_all(const uint32_t* arrive, int world, uint32_t target, Load load, Now now, uint64_t limit_ns) {
  const uint64_t t0 = now();
  uint32_t polls = 0;
  for (int r = 0; r < world; ++r) {
    while (!tp_arrived(load(arrive + r), target)) {
      if ((++polls & 255u) == 0u && (now() - t0 > limit_ns || polls > (1u << 26))) return false;
    }
  }
  return true;
}

// Sum of one value over the ranks' partials, in rank order, then added to
// the residual: base + (p_0 + p_1 + ... + p_{world-1}).
template <typename LoadPart>
TP_HD float tp_rank_sum(float base, int world, LoadPart part) {
  float t = part(0);
  for (int r = 1; r < world; ++r) t = t + part(r);
  return base + t;
}

}  // namespace mcpo
