// tp_proto.h -- the tensor-parallel exchange protocol, shared by the CUDA
// kernels (tp.cu, gemv_dev.cuh) and the host-thread harness of its CPU test.
//
// Every rank of a tensor-parallel decode runs the same sequence of steps,
// and every step the same number `nx` of exchanges (two per layer: after the
// row-parallel o and down projections).  In exchange x of step s (the step
// counter counts from 1) every source rank stores its partial vector of
// `rows` values into a slot of every rank's exchange buffer (remote stores
// over NVLink).  Each value travels with the exchange's tag in one
// naturally aligned 64-bit word (value bits in the low half, tag in the
// high half), written and read as single-copy-atomic 64-bit accesses: a
// reader that sees the tag it expects has the value of that exchange, so
// no fence, release or arrival counter is needed.  The consumer of the
// exchange waits (bounded) element by element until every source's word
// carries the tag, then sums the partials in rank order, so every rank
// computes identical bits.
//
// Tags are the exchange's global index mod 2^32 - 1, plus one: never 0 (the
// zeroed buffer's content) and different for the two exchanges that can
// share a slot.  Slots alternate between two parities by the global index:
// a source can only write an exchange's slot again two exchanges later,
// after every rank has consumed the exchange in between, which it cannot do
// before this rank has contributed to it, i.e. before this rank finished
// reading the slot.
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

// The slot parity of exchange `index`.
TP_HD int tp_parity(uint32_t index) { return (int)(index & 1u); }

// The tag of exchange `index`: 1 .. 2^32 - 1.
TP_HD uint32_t tp_tag(uint32_t index) { return index % 0xffffffffu + 1u; }

TP_HD uint64_t tp_ll_pack(uint32_t bits, uint32_t tag) { return (uint64_t)bits | ((uint64_t)tag << 32); }
TP_HD uint32_t tp_ll_tag(uint64_t w) { return (uint32_t)(w >> 32); }
TP_HD uint32_t tp_ll_bits(uint64_t w) { return (uint32_t)w; }

// Waits until the word at p carries `tag` and returns its value bits.
// load(p) is a single-copy-atomic 64-bit load, now() a clock in
// nanoseconds.  Gives up once now() passes `deadline` (or after a fixed
// number of polls), clearing *ok; a caller whose *ok is already clear does
// not wait again.  Returns 0 when it gave up.
template <typename Load, typename Now>
TP_HD uint32_t tp_ll_wait(const uint64_t* p, uint32_t tag, Load load, Now now, uint64_t deadline, bool* ok) {
  uint64_t w = load(p);
  uint32_t polls = 0;
  while (tp_ll_tag(w) != tag) {
    if (!*ok) return 0u;
    if ((++polls & 63u) == 0u && (now() > deadline || polls > (1u << 24))) {
      *ok = false;
      return 0u;
    }
    w = load(p);
  }
  return tp_ll_bits(w);
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
