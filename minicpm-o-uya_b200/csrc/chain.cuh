// chain.cuh -- a chain of GEMVs as one persistent launch (decode_mode 3).
//
// Between two attentions a decode layer is four dependent GEMVs: o (+
// residual), gate/up (RMSNorm prologue, SwiGLU + Q8_1 epilogue), down (+
// residual), and the next layer's q/k/v (RMSNorm prologue).  As separate
// launches each pays a kernel boundary: the release of the previous grid,
// its own start-up and tail, and a weight stream that stops until its CTAs
// are resident.  The chain kernel runs them as stages of one launch: one CTA
// per SM, the stages separated by grid barriers, and one producer warp whose
// lanes stream every stage's step blocks into the consumer warps' rings in
// order -- across the barriers, so the next stage's weights arrive while
// the current one finishes and the barrier settles.  Each stage is the
// standalone GEMV's arithmetic (gemv_build_x, gemv_items), so the results
// are bit-identical to the per-operation graph.
#pragma once

#include <cuda_runtime.h>

#include "gemv.cuh"
#include "gemv_dev.cuh"

namespace mcpo {

constexpr int kMaxChain = 4;

struct GemvChain {
  const GemvArgs* stages;  // device array of n stages (prepared by gemv_prepare)
  int n;                   // 1..kMaxChain
  int cls;                 // GemvClass covering every stage's weight types
  int nc, S, slot;         // consumer warps, ring slots per warp, bytes per slot
  int x_bytes;             // activation region (the largest stage's)
  int q8_floats;           // floats of the Q8_1-epilogue staging buffer (0: no stage has one)
  unsigned* bar;           // n - 1 grid-barrier arrival counters, zero before the launch
  int* abort;              // set by a CTA that gives up (zero before the launch)
  int* err;                // error word (StepState::err)
  // MCPO_TRACE builds: per stage and CTA four globaltimer stamps (stage
  // start, activations ready, rows done, stage done) at
  // trace[((stage / 2) * trace_ctas + cta) * 8 + (stage % 2) * 4 + i]; null: none
  unsigned long long* trace;
  int trace_ctas;
};

// Kernel class and ring layout of a chain over the given (host-side,
// prepared) stages with their gemv_prepare dtype masks; false when the
// stages cannot share a kernel or do not fit a CTA.
bool chain_layout(const GemvArgs* stages, const int* dtype_masks, int n, int sm_count, GemvChain* c, size_t* smem);
cudaError_t chain_init();
// grid = the SM count (every CTA must be resident: the stages synchronise
// through grid barriers); the launch lets the next kernel start only after
// all of its CTAs have started.
cudaError_t launch_gemv_chain(const GemvChain& c, int grid, size_t smem, cudaStream_t st);

}  // namespace mcpo
