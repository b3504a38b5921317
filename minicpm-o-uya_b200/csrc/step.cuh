// step.cuh -- the persistent decode-step kernel: one cooperative launch
// runs a whole token's layer chain (the stage list below) on one CTA per SM.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "attention.cuh"
#include "gemv.cuh"

namespace mcpo {

enum StageKind : int { kStageGemv = 0, kStageAttn = 1 };

// One stage of the step.  Every stage reads what earlier stages wrote, so
// stages are separated by grid-wide barriers; the weight stream of GEMV
// stages runs ahead of them.
struct alignas(16) StageDesc {  // size a multiple of 16: copied with cp.async.bulk
  int kind;
  GemvArgs g;   // kStageGemv (prepared by gemv_prepare)
  AttnArgs at;  // kStageAttn (fused norm/rope/append; counters zero at rest)
};

struct StepPlan {
  const StageDesc* stages;  // device array
  int n_stages;
  int nc;        // consumer warps per CTA (plus one producer warp)
  int S;         // ring slots per consumer warp
  int slot;      // bytes per ring slot (largest step block of the plan)
  int x_bytes;   // shared region for the activations / the attention stage
  unsigned* bar; // grid barrier arrivals (zero before each launch)
  int* abort;    // set by a CTA that gives up (zero before each launch)
  int* err;      // error word (StepState::err)
  int preissue;  // ring copies per warp issued for an f32-input GEMV stage before its prologue is done
  unsigned long long* trace;  // optional: [stage][CTA][3] globaltimer ns: start, activations ready, all warps done
};

// Shared memory the attention stage needs for head_dim hd.
size_t step_attn_bytes(int hd);
// Picks the consumer-warp count and ring depth for a plan whose largest step
// block is `slot` bytes and whose shared activation/attention region is
// x_bytes; returns false when the plan does not fit a CTA.
bool step_layout(int slot, size_t x_bytes, int* nc, int* S, size_t* smem);
cudaError_t decode_step_init();
// q80: every GEMV stage is Q8_0 (else every GEMV stage is Q4_K/Q6_K);
// kv_f16: the attention stages' KV cache is f16.  grid CTAs must be
// co-resident (one per SM); the launch is cooperative.
cudaError_t launch_decode_step(const StepPlan& p, int grid, size_t smem, bool q80, bool kv_f16, cudaStream_t st);

}  // namespace mcpo
