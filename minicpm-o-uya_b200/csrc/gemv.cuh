// gemv.cuh -- host-visible launch descriptors for the quantised GEMV and the
// activation (Q8_1) producers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "layout.cuh"
#include "tp.cuh"

// Kernel timelines (trace fields below) are compiled in only when the
// library is built with MCPO_TRACE=1 (make TRACE=1).
#ifndef MCPO_TRACE
#define MCPO_TRACE 0
#endif

namespace mcpo {

enum GemvEpilogue : int {
  kEpiStore = 0,   // y[row] = W.x
  kEpiAdd = 1,     // y[row] = y[row] + W.x   (residual add, qwen3.uya:1964-1973)
  kEpiSwiglu = 2,  // y[row] = silu(Wg.x) * (Wu.x)   (kernels.uya:198, qwen3.uya:1970)
  kEpiTpPush = 3,  // tensor parallelism: W.x of row r to tp.dst[d][r] on every rank d, then the arrival counts
};

struct GemvSeg {
  const uint8_t* w;   // tiled weights
  const uint8_t* w2;  // kEpiSwiglu: tiled "up" weights, same geometry as w
  float* y;
  int dtype;
  int rows;
  int lpr, rpw, ks;
  int step_bytes;
  int n_wr;           // warp-rows
  int wr_begin;       // first warp-row of this segment in the launch's warp-row space
  int epi;
  size_t wr_bytes;
};

constexpr int kMaxSegs = 3;

// Where a GEMV's Q8_1 input comes from.  Each CTA builds the shared-memory
// copy of the activations in its prologue; the f32 modes quantise there with
// the arithmetic of k_quantize_q8_1 / k_rmsnorm_q8_1, so the quants and
// scales are bit-identical to feeding those kernels' output through xq.
enum GemvInput : int {
  kInQ8_1 = 0,     // xq: Q8_1 blocks in global memory
  kInF32 = 1,      // xf: f32 values, quantised in the prologue
  kInRmsNorm = 2,  // xf: f32 values; RMSNorm(xf) * norm_w (eps), then quantised
  // tensor parallelism: x = xf + (sum of the ranks' partials of exchange
  // tp, rank order) once they have all arrived; x also goes to tp.sum_out
  // (each CTA its share); then as kInRmsNorm on x
  kInRmsNormTp = 3,
};

// All segments of one launch share the input width `cols` (hence lpr/ks);
// a kEpiSwiglu launch has exactly one segment.
struct GemvArgs {
  GemvSeg seg[kMaxSegs];
  int nseg;
  int cols;
  int total_wr;
  int stages;          // ring slots per consumer warp
  int slot_bytes;      // max step block bytes over the segments
  int input;           // GemvInput
  const uint8_t* xq;   // kInQ8_1: Q8_1 activations, cols/32 blocks of 36 B
  const float* xf;     // kInF32 / kInRmsNorm: f32 activations [cols]
  const void* norm_w;  // kInRmsNorm: norm weight [cols] (F32 / F16 / BF16)
  int norm_dtype;
  float eps;
  int* dots;           // optional: per-block integer dots, [row][block] (parity tests)
  int* err;            // set to 1 when a bounded wait gives up
  // several input vectors against one pass over the weights (prompt
  // prefill): vector n reads xf + n*x_stride (floats) or xq + n*xq_stride
  // (bytes) and writes y + n*y_stride (floats) of each segment; nvec <= 1:
  // one vector
  int nvec;
  int x_stride, xq_stride, y_stride;
  // optional (one segment, one vector): the outputs also as Q8_1 blocks
  // (36 B per 32 rows, the bits k_quantize_q8_1 gives for y), each CTA
  // taking whole 32-row blocks; a following GEMV reads them as kInQ8_1
  uint8_t* q8_out;
  // kEpiTpPush / kInRmsNormTp: the exchange produced or consumed
  TpXchg tp;
  // optional timeline (builds with MCPO_TRACE=1), [CTA][8] globaltimer ns:
  // start, past the wait for the previous kernel, activations ready, all
  // consumer warps done (4 unused)
  unsigned long long* trace;
};

constexpr int kGemvMaxVec = 4;  // input vectors per multi-vector launch

// Fills seg from a tile geometry.
inline void gemv_seg_from_geom(const TileGeom& g, const uint8_t* w, const uint8_t* w2, float* y, int epi,
                               GemvSeg* s) {
  s->w = w;
  s->w2 = w2;
  s->y = y;
  s->dtype = g.dtype;
  s->rows = g.rows;
  s->lpr = g.lpr;
  s->rpw = g.rpw;
  s->ks = g.ks;
  s->step_bytes = g.step_bytes;
  s->n_wr = g.n_wr;
  s->wr_begin = 0;
  s->epi = epi;
  s->wr_bytes = g.wr_bytes;
}

// One-time per-device setup (opts the GEMV kernels into large shared memory).
cudaError_t gemv_init();
// Bytes of the shared-memory activation region of a GEMV over `cols` inputs.
size_t gemv_x_bytes_host(int cols);
// Lays the segments out in one warp-row space (wr_begin, total_wr,
// slot_bytes) and validates them; *dtypes_mask gets bit 0 Q4_K, 1 Q6_K,
// 2 Q8_0.
cudaError_t gemv_prepare(GemvArgs& a, int* dtypes_mask);
// Launches over `grid` persistent CTAs (one per SM); fills wr_begin, total_wr,
// stages and slot_bytes.  pdl: allow programmatic dependent launch.
cudaError_t launch_gemv(GemvArgs& a, int grid, cudaStream_t st, bool pdl);

// Q8_1 producers (36-byte blocks in the reference layout, gpu_shim.c:37-41).
// x f32 [n] -> xq
cudaError_t launch_quantize_q8_1(const float* x, int n, uint8_t* xq, cudaStream_t st, bool pdl = false);
// RMSNorm(x) * w -> (optional f32 out) -> xq.  eps as given; reduction order
// of gpu_shim.c:694-718 (256 strided partial sums, halving tree), exact
// 1/sqrtf.  xq may be null (plain RMSNorm).
cudaError_t launch_rmsnorm_q8_1(const float* x, const void* w, int w_dtype, int n, float eps, float* out,
                                uint8_t* xq, cudaStream_t st, bool pdl = false);

// Dense F32/F16/BF16 GEMV (row-major GGUF layout), f32 activations.
cudaError_t launch_dense_gemv(const void* w, int dtype, int rows, int cols, const float* x, float* y,
                              cudaStream_t st, bool pdl = false);

// Launch helper: programmatic dependent launch attribute when pdl is set.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                     Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace mcpo
