// gemv.cuh -- host-visible launch descriptors for the quantised GEMV and the
// activation (Q8_1) producers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "layout.cuh"

namespace mcpo {

enum GemvEpilogue : int {
  kEpiStore = 0,   // y[row] = W.x
  kEpiAdd = 1,     // y[row] = y[row] + W.x   (residual add, qwen3.uya:1964-1973)
  kEpiSwiglu = 2,  // y[row] = silu(Wg.x) * (Wu.x)   (kernels.uya:198, qwen3.uya:1970)
};

struct GemvSeg {
  const uint8_t* w;   // tiled weights
  const uint8_t* w2;  // kEpiSwiglu: tiled "up" weights, same geometry as w
  float* y;
  int dtype;
  int rows;
  int lpr, rpw, ks;
  int step_bytes;
  int tile_begin;     // first CTA tile of this segment in the launch's tile space
  int n_tiles;
  int epi;
  size_t cta_tile_bytes;
};

constexpr int kMaxSegs = 3;

struct GemvArgs {
  GemvSeg seg[kMaxSegs];
  int nseg;
  int cols;
  int total_tiles;
  const uint8_t* xq;  // Q8_1 activations, cols/32 blocks of 36 B
  int* dots;          // optional: per-block integer dots, [row][block] (parity tests)
};

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
  s->n_tiles = g.n_cta_tiles;
  s->epi = epi;
  s->cta_tile_bytes = g.cta_tile_bytes;
  s->tile_begin = 0;
}

size_t gemv_smem_bytes(int cols);
// CTAs of the GEMV kernel resident per SM for this input width (also opts the
// kernel into the dynamic shared memory it needs; call before launching).
int gemv_occupancy(int cols);
cudaError_t launch_gemv(GemvArgs& a, int grid, cudaStream_t st);

// Q8_1 producers (36-byte blocks in the reference layout, gpu_shim.c:37-41).
// x f32 [n] -> xq
cudaError_t launch_quantize_q8_1(const float* x, int n, uint8_t* xq, cudaStream_t st);
// RMSNorm(x) * w -> (optional f32 out) -> xq.  eps as given; reduction order
// of gpu_shim.c:694-718 (256 strided partial sums, halving tree), exact
// 1/sqrtf.  xq may be null (plain RMSNorm).
cudaError_t launch_rmsnorm_q8_1(const float* x, const void* w, int w_dtype, int n, float eps, float* out,
                                uint8_t* xq, cudaStream_t st);

// Dense F32/F16/BF16 GEMV (row-major GGUF layout), f32 activations.
cudaError_t launch_dense_gemv(const void* w, int dtype, int rows, int cols, const float* x, float* y,
                              cudaStream_t st);

}  // namespace mcpo
