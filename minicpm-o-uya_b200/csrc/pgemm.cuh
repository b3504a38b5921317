// pgemm.cuh -- prompt-prefill projections on the sm_100a tensor cores.
//
// A prompt of T tokens multiplies every linear weight with T activation
// vectors.  The decode GEMV (gemv.cu) computes, per row and 32-value block
// (16 for Q6_K), an exact int32 dot of the weight's integer values with the
// Q8_1 quants, then combines the dots with the block scales in a fixed
// float order.  Here the integer dots of 128 rows x 32 tokens come from
// tcgen05.mma kind::i8 (s8 x s8 -> s32, exact), one MMA per block into its
// own tensor-memory region, and the epilogue warps combine them in the
// decode's float order -- per super-block the same fma chains, per lane the
// same sequential sum over its super-blocks, per row the same butterfly
// tree -- so every output is bit-identical to the decode GEMV's.
//
// Operands (built once per matrix from the tiled GEMV copy, layout.cuh):
//   A[tile][sb]: 128 rows x 256 int8 values of super-block sb in natural
//     value order (Q4_K: q in 0..15; Q6_K: q - 32; Q8_0: q), as K-major
//     8-row x 16-byte core matrices: core (chunk c, row group g) at byte
//     (c * 16 + g) * 128, row r%8 at +16*(r%8).
//   S[tile][sb]: 32 bytes per row: Q4_K the 16-byte {d, dmin, scales[12]}
//     header; Q6_K the 16 int8 scales and the f16 d; Q8_0 the 8 f16 d's.
// Activations (per call, launch_pgemm_act):
//   B[ttile][sb]: 32 tokens x 256 Q8_1 quants, core (chunk c, token group
//     g) at (c * 4 + g) * 128;  Bm[ttile][sb][half]: B with the odd (half 0)
//     or even (half 1) 16-value chunks zeroed, for Q6_K's 16-value groups;
//   X[ttile][sb]: per block j and token n, d8 (the Q8_1 block's f16 d) at
//     [j][n] and d8 * (sum of the block's quants) at [256 + j * 32 + n].
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "layout.cuh"

namespace mcpo {

constexpr int kPgRows = 128;                // rows per CTA tile (the MMA's M)
constexpr int kPgTok = 32;                  // tokens per CTA tile (the MMA's N)
constexpr int kPgABytes = kPgRows * 256;    // 32768
constexpr int kPgSBytes = kPgRows * 32;     // 4096
constexpr int kPgBBytes = kPgTok * 256;     // 8192
constexpr int kPgXFloats = 2 * 8 * kPgTok;  // 512

struct PgemmMat {
  int dtype = 0, rows = 0, cols = 0, tiles = 0, nb = 0;
  int lpr = 1, ks = 1;   // the decode GEMV's lanes per row and steps (its reduction tree)
  uint8_t* a = nullptr;  // [tiles][nb][kPgABytes]
  uint8_t* s = nullptr;  // [tiles][nb][kPgSBytes]
};

struct PgemmAct {
  int tmax = 0, K = 0;
  uint8_t* b = nullptr;   // [ttiles][nb][kPgBBytes]
  uint8_t* bm = nullptr;  // [ttiles][nb][2][kPgBBytes]
  float* xs = nullptr;    // [ttiles][nb][kPgXFloats]
  // launches with fewer CTAs than SMs split each row tile over the GEMV
  // lanes (subtrees of the row's reduction tree) into at most split_ctas
  // CTAs: their roots (split_ctas x 32 x 128 floats) and per-tile arrival
  // counts (zero at rest)
  int split_ctas = 0;
  float* part = nullptr;
  unsigned* cnt = nullptr;
};

enum PgemmEpi : int { kPgStore = 0, kPgAdd = 1, kPgSwiglu = 2 };

// Builds the operand copy of a tiled quantised matrix (allocates a and s).
cudaError_t pgemm_build(const TileGeom& g, const uint8_t* tiled, PgemmMat* out, cudaStream_t st);
void pgemm_free(PgemmMat* m);
size_t pgemm_mat_bytes(const TileGeom& g);

// Activation buffers for up to tmax tokens of K values (K % 256 == 0).
cudaError_t pgemm_act_alloc(int tmax, int K, PgemmAct* a);
void pgemm_act_free(PgemmAct* a);

// T rows of K f32 values (row stride ldx) -> Q8_1 operands, optionally
// after RMSNorm with weights norm_w (null: none), in the decode GEMV's
// arithmetic (gemv_build_x).
cudaError_t launch_pgemm_act(const float* x, int ldx, int T, const void* norm_w, int norm_dtype, float eps,
                             const PgemmAct& a, cudaStream_t st);

// y[t * ldy + r] (t < T, r < rows) = the decode GEMV's output for token t:
// kPgStore: the row value; kPgAdd: y + value; kPgSwiglu: silu_mul_det(gate[t * ldg + r], value).
cudaError_t launch_pgemm(const PgemmMat& w, const PgemmAct& x, int T, int epi, float* y, int ldy, const float* gate,
                         int ldg, int* err, cudaStream_t st);

cudaError_t pgemm_init();

}  // namespace mcpo
