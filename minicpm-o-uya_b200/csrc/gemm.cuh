// gemm.cuh -- batched decode projections on the 5th-generation tensor cores:
// Y[n][row] (+)= sum_k W[row][k] * X[n][k] for up to 32 independent
// sequences n, with W a GGUF Q8_0 matrix in its raw row layout.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mcpo {

constexpr int kGemmTileRows = 128;  // rows per CTA tile (the MMA's M)
constexpr int kGemmKTile = 256;     // K values per staged tile (8 Q8_0 blocks per row)
constexpr int kGemmMaxN = 32;       // sequences per launch
constexpr int kGemmMaxSegs = 3;

enum GemmEpi : int { kGemmStore = 0, kGemmAdd = 1 };

// One matrix of a launch: Q8_0 bytes re-tiled by launch_gemm_tile_weights
// (one 34816-byte block per 128 rows x 256 values, [rows/128][cols/256]).
struct GemmSeg {
  const uint8_t* w;
  int rows;  // multiple of kGemmTileRows
};

// A launch covers the concatenation of up to three matrices sharing the
// input (rows of segment i follow those of segment i-1); output row r of
// the concatenation goes to y[n * ldy + r].
struct GemmArgs {
  GemmSeg seg[kGemmMaxSegs];
  int nseg;
  int rows_total;
  int K;              // multiple of kGemmKTile
  const uint8_t* x;   // activations, f16, operand layout (gemm_x_offset)
  int N;              // 16 or 32 (operand rows; rows >= n_valid are zero)
  int n_valid;        // sequences written
  float* y;
  int ldy;
  int epi;            // GemmEpi
  int ksplit;         // K-tile ranges per row tile (1: no partials)
  float* partial;     // [ksplit][N][rows_total] when ksplit > 1
  unsigned* counters; // [rows_total / 128], zero at rest, when ksplit > 1
  int* err;           // raised by a bounded wait that gave up
};

// Byte offset of element (n, k) in the f16 operand layout of N rows:
// [K/256 tiles][32 chunks of 8 values][N/8 row groups][8 rows][8 values].
// One K-tile of all N rows is contiguous (N * 512 bytes), and inside it the
// 8x16-byte core matrices of the tensor-core K-major layout.
__host__ __device__ inline size_t gemm_x_offset(int n, int k, int N) {
  return ((size_t)(k >> 8) * 32 + ((k & 255) >> 3)) * (size_t)(N >> 3) * 128 + (size_t)(n >> 3) * 128 +
         (size_t)(n & 7) * 16 + (size_t)(k & 7) * 2;
}

// Split count for a launch of `tiles` row tiles over `ktiles` K-tiles on
// `sms` SMs (one CTA per SM): enough CTAs to cover the SMs once.
int gemm_pick_ksplit(int tiles, int ktiles, int sms);

cudaError_t gemm_init();
// GGUF Q8_0 rows [rows][K/32 * 34 bytes] (device) -> the GemmSeg tiling
// (same size); rows % 128 == 0, K % 256 == 0.
cudaError_t launch_gemm_tile_weights(const uint8_t* src, uint8_t* dst, int rows, int K, cudaStream_t st);
cudaError_t launch_gemm_q80(const GemmArgs& a, cudaStream_t st, bool pdl = false);

// f32 rows x[n][ld] (n < n_valid, k < K) -> the f16 operand layout; rows
// n_valid..N-1 of the operand are left as they are (zero at allocation).
cudaError_t launch_pack_x16(const float* x, int ld, int n_valid, int K, int N, uint8_t* x16, cudaStream_t st,
                            bool pdl = false);
// RMSNorm of each row (reduction order of gpu_shim.c:694-718, exact
// 1/sqrtf) times the weight, into the operand layout.
cudaError_t launch_rmsnorm_x16(const float* x, int ld, const void* w, int w_dtype, int n_valid, int K, float eps,
                               int N, uint8_t* x16, cudaStream_t st, bool pdl = false);
// SwiGLU of gate/up rows gu[n][2*F] (gate first) into the operand layout of
// K = F values: silu(g) * u with silu(g) = g / (1 + exp(-g)).
cudaError_t launch_swiglu_x16(const float* gu, int F, int n_valid, int N, uint8_t* x16, cudaStream_t st,
                              bool pdl = false);

}  // namespace mcpo
