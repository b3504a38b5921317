// layout.cuh -- the device layout of quantised weight matrices.
//
// GGUF stores a matrix row-major with each row a run of blocks
// (src/minicpmo/tensor.uya:260-294; rows = shape[1], cols = shape[0]).
// Q6_K (210 B) and Q8_0 (34 B) blocks are not 16-byte multiples, so a row of
// them cannot be streamed with 128-bit loads.  At upload the helper rewrites
// every quantised matrix into "warp tiles": the bytes are only moved, never
// changed, so dequantisation is bit-identical to the GGUF bytes.
//
//   super-block (SB): 256 values of one row.  Q4_K and Q6_K SBs are the GGUF
//     blocks; for Q8_0 an SB is 8 consecutive GGUF blocks (272 B).
//   chunk: 16 B of an SB.  Q4_K: chunk 0 = {d, dmin, scales[12]}, chunks 1..8 =
//     qs.  Q6_K: chunks 0..7 = ql, 8..11 = qh, 12 = sc, plus a 2-byte d.
//     Q8_0: chunk 0 = the 8 f16 d's, chunks 1..16 = the 256 int8 quants.
//   warp-row: a warp processes RPW rows at a time, LPR lanes per row
//     (LPR = the largest power of two <= 32 dividing nb = cols/256); lane
//     l covers row l/LPR and, at step k, SB k*LPR + l%LPR.  KS = nb/LPR steps.
//   step block: for one step k, the chunks of all 32 lanes, chunk-major:
//     [chunk c][lane] x 16 B (+ [lane] x 2 B of Q6_K d) = 32 * SB bytes, so a
//     warp reading one chunk reads 512 contiguous bytes.
//   Warp-rows are stored one after another, each as its KS step blocks in
//   order: a range of warp-rows is one contiguous byte range, and one step
//   block is one 16-byte aligned bulk copy.
//   Rows are padded with zero bytes up to a whole number of warp-rows.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace mcpo {

struct TileGeom {
  int dtype;
  int rows, cols;
  int nb;        // super-blocks per row
  int lpr;       // lanes per row
  int rpw;       // rows per warp
  int ks;        // steps per lane tile
  int sb_bytes;  // bytes per super-block
  int chunks;    // 16-byte chunks per super-block (excluding Q6_K's d)
  int step_bytes;   // 32 * sb_bytes
  int n_wr;         // warp-rows, ceil(rows / rpw)
  size_t wr_bytes;  // ks * step_bytes
  size_t total_bytes;
};

__host__ __device__ inline bool is_quant(int dtype) {
  return dtype == kQ4_K || dtype == kQ6_K || dtype == kQ8_0;
}

__host__ __device__ inline int sb_bytes_of(int dtype) {
  return dtype == kQ4_K ? 144 : dtype == kQ6_K ? 210 : dtype == kQ8_0 ? 272 : 0;
}

__host__ __device__ inline int chunks_of(int dtype) {
  return dtype == kQ4_K ? 9 : dtype == kQ6_K ? 13 : dtype == kQ8_0 ? 17 : 0;
}

// GGUF bytes of one row.
__host__ __device__ inline size_t gguf_row_bytes(int dtype, size_t cols) {
  switch (dtype) {
    case kF32: return cols * 4;
    case kF16: case kBF16: return cols * 2;
    case kQ8_0: return cols % 32 ? 0 : cols / 32 * 34;
    case kQ4_K: return cols % 256 ? 0 : cols / 256 * 144;
    case kQ6_K: return cols % 256 ? 0 : cols / 256 * 210;
    default: return 0;
  }
}

__host__ __device__ inline bool make_geom(int dtype, int rows, int cols, TileGeom* g) {
  if (!is_quant(dtype) || rows <= 0 || cols <= 0 || cols % 256) return false;
  g->dtype = dtype;
  g->rows = rows;
  g->cols = cols;
  g->nb = cols / 256;
  int lpr = 32;
  while (lpr > 1 && (g->nb % lpr) != 0) lpr >>= 1;
  g->lpr = lpr;
  g->rpw = 32 / lpr;
  g->ks = g->nb / lpr;
  g->sb_bytes = sb_bytes_of(dtype);
  g->chunks = chunks_of(dtype);
  g->step_bytes = 32 * g->sb_bytes;
  g->n_wr = (rows + g->rpw - 1) / g->rpw;
  g->wr_bytes = (size_t)g->ks * g->step_bytes;
  g->total_bytes = (size_t)g->n_wr * g->wr_bytes;
  return true;
}

// Byte offset, inside the tiled buffer, of the step block holding SB `sb` of
// row `row`, and the lane that owns it.
__host__ __device__ inline size_t step_block_offset(const TileGeom& g, int row, int sb, int* lane) {
  const int wr = row / g.rpw;
  const int riw = row % g.rpw;
  const int k = sb / g.lpr;
  *lane = riw * g.lpr + sb % g.lpr;
  return (size_t)wr * g.wr_bytes + (size_t)k * g.step_bytes;
}

// Address of byte `o` (0 <= o < sb_bytes, in GGUF SB order) of SB `sb` of
// row `row` in the tiled buffer.  For Q8_0, `o` indexes the 272-byte SB in
// the tiled order (chunk 0 = d's); gguf_q8_0_to_tiled() maps GGUF bytes.
__host__ __device__ inline size_t tiled_byte_offset(const TileGeom& g, int row, int sb, int o) {
  int lane;
  size_t base = step_block_offset(g, row, sb, &lane);
  if (g.dtype == kQ6_K && o >= 208) return base + 13 * 512 + lane * 2 + (o - 208);
  return base + (size_t)(o / 16) * 512 + lane * 16 + (o % 16);
}

}  // namespace mcpo
