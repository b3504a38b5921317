/*
 * ref_kernel_emul.cpp -- runs the reference GPU shim's own device code on
 * the CPU.  TEST INFRASTRUCTURE ONLY.
 *
 * The reference keeps its CUDA kernels as a C string inside
 * src/minicpmo/gpu_shim.c:500-979 (compiled at run time with NVRTC, no
 * --use_fast_math, --fmad=false).  oracle/Makefile extracts that string,
 * unmodified, into oracle/_ref/shim_kernels.cu; this file compiles it as
 * host C++ by defining the CUDA keywords away, then drives the
 * sync-free per-thread device functions exactly as the kernels'
 * launch shapes do (gpu_shim.c:1215-1264: 128 threads per row, a shared
 * memory halving tree).  The result is the reference CUDA path's float
 * arithmetic, evaluated in the same order, on the host.
 *
 * Only the sync-free device functions are called.  Kernels that use
 * __syncthreads (quantize, norms, attention) are compiled but never run.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#define __device__
#define __global__
#define __forceinline__ inline
#define __shared__ static
static inline void __syncthreads(void) {}
struct refk_dim3 { unsigned x, y, z; };
static thread_local refk_dim3 threadIdx, blockIdx, blockDim;
static inline float rsqrtf(float x) { return 1.0f / sqrtf(x); }

#include "_ref/shim_kernels.cu"

namespace {
template <float (*DotRow)(const unsigned char *, const unsigned char *, int, int)>
void emulate_matvec(const unsigned char *w, const unsigned char *xq, float *y, int rows, int cols) {
    float buf[128];
    for (int row = 0; row < rows; ++row) {
        for (int tid = 0; tid < 128; ++tid) {
            threadIdx.x = (unsigned) tid;
            buf[tid] = DotRow(w, xq, row, cols);
        }
        for (int stride = 64; stride > 0; stride >>= 1)
            for (int tid = 0; tid < stride; ++tid) buf[tid] += buf[tid + stride];
        y[row] = buf[0];
    }
}
}  // namespace

extern "C" {

/* gpu_shim.c:809-820 + 843-855 launched as grid=rows, block=128 */
void refk_q4_k_matvec(const unsigned char *w, const unsigned char *xq, float *y, int rows, int cols) {
    emulate_matvec<minicpmo_q4_k_dot_row>(w, xq, y, rows, cols);
}

/* gpu_shim.c:879-890 + 913-925 */
void refk_q6_k_matvec(const unsigned char *w, const unsigned char *xq, float *y, int rows, int cols) {
    emulate_matvec<minicpmo_q6_k_dot_row>(w, xq, y, rows, cols);
}

/* gpu_shim.c:572-597 (device f32 -> f16) */
unsigned short refk_float_to_half(float v) { return minicpmo_float_to_half(v); }
float refk_half_to_float(unsigned short b) { return minicpmo_half_to_float(b); }

/* gpu_shim.c:665-693, launched grid=heads, block=256 (table form) */
void refk_apply_rope(float *vec, int head_count, int head_dim, int pos, const float *cos_t, const float *sin_t) {
    for (int h = 0; h < head_count; ++h) {
        blockIdx.x = (unsigned) h;
        for (int d = 0; d < 256; ++d) {
            threadIdx.x = (unsigned) d;
            minicpmo_apply_rope(vec, head_count, head_dim, pos, 1000000.0f, 1.0f, cos_t, sin_t);
        }
    }
}

/* gpu_shim.c:659-664 */
void refk_silu_mul(float *dst, const float *gate, const float *up, int n) {
    blockDim.x = 256;
    for (int b = 0; b < (n + 255) / 256; ++b) {
        blockIdx.x = (unsigned) b;
        for (int t = 0; t < 256; ++t) {
            threadIdx.x = (unsigned) t;
            minicpmo_silu_mul(dst, gate, up, n);
        }
    }
}

}  // extern "C"
