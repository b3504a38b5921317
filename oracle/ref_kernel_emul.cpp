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
 * The sync-free device functions are driven per thread in order.  Kernels
 * that use __syncthreads (the RMSNorm, head-norm and decode-attention
 * kernels) run one block at a time with one host thread per CUDA thread and
 * a barrier for __syncthreads, so every thread reaches each barrier before
 * any passes it: the kernel's own phase order.  Their __shared__ variables
 * are function statics, shared by the block's threads.  rsqrtf is taken as
 * 1/sqrtf (CUDA's is an approximation within 2 ulp of that), expf is the
 * host's.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>

#include <thread>
#include <vector>

#define __device__
#define __global__
#define __forceinline__ inline
#define __shared__ static
static pthread_barrier_t refk_block_barrier;
static inline void __syncthreads(void) { pthread_barrier_wait(&refk_block_barrier); }
struct refk_dim3 { unsigned x, y, z; };
static thread_local refk_dim3 threadIdx, blockIdx, blockDim;
static inline float rsqrtf(float x) { return 1.0f / sqrtf(x); }

#include "_ref/shim_kernels.cu"

namespace {
// One block of `threads` CUDA threads as host threads meeting at a barrier.
template <typename Body>
void run_block(unsigned block, unsigned threads, Body body) {
    pthread_barrier_init(&refk_block_barrier, NULL, threads);
    std::vector<std::thread> ts;
    ts.reserve(threads);
    for (unsigned t = 0; t < threads; ++t)
        ts.emplace_back([=] {
            threadIdx = refk_dim3{t, 0, 0};
            blockIdx = refk_dim3{block, 0, 0};
            blockDim = refk_dim3{threads, 1, 1};
            body();
        });
    for (auto &th : ts) th.join();
    pthread_barrier_destroy(&refk_block_barrier);
}
}  // namespace

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

/* gpu_shim.c:694-718, launched grid=1, block=256 (gpu_shim.c:3344-3350) */
void refk_rms_norm(float *dst, const float *src, const unsigned char *weight, int weight_dtype, int n, float eps) {
    run_block(0, 256, [=] { minicpmo_rms_norm(dst, src, weight, weight_dtype, n, eps); });
}

/* gpu_shim.c:719-745, launched grid=heads, block=256 (gpu_shim.c:3424-3430) */
void refk_head_norm(float *vec, const unsigned char *weight, int weight_dtype, int head_count, int head_dim) {
    for (int h = 0; h < head_count; ++h)
        run_block((unsigned) h, 256, [=] { minicpmo_head_norm(vec, weight, weight_dtype, head_dim); });
}

/* gpu_shim.c:926-979, launched grid=heads, block=256 (gpu_shim.c:1542-1570) */
void refk_attention_decode(const float *q, const float *k_cache, const float *v_cache, float *dst, int layer, int pos,
                           int head_count, int kv_head_count, int head_dim, int context_capacity, float scale) {
    for (int h = 0; h < head_count; ++h)
        run_block((unsigned) h, 256, [=] {
            minicpmo_qwen3_attention_decode(q, k_cache, v_cache, dst, layer, pos, head_count, kv_head_count, head_dim,
                                            context_capacity, scale);
        });
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
