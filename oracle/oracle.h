/*
 * oracle.h -- CPU restatement of the Qwen3 quantised decode path of
 * uya-lang/minicpm-o-uya.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls
 * this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker / the timed CPU baseline.
 *
 * Every function cites the reference file:line it restates (paths are
 * relative to the reference project root).  Parity pins: see
 * oracle/Makefile (reference sources compiled into oracle/_ref/) and
 * tests/test_oracle_pins.py.
 */
#ifndef MINICPMO_ORACLE_H
#define MINICPMO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Uya TensorDType ordinals (src/minicpmo/tensor.uya:31-54). */
enum {
    ORC_F32 = 0,
    ORC_F16 = 1,
    ORC_Q8_0 = 6,
    ORC_Q4_K = 10,
    ORC_Q6_K = 12,
    ORC_BF16 = 20,
};

/* ---- scalar conversions (src/minicpmo/kernels.uya:48-108, gpu_shim.c:2124-2192) ---- */
float orc_f16_to_f32(uint16_t bits);
float orc_bf16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16(float value); /* reference rounding: ties away from zero */

/* ---- block formats ---- */
size_t orc_row_bytes(int dtype, size_t cols); /* 0 when cols is not a legal multiple */
int orc_dequant_row(int dtype, const uint8_t *row, size_t cols, float *out);

/* Q8_1 (36-byte f16-scale block), gpu_shim.c:336-401 (variant B). */
int orc_q8_1_quantize(const float *x, size_t n, uint8_t *dst);
/* Sum of the 32 int8 quants of each Q8_1 block (what dp4a(0x01010101, q8) yields). */
int orc_q8_1_block_sums(const uint8_t *xq, size_t nblocks, int32_t *sums);

/* Per-block integer dot products (bit-exact contract).
 * Q4_K: per 32-element sub-block j: dot_d[j] = sum q4*q8 (gpu_shim.c:746-808,
 *       kernels.uya:503-547); dot_m[j] = sum q8.
 * Q6_K: per 16-element scale group g: dots[g] = sum (q6-32)*q8 (gpu_shim.c:856-878).
 * Q8_0: per 32-element block b: dots[b] = sum qw*q8. */
int orc_q4_k_block_dots(const uint8_t *row, const uint8_t *xq, size_t cols, int32_t *dot_d, int32_t *dot_m);
int orc_q6_k_block_dots(const uint8_t *row, const uint8_t *xq, size_t cols, int32_t *dots);
int orc_q8_0_block_dots(const uint8_t *row, const uint8_t *xq, size_t cols, int32_t *dots);

/* y = W . x with Q8_1 activations (the reference CUDA path's arithmetic). */
int orc_matvec_q8_1(int dtype, const uint8_t *w, size_t rows, size_t cols, const uint8_t *xq, float *y);
/* y = W . x with f32 activations (the reference CPU path, qwen3.uya:869-1014 and
 * cpu_kernels.c:254-395 scalar forms). */
int orc_matvec_f32(int dtype, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y);

/* ---- elementwise / normalisation ---- */
/* order 0: sequential sum (qwen3.uya:1176-1186); order 1: the 256-lane strided
 * partial sums + halving tree of gpu_shim.c:694-718 with an exact 1/sqrtf. */
int orc_rms_norm(const float *x, const void *w, int w_dtype, size_t n, float eps, int order, float *out);
/* qwen3.uya:1543-1558 (order 0) / gpu_shim.c:719-745 (order 1), eps fixed 1e-6 */
int orc_head_norm(float *vec, const void *w, int w_dtype, size_t head_count, size_t head_dim, int order);
/* qwen3.uya:1633-1662 */
int orc_rope_table(size_t context, size_t head_dim, float freq_base, float freq_scale, float *cos_out, float *sin_out);
/* qwen3.uya:1605-1631 (table form) */
int orc_rope_apply(float *vec, size_t head_count, size_t head_dim, size_t pos, const float *cos_t, const float *sin_t);
/* qwen3.uya:1664-1713 + softmax kernels.uya:149-160 */
int orc_attention(float *out, const float *q, const float *k_cache, const float *v_cache, size_t layer, size_t pos,
                  size_t head_count, size_t kv_head_count, size_t head_dim, size_t context);
/* kernels.uya:198 + qwen3.uya:1970 */
void orc_silu_mul(float *dst, const float *gate, const float *up, size_t n);
/* qwen3.uya:1734-1752, plus the gap between the best and second-best
 * (penalised) values; gap is +inf when n == 1. */
uint32_t orc_argmax_penalized(const float *values, size_t n, const uint32_t *seen, size_t seen_count, float penalty,
                              float *top2_gap);
/* qwen3_sample (qwen3.uya:2073-2138), see oracle.c; *seed is the xorshift32 state. */
uint32_t orc_sample(const float *logits, size_t vocab, const uint32_t *seen, size_t seen_count, float temp,
                    uint32_t top_k, float top_p, float min_p, float penalty, uint32_t *seed, float *margin);

/* ---- device evaluation order --------------------------------------------
 * The reference fixes each operation's formula but not the order of float
 * sums (its CPU and CUDA paths differ).  The B200 kernels evaluate in one
 * documented order using only correctly rounded IEEE operations; the
 * functions below restate that order so the whole decode step can be
 * compared bit for bit.  Same formulas as the reference, fixed order:
 *  - matvec: per row, LPR lanes (largest power of two <= 32 dividing
 *    cols/256); lane l sums super-blocks l, l+LPR, ... in order; the lanes
 *    are combined by an xor butterfly (LPR/2 .. 1) and lane 0 is the row;
 *  - attention: positions in blocks of 32; per block and head a partial
 *    (m = max score, l = butterfly sum of exp(s - m), acc = sum p v in
 *    position order), the blocks merged in block order;
 *  - exp: orc_expf_det (Cody-Waite reduction + degree-7 Taylor/Horner).
 */
float orc_expf_det(float x);
int orc_attn_n_split(int n_kv);
uint16_t orc_f32_to_f16_rne(float v); /* IEEE round-to-nearest-even (f16 KV cache) */
int orc_matvec_q8_1_dev(int dtype, const uint8_t *w, size_t rows, size_t cols, const uint8_t *xq, float *y);
int orc_matvec_dense_dev(int dtype, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y);
void orc_silu_mul_dev(float *dst, const float *gate, const float *up, size_t n);
/* k_cache/v_cache hold f32 values (already rounded through f16 when the
 * cache is f16); cur_k/cur_v are the current position's unrounded rows. */
int orc_attention_dev(float *out, const float *q, const float *k_cache, const float *v_cache, const float *cur_k,
                      const float *cur_v, size_t layer, size_t pos, size_t head_count, size_t kv_head_count,
                      size_t head_dim, size_t context);

/* ---- whole decode step (qwen3.uya:1920-1995) ---- */
typedef struct orc_layer {
    const void *attn_norm; int attn_norm_dtype;
    const uint8_t *q; int q_dtype;
    const uint8_t *k; int k_dtype;
    const uint8_t *v; int v_dtype;
    const void *q_norm; int q_norm_dtype; /* may be NULL */
    const void *k_norm; int k_norm_dtype; /* may be NULL */
    const uint8_t *o; int o_dtype;
    const void *ffn_norm; int ffn_norm_dtype;
    const uint8_t *gate; int gate_dtype;
    const uint8_t *up; int up_dtype;
    const uint8_t *down; int down_dtype;
} orc_layer;

typedef struct orc_model {
    uint32_t layers, hidden, heads, kv_heads, head_dim, ffn, vocab, context;
    float eps;
    const uint8_t *token_embd; int token_embd_dtype;
    const void *output_norm; int output_norm_dtype;
    const uint8_t *output; int output_dtype; /* tied: token_embd */
    const orc_layer *layer;
    const float *rope_cos; /* [context][head_dim/2] */
    const float *rope_sin;
} orc_model;

/* Matvec hook so the CPU baseline can substitute the reference's own
 * threaded matvec (cpu_kernels.c:791-851).  Returns 1 on success. */
typedef int (*orc_matvec_fn)(void *user, int dtype, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y);

typedef struct orc_state {
    float *k_cache; /* [layers][context][kv_dim] */
    float *v_cache;
    /* mode 1: Q8_1 activations + per-block int dots (the CUDA path);
     * mode 0: f32 activations (the CPU path). */
    int q8_1_activations;
    /* 0: the reference CPU order (sequential sums, libm expf);
     * 1: the device evaluation order above (bit-exact contract) */
    int norm_order;
    int kv_f16; /* order 1 only: the KV cache stores f16 (RNE) values */
    /* optional row pool (cpu_pool.c): mode 0 through matvec, mode 1 through
     * orc_pool_matvec_q8_1 on matvec_user */
    orc_matvec_fn matvec; void *matvec_user;
} orc_state;

/* cpu_pool.c: a row-partitioned thread pool (threads >= 1; ref_cpu_so names
 * the reference's cpu_kernels.c build for mode 0, or NULL) */
void *orc_pool_create(int threads, const char *ref_cpu_so);
void orc_pool_destroy(void *pool);
void orc_state_attach_pool(orc_state *st, void *pool);
/* Q8_1 matvec over the pool's threads: order 1 device order, 0 natural
 * order; every row's bits equal the single-threaded call's */
int orc_pool_matvec_q8_1(void *pool, int order, int dtype, const uint8_t *w, size_t rows, size_t cols,
                         const uint8_t *xq, float *y);

size_t orc_state_kv_floats(const orc_model *m);
/* logits may be NULL (no lm_head); hidden_out may be NULL. */
int orc_forward_token(const orc_model *m, orc_state *st, uint32_t token, size_t pos, float *logits, float *hidden_out);
/* The same on a caller-given f32 input row (qwen3_append_prompt_embeddings, qwen3.uya:2534-2557). */
int orc_forward_embedding(const orc_model *m, orc_state *st, const float *emb, size_t pos, float *logits,
                          float *hidden_out);

#ifdef __cplusplus
}
#endif
#endif
