/*
 * minicpmo_gpu.h -- C ABI of libminicpmo_gpu_helper.so, the B200 (sm_100a)
 * drop-in for the GPU helper of uya-lang/minicpm-o-uya.
 *
 * Part 1 is the reference helper ABI, symbol for symbol: the reference's
 * bridge (src/minicpmo/gpu_bridge.c:72-90) dlmopen()s
 * <exe dir>/libminicpmo_gpu_helper.so and requires exactly these 19 symbols
 * (gpu_bridge.c:146-176); each declaration cites the reference
 * implementation it replaces (src/minicpmo/gpu_shim.c).  Conventions are the
 * reference's: functions return 1 on success and 0 on error, copying an
 * "error: ..." message into (error, error_cap); dtype integers are the Uya
 * TensorDType ordinals F32=0, F16=1, Q8_0=6, Q4_K=10, Q6_K=12, BF16=20
 * (src/minicpmo/tensor.uya:31-54); weight tensors are keyed by the caller's
 * host pointer (gpu_shim.c:1592-1600); 2-D tensors pass cols = shape[0]
 * (contiguous) and rows = shape[1] (src/minicpmo/gpu.uya:137-148).
 *
 * Part 2 holds versioned extensions (discover with dlsym; old hosts ignore
 * them): device embedding lookup and greedy sampler, the fused whole-token
 * Qwen3 decode step, batched decode, tensor-parallel contexts, and
 * measurement/parity helpers.
 */
#ifndef MINICPMO_GPU_H
#define MINICPMO_GPU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MINICPMO_API __attribute__((visibility("default")))
#else
#define MINICPMO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* gpu_bridge.c:11-25 / gpu_shim.c:129-143: 13 x u64, layout fixed (the
 * caller allocates it). */
typedef struct minicpmo_gpu_stats {
    uint64_t backend_init_us;
    uint64_t host_to_device_bytes;
    uint64_t device_to_host_bytes;
    uint64_t weight_upload_bytes;
    uint64_t scratch_x_bytes;
    uint64_t scratch_y_bytes;
    uint64_t uploaded_weight_count;
    uint64_t native_quant_matvec_count;
    uint64_t staged_quant_matvec_count;
    uint64_t q8_1_x_bytes;
    uint64_t attention_kernel_calls;
    uint64_t kv_device_bytes;
    uint64_t kv_host_to_device_bytes;
} minicpmo_gpu_stats;

/* ===================== Part 1: reference helper ABI ===================== */

/* gpu_shim.c:2207-2345 */
MINICPMO_API int minicpmo_gpu_context_create(unsigned int device_index, int debug, void **out_handle, char *error, size_t error_cap);
/* gpu_shim.c:2347-2423 (NULL-safe) */
MINICPMO_API void minicpmo_gpu_context_destroy(void *handle);
/* gpu_shim.c:2425-2454 */
MINICPMO_API int minicpmo_gpu_context_smoke(void *handle, char *error, size_t error_cap);
/* gpu_shim.c:2456-2527 */
MINICPMO_API int minicpmo_gpu_context_upload_tensor(void *handle, const char *name, const void *host_ptr, size_t bytes, int dtype,
                                       size_t rows, size_t cols, char *error, size_t error_cap);
/* gpu_shim.c:2529-2719 (host x in, host dst out) */
MINICPMO_API int minicpmo_gpu_context_matvec(void *handle, const char *tensor_name, const void *host_ptr, int dtype, const float *x,
                                size_t in_dim, size_t out_dim, float *dst, char *error, size_t error_cap);
/* gpu_shim.c:1385-1454 */
MINICPMO_API int minicpmo_gpu_context_prepare_attention(void *handle, size_t layer_count, size_t context_capacity, size_t kv_dim,
                                           char *error, size_t error_cap);
/* gpu_shim.c:1456-1590 (host q/k/v in, host dst out; appends k/v at pos) */
MINICPMO_API int minicpmo_gpu_context_attention(void *handle, const float *q, const float *k, const float *v, size_t layer, size_t pos,
                                   size_t head_count, size_t kv_head_count, size_t head_dim, size_t context_capacity,
                                   float *dst, char *error, size_t error_cap);
/* gpu_shim.c:2721-2747 */
MINICPMO_API int minicpmo_gpu_context_slot_upload_f32(void *handle, unsigned int slot, const float *src, size_t len, char *error,
                                         size_t error_cap);
/* gpu_shim.c:2749-2774 (synchronises) */
MINICPMO_API int minicpmo_gpu_context_slot_download_f32(void *handle, unsigned int slot, float *dst, size_t len, char *error,
                                           size_t error_cap);
/* gpu_shim.c:2776-3008 */
MINICPMO_API int minicpmo_gpu_context_slot_matvec(void *handle, unsigned int dst_slot, const char *tensor_name, const void *host_ptr,
                                     int dtype, unsigned int src_slot, size_t in_dim, size_t out_dim, char *error,
                                     size_t error_cap);
/* gpu_shim.c:3233-3255 */
MINICPMO_API int minicpmo_gpu_context_slot_matvec2(void *handle, unsigned int dst_slot0, const char *tensor_name0,
                                      const void *host_ptr0, int dtype0, size_t out_dim0, unsigned int dst_slot1,
                                      const char *tensor_name1, const void *host_ptr1, int dtype1, size_t out_dim1,
                                      unsigned int src_slot, size_t in_dim, char *error, size_t error_cap);
/* gpu_shim.c:3257-3284 */
MINICPMO_API int minicpmo_gpu_context_slot_matvec3(void *handle, unsigned int dst_slot0, const char *tensor_name0,
                                      const void *host_ptr0, int dtype0, size_t out_dim0, unsigned int dst_slot1,
                                      const char *tensor_name1, const void *host_ptr1, int dtype1, size_t out_dim1,
                                      unsigned int dst_slot2, const char *tensor_name2, const void *host_ptr2,
                                      int dtype2, size_t out_dim2, unsigned int src_slot, size_t in_dim, char *error,
                                      size_t error_cap);
/* gpu_shim.c:3286-3368 */
MINICPMO_API int minicpmo_gpu_context_slot_rms_norm(void *handle, unsigned int dst_slot, unsigned int src_slot,
                                       const void *weight_host_ptr, size_t n, float eps, char *error, size_t error_cap);
/* gpu_shim.c:3370-3448 (in place, eps 1e-6) */
MINICPMO_API int minicpmo_gpu_context_slot_head_norm(void *handle, unsigned int slot, const void *weight_host_ptr, size_t head_count,
                                        size_t head_dim, char *error, size_t error_cap);
/* gpu_shim.c:3450-3526 (table keyed by host pointer; NULL tables -> computed) */
MINICPMO_API int minicpmo_gpu_context_slot_rope(void *handle, unsigned int slot, size_t head_count, size_t head_dim, size_t pos,
                                   float freq_base, float freq_scale, const float *rope_cos, const float *rope_sin,
                                   size_t rope_context, char *error, size_t error_cap);
/* gpu_shim.c:3528-3577 */
MINICPMO_API int minicpmo_gpu_context_slot_add_inplace(void *handle, unsigned int dst_slot, unsigned int src_slot, size_t len,
                                          char *error, size_t error_cap);
/* gpu_shim.c:3579-3633 */
MINICPMO_API int minicpmo_gpu_context_slot_silu_mul(void *handle, unsigned int dst_slot, unsigned int gate_slot,
                                       unsigned int up_slot, size_t len, char *error, size_t error_cap);
/* gpu_shim.c:3635-3743 (appends k/v at pos, then attends) */
MINICPMO_API int minicpmo_gpu_context_attention_slots(void *handle, unsigned int dst_slot, unsigned int q_slot, unsigned int k_slot,
                                         unsigned int v_slot, size_t layer, size_t pos, size_t head_count,
                                         size_t kv_head_count, size_t head_dim, size_t context_capacity, char *error,
                                         size_t error_cap);
/* gpu_shim.c:3745-3753 */
MINICPMO_API void minicpmo_gpu_context_snapshot(void *handle, minicpmo_gpu_stats *stats);

/* ========================= Part 2: extensions =========================== */

#define MINICPMO_GPU_ABI_VERSION 1

/* No reference counterpart: lets a host detect the extensions. */
MINICPMO_API int minicpmo_gpu_abi_version(void);

/* Stream the context enqueues on (cudaStream_t as void*).  The reference uses
 * the legacy NULL stream (gpu_shim.c:1238-1248); this helper owns a
 * non-blocking stream.  set_stream adopts a caller stream (not owned). */
MINICPMO_API void *minicpmo_gpu_context_stream(void *handle);
MINICPMO_API int minicpmo_gpu_context_set_stream(void *handle, void *stream, char *error, size_t error_cap);

/* Device token-embedding dequant lookup into a slot (replaces the host
 * qwen3_copy_embedding, src/minicpmo/qwen3.uya:1164-1174, and its 4*h byte
 * upload per token, qwen3.uya:1876). */
MINICPMO_API int minicpmo_gpu_context_embed_lookup(void *handle, unsigned int dst_slot, const void *host_ptr, int dtype,
                                      uint32_t token, size_t hidden, char *error, size_t error_cap);

/* Device greedy sampler over a slot (replaces the host
 * qwen3_argmax_penalized, qwen3.uya:1734-1752, and its 4*V byte download):
 * first maximum of the penalised values, plus the gap to the second best. */
MINICPMO_API int minicpmo_gpu_context_argmax_penalized(void *handle, unsigned int slot, size_t n, const uint32_t *seen,
                                          size_t seen_count, float penalty, uint32_t *out_id, float *out_top2_gap,
                                          char *error, size_t error_cap);

/* Whole-model decode step (replaces the ~20 calls per layer of
 * qwen3_forward_embedding_runtime_cuda, qwen3.uya:1865-1918, with one CUDA
 * graph launch).  Tensors are found in the upload registry by their GGUF
 * names (blk.N.attn_q.weight, ...; output.weight, then lm_head.weight, then
 * token_embd.weight for the lm_head as tensor_lookup_root_output,
 * src/minicpmo/tensor.uya:503-509). */
typedef struct minicpmo_qwen3_config {
    uint32_t layers, hidden, heads, kv_heads, head_dim, ffn, vocab, context;
    float rms_eps;          /* the reference forward uses 1e-6 (qwen3.uya:108) */
    float rope_freq_base;   /* qwen3.rope.freq_base, default 1e6 */
    float rope_freq_scale;  /* 1/linear factor (qwen3.uya:1578-1603) */
    const float *rope_cos;  /* host tables [context][head_dim/2] or NULL: */
    const float *rope_sin;  /*   then built as qwen3_precompute_rope (qwen3.uya:1633-1662) */
    int kv_f16;             /* 0: f32 KV cache (reference); 1: f16 */
    int max_batch;          /* sequences of the batched decode (forward_batch,
                               decode_batch): 0 or 1 -> none; 2..32 needs every
                               linear weight Q8_0 */
    int decode_mode;        /* 0: the default (currently 1, the faster one measured);
                               1: one kernel per operation (a CUDA graph of ~5 per
                               layer); 2: one persistent kernel per decode step when
                               the model fits it (all linear weights Q4_K/Q6_K, or
                               all Q8_0), else 1; 3: per layer the attention and one
                               launch chaining the o, gate/up, down and next q/k/v
                               GEMVs (one GPU, tiled weights, head_dim % 32 == 0;
                               the bind fails otherwise).  Same results in every
                               mode. */
    int batch_exact;        /* with max_batch: 1 runs the batch's projections as the
                               prompt prefill does (int8 block dots on the tensor
                               cores), so every sequence gets the single-sequence
                               decode's bits (slower: about 0.8x at 32 sequences);
                               0: f16 operands on the tensor cores (within 1e-3) */
    int reserved[4];
} minicpmo_qwen3_config;

MINICPMO_API int minicpmo_gpu_context_qwen3_bind(void *handle, const minicpmo_qwen3_config *config, char *error, size_t error_cap);

/* ---- tensor parallelism over the GPUs of one node (one process per GPU) ----
 * 1. every rank: minicpmo_gpu_context_tp_buffer(hidden) allocates this rank's
 *    exchange buffer and returns its cudaIpcMemHandle_t (64 bytes);
 * 2. the host all-gathers the handles (rank order) by any means;
 * 3. every rank uploads the full tensors as for qwen3_bind, then calls
 *    qwen3_bind_tp(cfg, rank, world, handles): the rank keeps its shards --
 *    q/k/v by heads, gate/up/down by 256-value FFN blocks, o by its heads'
 *    input columns, the lm_head by vocab rows -- in buffers of their own and
 *    releases the full copies of those tensors (they leave the upload
 *    registry; re-upload them to bind again).  Its decode graph sums the o
 *    and down partials of all ranks inside the GEMVs around them: the o and
 *    down GEMVs store their partial rows into every rank's exchange buffer
 *    over NVLink, and the next GEMV's prologue waits (bounded) for all of
 *    them and adds them in rank order.  The per-rank samplers are merged;
 * 4. the host barriers the ranks, then drives qwen3_forward / qwen3_decode on
 *    every rank with the same tokens; every rank returns the same token.
 * heads, kv_heads must divide by world; ffn by 256.  With tensor parallelism
 * qwen3_forward's logits_out receives only this rank's vocab slice (at its
 * offset).  No reference counterpart (the reference is single-GPU). */
MINICPMO_API int minicpmo_gpu_context_tp_buffer(void *handle, size_t hidden, void *ipc_handle_out, char *error,
                                   size_t error_cap);
MINICPMO_API int minicpmo_gpu_context_qwen3_bind_tp(void *handle, const minicpmo_qwen3_config *config, int rank, int world,
                                       const void *peer_ipc_handles, char *error, size_t error_cap);

/* Forward `token` at `pos` (qwen3_forward_token_runtime, qwen3.uya:1991-1995)
 * and sample greedily on the device.  flags bit 0: skip the lm_head and the
 * sampler (prompt tokens that need no logits).  logits_out (may be NULL)
 * receives the vocab logits; hidden_out (may be NULL) the final hidden
 * state.  repeat_penalty <= 1 disables the penalty (qwen3.uya:1734-1752);
 * every forwarded token joins the penalty's seen set. */
MINICPMO_API int minicpmo_gpu_context_qwen3_forward(void *handle, uint32_t token, size_t pos, int flags, float repeat_penalty,
                                       uint32_t *out_token, float *out_top2_gap, float *logits_out, float *hidden_out,
                                       char *error, size_t error_cap);
/* Forward one caller-given f32 input row (`n` = hidden values, host memory)
 * at `pos` in place of a token's embedding row, with `placeholder_id` as the
 * token recorded for it (it joins the repeat penalty's seen set): one step of
 * qwen3_append_prompt_embeddings (qwen3.uya:2534-2557, which forwards each
 * span row through qwen3_forward_embedding_runtime and records the
 * placeholder in prompt_ids).  flags, outputs and errors as
 * minicpmo_gpu_context_qwen3_forward. */
MINICPMO_API int minicpmo_gpu_context_qwen3_forward_embedding(void *handle, const float *embedding, size_t n,
                                                 uint32_t placeholder_id, size_t pos, int flags, float repeat_penalty,
                                                 uint32_t *out_token, float *out_top2_gap, float *logits_out,
                                                 float *hidden_out, char *error, size_t error_cap);
/* qwen3_sample (qwen3.uya:2073-2138) on the logits of the last forward that
 * computed them: seen[seen_count] is the token history (prompt_ids, with
 * repeats), *seed_state the xorshift32 state (advanced when a draw is made).
 * As in the reference, vocabularies above 256 tokens, temperature <= 1e-6
 * or top_k <= 1 sample greedily (the penalty once per seen token); else the
 * penalty per history entry, temperature, softmax, top-k, top-p, min-p and
 * one draw.  Not available under tensor parallelism.  Returns 1, or 0 with
 * a message in `error`. */
MINICPMO_API int minicpmo_gpu_context_qwen3_sample(void *handle, const uint32_t *seen, size_t seen_count,
                                      float temperature, uint32_t top_k, float top_p, float min_p,
                                      float repeat_penalty, uint32_t *seed_state, uint32_t *out_token, char *error,
                                      size_t error_cap);
/* Forward the n prompt tokens tokens[0..n) at positions first_pos.. in
 * passes over the weights (the reference prefills token by token,
 * qwen3.uya:2485-2506): 16 tokens or more in passes of up to 256 with the
 * projections on the tensor cores (exact int8 block dots, the first call
 * builds an int8 operand copy of the weights, about 1.1 bytes per weight;
 * MCPO_PREFILL_TC=0 turns this off), fewer in passes of up to 4 through the
 * GEMVs.  Every token's arithmetic is that of qwen3_forward, so the KV
 * cache and the last token's logits and greedy sample (flags bit 0 clear)
 * equal those of n forwards.
 * The tokens join the penalty's seen set.  Models whose weights are not all
 * in the tiled GEMV layouts (or under tensor parallelism) are refused with
 * an error; use qwen3_forward for them. */
MINICPMO_API int minicpmo_gpu_context_qwen3_prefill(void *handle, const uint32_t *tokens, size_t n, size_t first_pos,
                                       int flags, float repeat_penalty, uint32_t *out_token,
                                       float *out_top2_gap, float *logits_out, char *error, size_t error_cap);
/* Clears the sampler's seen set (a new session, qwen3.uya:2999-3007). */
MINICPMO_API int minicpmo_gpu_context_qwen3_reset(void *handle, char *error, size_t error_cap);
/* Save and restore a session's KV prefix: copy rows [first_pos, first_pos +
 * n_pos) of layer `layer`'s K and V caches from host memory (kv_write) or
 * to it (kv_read).  A row is kv_heads * head_dim values (under tensor
 * parallelism this rank's heads) in the cache's element type: f32, or f16
 * when the model was bound with kv_f16.  Synchronous.  Not available for a
 * batched model.  No reference counterpart (the reference keeps its cache in
 * the helper, gpu_shim.c:1385-1454, and never exposes it). */
MINICPMO_API int minicpmo_gpu_context_qwen3_kv_write(void *handle, size_t layer, size_t first_pos, size_t n_pos,
                                        const void *k_rows, const void *v_rows, char *error, size_t error_cap);
MINICPMO_API int minicpmo_gpu_context_qwen3_kv_read(void *handle, size_t layer, size_t first_pos, size_t n_pos,
                                       void *k_rows, void *v_rows, char *error, size_t error_cap);

/* Greedy decode of n_steps tokens entirely on the device, feeding each
 * sampled token back (the generate loop, qwen3.uya:2559-2639, without host
 * round trips).  tokens_out[n_steps] receives the sampled ids. */
MINICPMO_API int minicpmo_gpu_context_qwen3_decode(void *handle, uint32_t first_token, size_t first_pos, size_t n_steps,
                                      float repeat_penalty, uint32_t *tokens_out, char *error, size_t error_cap);

/* ---- batched decode of independent sequences (config: all linear weights
 * Q8_0; no reference counterpart -- the reference decodes one sequence,
 * qwen3.uya:2412-2639, and has no GPU Q8_0 path, gpu.uya:130-132) ----
 * Bound by qwen3_bind with max_batch in 2..32: every linear weight (q, k, v,
 * o, gate, up, down, lm_head) must be Q8_0 with rows % 128 == 0 and
 * cols % 256 == 0.  The projections run on the tensor cores (weights and
 * activations rounded to f16, sums in f32); every sequence has its own KV
 * cache ([layer][sequence][context][kv_dim]), position and greedy sampler
 * (no repeat penalty).  n_seq must equal max_batch. */
/* One step: sequence i forwards tokens[i] at positions[i].  flags bit 0:
 * skip the lm_head and samplers (prompt positions).  out_tokens /
 * out_top2_gaps [n_seq] and logits_out [n_seq][vocab] may be NULL. */
MINICPMO_API int minicpmo_gpu_context_qwen3_forward_batch(void *handle, size_t n_seq, const uint32_t *tokens,
                                             const uint32_t *positions, int flags, uint32_t *out_tokens,
                                             float *out_top2_gaps, float *logits_out, char *error,
                                             size_t error_cap);
/* Greedy decode of n_steps tokens per sequence on the device, feeding each
 * sampled token back; tokens_out [n_seq][n_steps] (may be NULL). */
MINICPMO_API int minicpmo_gpu_context_qwen3_decode_batch(void *handle, size_t n_seq, const uint32_t *first_tokens,
                                            const uint32_t *first_positions, size_t n_steps, uint32_t *tokens_out,
                                            char *error, size_t error_cap);
/* Device time of n_steps batched decode steps (graph replays, CUDA events
 * on the context stream); total_ms over all steps. */
MINICPMO_API int minicpmo_gpu_context_qwen3_time_decode_batch(void *handle, size_t n_seq, const uint32_t *first_tokens,
                                                 const uint32_t *first_positions, size_t n_steps, float *total_ms,
                                                 char *error, size_t error_cap);
/* Kernel launches in one batched step's graph; 0 without a batched model. */
MINICPMO_API int minicpmo_gpu_context_qwen3_batch_kernels(void *handle, int with_logits);

/* ---- parity and measurement helpers (no reference counterpart) ---- */

/* Device Q8_1 quantisation of host f32 values (36-byte blocks, the
 * reference's host quantiser gpu_shim.c:336-401 bit for bit). */
MINICPMO_API int minicpmo_gpu_context_q8_1_quantize(void *handle, const float *x, size_t n, void *xq_out, char *error,
                                       size_t error_cap);
/* Device RMSNorm -> Q8_1 producer of the decode step on host data:
 * out = x * (1/sqrtf(sum(x^2)/n + eps)) * w with the sum in the order of
 * gpu_shim.c:694-718; the weight is an uploaded tensor. */
MINICPMO_API int minicpmo_gpu_context_rms_norm_q8_1(void *handle, const float *x, const void *weight_host_ptr, size_t n, float eps,
                                       float *out, void *xq_out, char *error, size_t error_cap);
/* GEMV of an uploaded quantised tensor with caller-given Q8_1 activations;
 * dots_out (may be NULL) receives every per-block int32 dot, row-major
 * [out_dim][in_dim/32] (Q4_K, Q8_0) or [out_dim][in_dim/16] (Q6_K). */
MINICPMO_API int minicpmo_gpu_context_matvec_q8_1(void *handle, const void *host_ptr, const void *xq, size_t in_dim, size_t out_dim,
                                     float *y_out, int32_t *dots_out, char *error, size_t error_cap);
/* Batched projection on the tensor cores (the decode path of
 * minicpmo_gpu_context_qwen3_forward_batch): y[n][out_dim] = W . x[n] for
 * n_seq <= 32 host f32 rows x[n][in_dim], W an uploaded Q8_0 tensor with
 * out_dim % 128 == 0 and in_dim % 256 == 0.  W and x are rounded to f16
 * and the products summed in f32.  No reference counterpart (the
 * reference has no GPU Q8_0 path, gpu.uya:130-132; its CPU path is
 * qwen3_q8_0_matvec_range, qwen3.uya:1200-1231). */
MINICPMO_API int minicpmo_gpu_context_matmul_q8_0_batch(void *handle, const void *host_ptr, const float *x, size_t n_seq,
                                           size_t in_dim, size_t out_dim, float *y_out, char *error,
                                           size_t error_cap);
/* Mean device time (us) of the tensor-core projection of an uploaded Q8_0
 * tensor for n_seq sequences, over `iters` launches with the L2 flushed
 * (a 256 MB write) before each, so every launch streams W from HBM. */
MINICPMO_API int minicpmo_gpu_context_time_matmul_q8_0_batch(void *handle, const void *host_ptr, size_t n_seq, int iters,
                                                float *avg_us, char *error, size_t error_cap);
/* GEMV of an uploaded quantised tensor on host f32 activations that the
 * GEMV kernel quantises to Q8_1 itself (as the decode step's fused down and
 * o projections do), after RMSNorm with the uploaded weight norm_host_ptr
 * (eps) when that is not NULL (as the fused q/k/v, gate/up and lm_head
 * GEMVs do).  Same bits as rms_norm_q8_1 / q8_1_quantize then matvec_q8_1. */
MINICPMO_API int minicpmo_gpu_context_matvec_f32_input(void *handle, const void *host_ptr, const float *x,
                                          const void *norm_host_ptr, float eps, size_t in_dim, size_t out_dim,
                                          float *y_out, char *error, size_t error_cap);
/* Runs the GEMV of an uploaded tensor `iters` times back to back on
 * device-resident activations and reports the mean kernel time (CUDA
 * events on the context stream). */
MINICPMO_API int minicpmo_gpu_context_time_matvec(void *handle, const void *host_ptr, size_t in_dim, size_t out_dim, int iters,
                                     float *avg_us, char *error, size_t error_cap);
/* time_matvec with the GEMV's input mode: 0 Q8_1 activations (as
 * time_matvec), 1 f32 activations quantised to Q8_1 in the GEMV's prologue,
 * 2 RMSNorm(f32) with the uploaded weight norm_host_ptr (eps 1e-6), then
 * quantised in the prologue (the fused producers of the decode step). */
MINICPMO_API int minicpmo_gpu_context_time_matvec_input(void *handle, const void *host_ptr, size_t in_dim, size_t out_dim,
                                           int iters, int input, const void *norm_host_ptr, float *avg_us,
                                           char *error, size_t error_cap);
/* Device time of the bound model's fused ffn gate/up GEMV exactly as the
 * decode step launches it (RMSNorm prologue from the current hidden state,
 * SwiGLU epilogue, Q8_1 output for the down GEMV; programmatic dependent
 * launch), back to back over the layers in turn (every launch streams its
 * weights from HBM): the average microseconds per launch and the
 * algorithmic bytes of one launch.  Overwrites only scratch activations. */
MINICPMO_API int minicpmo_gpu_context_qwen3_time_ffn(void *handle, int iters, float *avg_us, double *bytes_per_launch,
                                                     char *error, size_t error_cap);
/* Device time of n_steps auto-advancing decode steps (graph replays, no host
 * copies); reports the total milliseconds. */
MINICPMO_API int minicpmo_gpu_context_qwen3_time_decode(void *handle, uint32_t first_token, size_t first_pos, size_t n_steps,
                                           float *total_ms, char *error, size_t error_cap);
/* Kernel launches in one decode step's graph (with or without the lm_head
 * and sampler); 0 when no model is bound. */
MINICPMO_API int minicpmo_gpu_context_qwen3_step_kernels(void *handle, int with_logits);
/* Prefill passes so far (qwen3_prefill) whose projections ran on the tensor
 * cores, and in *gemv_passes (may be NULL) those that ran through the
 * multi-vector GEMVs; -1 when no model is bound. */
MINICPMO_API long long minicpmo_gpu_context_qwen3_prefill_passes(void *handle, long long *gemv_passes);
/* With MCPO_STEP_TRACE=1 in the environment at bind time, the persistent
 * step kernel records per stage and CTA the globaltimer (ns) at the start of
 * the stage, when the activations are ready (GEMV stages) and when all of the
 * CTA's warps are done; this copies the last step's record,
 * [stage][cta][start, ready, end], into out (cap entries).  0 when tracing
 * is off. */
MINICPMO_API int minicpmo_gpu_context_qwen3_step_trace(void *handle, uint64_t *out, size_t cap, uint32_t *n_stages,
                                          uint32_t *n_ctas);
/* In a library built with TRACE=1 (make -C minicpm-o-uya_b200/csrc TRACE=1;
 * the default build compiles the timeline out), with MCPO_GRAPH_TRACE=1 in
 * the environment at bind time, the per-operation decode step records per
 * launch and CTA the globaltimer (ns)
 * at the CTA's start, past its wait for the previous kernel, when its
 * activations are ready (attention: when its round of blocks begins) and
 * when it is done (attention also: its blocks done, past its cluster
 * barrier); launches in order q/k/v, attention, o, gate/up, down per layer,
 * then the lm_head.  This copies the last step's record, [launch][cta][8]
 * (zeros where nothing was recorded), into out (cap entries).  0 when
 * tracing is off. */
MINICPMO_API int minicpmo_gpu_context_qwen3_graph_trace(void *handle, uint64_t *out, size_t cap, uint32_t *n_launches,
                                           uint32_t *n_ctas);
/* Bytes of device memory held by the uploaded copy of a tensor. */
MINICPMO_API size_t minicpmo_gpu_context_tensor_device_bytes(void *handle, const void *host_ptr);

/* ---- allocation-free decode attention (no reference counterpart) ---- */

/* Limits of the fixed scratch the entry below uses instead of allocating:
 * at most 1024 KV heads, and head_count x ceil(context_capacity / 32) x
 * (head_dim + 4) x 4 bytes of per-block partial sums at most 2 MiB (Qwen3-8B's
 * 32 heads with head_dim 128 fit a 3968-position cache; Qwen3-32B's 64 heads
 * a 1984-position one).  Larger shapes are rejected with an error. */
#define MINICPMO_NOALLOC_MAX_KV_HEADS 1024
#define MINICPMO_NOALLOC_PARTIAL_BYTES (2u << 20)

/* The decode attention of minicpmo_gpu_context_attention over caller-owned
 * DEVICE buffers (q, one layer's K/V cache [context_capacity][kv_heads *
 * head_dim], f32 or f16 when kv_f16, 16-byte aligned, rows 0..pos filled; dst receives
 * head_count * head_dim floats), enqueued on `stream` (a cudaStream_t, NULL
 * for the legacy stream) without waiting for it.  No context, and no device
 * memory is allocated: for callers that cannot allocate while they run (a
 * serving loop that has reserved all memory up front, a host whose device
 * memory belongs to its own pool), because cudaMalloc can synchronise the
 * device and fail late.  The split-K scratch is one static device array per
 * device (limits above).  Set-up happens on the first call made with a given
 * device current (the symbol's address and the kernels' shared-memory
 * opt-in); make that first call before any stream capture.  Each call clears
 * the split counters and an error word on `stream` before launching.  Calls
 * that overlap on the GPU (other streams, other host threads) share the
 * scratch and race: serialise them.  head_count must be a multiple of
 * kv_head_count (at most 8 heads per kv head).  Returns 1, or 0 with a
 * message in `error`; the checks are on the host, before any CUDA call.  The
 * call is asynchronous: a bounded wait inside the kernel that gives up (only
 * a fault elsewhere on the device makes one) is recorded in the scratch's
 * error word but not reported back, and the output of that call is then
 * undefined. */
MINICPMO_API int minicpmo_gpu_attention_no_alloc(const float *q, const void *k_cache, const void *v_cache, int kv_f16,
                                    size_t pos, size_t head_count, size_t kv_head_count, size_t head_dim,
                                    size_t context_capacity, float *dst, void *stream, char *error, size_t error_cap);

#ifdef __cplusplus
}
#endif
#endif
