// misc.cuh -- launchers for the small kernels of the decode step.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "layout.cuh"

namespace mcpo {

// Device-resident step state read by the captured decode graph.  The host
// writes token/pos before a replay (or sets auto_advance so the sampler
// feeds its own output back), the sampler writes next_token/best/gap.
struct StepState {
  int token;
  int pos;
  int next_token;
  float best;
  float gap;
  int auto_advance;
  float penalty;    // repeat penalty (<= 1: off)
  int history_len;  // tokens appended to the history buffer while auto-advancing
  int err;
  int embed_input;  // 1: this step's input row is the caller's embedding (k_embed copies it)
};

cudaError_t launch_relayout(const uint8_t* src, uint8_t* dst, const TileGeom& g, size_t row_bytes, cudaStream_t st);
// token (from tok_ptr when non-null) outside [0, rows) yields zeros.  batch
// sequences: sequence b's token at tok_ptr[b * tok_stride], its row at
// out + b * hidden.  in_flag (optional, single sequence): when *in_flag is
// nonzero the row is copied from in_row (hidden f32 values) instead.
cudaError_t launch_embed(const uint8_t* w, const TileGeom& g, int dtype, int rows, int hidden, const int* tok_ptr, int tok,
                         float* out, cudaStream_t st, bool pdl = false, int batch = 1, int tok_stride = 0,
                         const float* in_row = nullptr, const int* in_flag = nullptr);
// grid CTAs; scratch holds 3 floats per CTA; counter is zero at rest.
// history (may be null) receives next_token at history_len when auto-advancing.
// vocab_base/tp_top: a tensor-parallel vocab slice -- indices are offset by
// vocab_base and the result (best, index, second) goes to tp_top instead of st.
// batch > 1: independent sequences -- logits [batch][n], scratch
// [batch][grid*3], counter [batch], st [batch], history [batch][history_cap];
// no repeat penalty (seen_bits null) and no vocab slices.
cudaError_t launch_argmax(const float* logits, int n, const uint32_t* seen_bits, float* scratch, unsigned* counter,
                          StepState* st, int* history, int history_cap, int grid, cudaStream_t s, bool pdl = false,
                          int vocab_base = 0, float* tp_top = nullptr, int batch = 1);
cudaError_t launch_mark_seen(uint32_t* bits, const StepState* st, int vocab, cudaStream_t s, bool pdl = false);
// qwen3_sample (qwen3.uya:2073-2138) over vocab <= 256 logits; io[0] the
// xorshift32 state (in/out), io[1] the token.
cudaError_t launch_sample_small(const float* logits, int vocab, const uint32_t* seen, int seen_count, float temp,
                                uint32_t top_k, float top_p, float min_p, float penalty, uint32_t* io, cudaStream_t st);
// Prompt prefill: QK-RMSNorm + RoPE of n_tok tokens' q/k heads in place and
// the append of their k/v rows at positions pos[0..n_tok) of one layer's cache.
cudaError_t launch_prompt_qk(float* q, float* k, const float* v, int stride, int n_tok, int n_head, int n_kv, int hd,
                             const void* qn, int qndt, const void* kn, int kndt, const float* cos_t, const float* sin_t,
                             float base, float fscale, const int* pos, void* kc, void* vc, int kv_f16,
                             cudaStream_t st);
// bits |= the tokens of list (those < vocab).
cudaError_t launch_seen_bits(uint32_t* bits, const uint32_t* list, int n, int vocab, cudaStream_t st);
cudaError_t launch_add_inplace(float* dst, const float* src, int n, cudaStream_t st);
cudaError_t launch_silu_mul(float* dst, const float* gate, const float* up, int n, cudaStream_t st);
cudaError_t launch_head_norm_rope(float* vec, int n_head, int hd, const void* w, int w_dtype, int do_rope,
                                  const float* cos_t, const float* sin_t, float base, float fscale, int pos,
                                  cudaStream_t st);

}  // namespace mcpo
