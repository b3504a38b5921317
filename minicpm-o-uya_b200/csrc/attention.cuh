// attention.cuh -- decode attention launch descriptor.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>


namespace mcpo {

struct AttnArgs {
  // inputs for the current position
  const float* q;  // [n_head*head_dim]
  const float* k;  // [n_kv*head_dim]
  const float* v;  // [n_kv*head_dim]
  // fused path: QK-RMSNorm (eps 1e-6) + NeoX RoPE + KV append before attention.
  int fuse_norm_rope_append;
  const void* q_norm; int q_norm_dtype;  // may be null
  const void* k_norm; int k_norm_dtype;  // may be null
  const float* rope_cos;                 // [rope_ctx][head_dim/2] or null
  const float* rope_sin;
  float rope_base, rope_scale;           // used when the tables are null
  // cache of this layer: [ctx][kv_dim], f32 or f16
  void* k_cache;
  void* v_cache;
  int kv_f16;
  const int* pos_ptr;  // device position (graph replay) or null
  int pos_static;
  int n_head, n_kv, head_dim, ctx;
  int n_split;  // CTAs per kv head (and sequence); CTA s takes blocks s, s + n_split, ...
  // 1: the CTAs of a kv head form one thread-block cluster and merge through
  // distributed shared memory (n_split <= kAttnMaxCluster, at most
  // kAttnMaxBlocksCta blocks per CTA; partial and counters unused); 0:
  // block partials in global memory, merged by the last-arriving CTA.  Same
  // arithmetic, same bits.
  int cluster;
  float scale;
  // scratch
  float* partial;      // [batch][n_head][attn_n_blocks(ctx)][attn_part_stride(head_dim)]: m, l, 2 pad, acc[head_dim]
  unsigned* counters;  // [batch][n_kv], zero at rest
  // outputs
  float* out;          // [n_head*head_dim]
  uint8_t* out_q8;     // optional Q8_1 of out (needs head_dim % 32 == 0)
  // independent sequences (grid z): sequence b reads q/k/v at + b*qkv_bstride
  // floats, its caches at + b*cache_bstride elements (0: every z reads the
  // same cache -- the tokens of one prompt, non-fused mode), its position at
  // pos_ptr[b * pos_stride] (pos_static when pos_ptr is null), and writes out at
  // + b*out_bstride floats and out_q8 at + b*outq8_bstride bytes.  batch 0
  // means 1.
  int batch;
  size_t qkv_bstride, cache_bstride, out_bstride, outq8_bstride;
  int pos_stride;  // ints between sequences' positions at pos_ptr (0: 1)
  int* err;        // raised by a bounded wait that gave up (may be null)
  // optional timeline (builds with MCPO_TRACE=1), [CTA (x fastest, then y,
  // z)][8] globaltimer ns: start, past the wait for the previous kernel, the
  // round of blocks begun, done, blocks done, past the cluster barrier, the
  // first round's tiles landed (1 unused)
  unsigned long long* trace;
};

constexpr int kAttnMaxCluster = 16;    // cluster size (beyond 8 needs the non-portable opt-in)
constexpr int kAttnMaxBlocksCta = 8;   // cluster path: blocks per CTA (partials kept in shared memory)

// Positions are attended in blocks of 32 (lane = position).
__host__ __device__ inline int attn_n_blocks(int ctx) { return (ctx + 31) / 32; }
// Floats per (head, block) partial: m, l, two pad floats, then head_dim
// accumulators (rows stay 16-byte aligned for bulk copies).
__host__ __device__ inline int attn_part_stride(int head_dim) { return head_dim + 4; }
size_t attn_partial_floats(int n_head, int n_blocks, int head_dim);
// One-time per-device setup (opts the kernels into their shared memory).
cudaError_t attention_init();
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl = false);

// Attention of T prompt tokens at positions pos[0..T) over a cache that
// already holds their K/V rows: per token the decode attention's arithmetic
// (same blocks, fma orders, softmax and block merge, so the same bits), but
// one CTA serves 8 tokens of a kv head and reads each K/V block once for
// them.  head_dim 64, 128 or 256.
struct PromptAttnArgs {
  const float* q;  // [T][q_stride], heads of head_dim after QK-norm and RoPE
  int q_stride;
  const void* k_cache;  // one layer's cache [ctx][n_kv*head_dim], f32 or f16
  const void* v_cache;
  int kv_f16;
  const int* pos;  // [T]
  int T;
  int n_head, n_kv, head_dim, ctx;
  float scale;
  float* partial;  // [T][n_head][attn_n_blocks(ctx)][attn_part_stride(head_dim)]
  float* out;      // [T][out_stride]
  int out_stride;
};
cudaError_t launch_prompt_attention(const PromptAttnArgs& a, cudaStream_t st);

}  // namespace mcpo
