// tp.cu -- tensor-parallel exchange kernels and descriptors (see tp.cuh).
//
// The hidden-vector exchanges after the row-parallel o and down GEMVs are
// fused into those GEMVs (push epilogue) and the GEMV that consumes them
// (summing prologue); the protocol is in tp_proto.h.  What remains here:
// the step counter, the consumer half of an exchange on its own, and the
// sampler merge, whose per-rank results travel as tagged words too (tag =
// the merge epoch), so no kernel here fences or waits on a flag.
#include "tp.cuh"

#include <math.h>

#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr uint64_t kTpWaitNs = 1000000000ull;

// The consumer half of an exchange on its own (the step without an lm_head):
// out = base + rank-order sum, each value once every rank's word of it has
// arrived.
__global__ void __launch_bounds__(1024) k_tp_finalize(const TpXchg t, const float* base, int* err) {
  pdl_wait();
  const uint32_t tag = tp_xchg_tag(t, *t.step);
  const uint64_t deadline = tp_now_ns() + kTpWaitNs;
  bool ok = true;
  // tp_rank_sum: base + (p_0 + ... + p_{world-1})
  tp_gather_sums(t, tag, threadIdx.x, blockDim.x, t.rows, deadline, &ok,
                 [&](int i, float s) { t.sum_out[i] = base[i] + s; });
  if (!ok && err) atomicExch(err, 1);
  pdl_launch_dependents();
}

__global__ void k_tp_step(unsigned* step) {
  pdl_wait();
  if (threadIdx.x == 0) *step = *step + 1u;
  pdl_launch_dependents();
}

// One warp.  Lane d < world sends this rank's sampler result (its own
// k_argmax wrote `top`) to rank d; lane r < world then waits for rank r's.
__global__ void k_tp_sample_merge(const TpPeers p, StepState* st, int* history, int history_cap, unsigned* epoch,
                                  int* err) {
  __shared__ float rb_s[kTpMaxWorld], rs_s[kTpMaxWorld];
  __shared__ int ri_s[kTpMaxWorld];
  pdl_wait();
  const int lane = threadIdx.x;
  const uint32_t e = tp_tag(*epoch);  // the merge's tag: epochs 0, 1, ... -> tags 1, 2, ...
  const float* own = p.top[p.rank];
  if (lane < p.world) {
    uint64_t* dst = p.merge[lane] + (size_t)p.rank * 4;
    for (int k = 0; k < 3; ++k) tp_st_word(dst + k, tp_ll_pack(__float_as_uint(own[k]), e));
  }
  bool ok = true;
  if (lane < p.world) {
    const uint64_t deadline = tp_now_ns() + kTpWaitNs;
    const uint64_t* src = p.merge[p.rank] + (size_t)lane * 4;
    uint32_t v[3];
    for (int k = 0; k < 3; ++k)
      v[k] = tp_ll_wait(src + k, e, [](const uint64_t* q) { return tp_ld_word(q); }, [] { return tp_now_ns(); },
                        deadline, &ok);
    rb_s[lane] = __uint_as_float(v[0]);
    ri_s[lane] = (int)v[1];
    rs_s[lane] = __uint_as_float(v[2]);
  }
  const bool all_ok = __all_sync(0xffffffffu, ok);
  __syncwarp();
  if (lane != 0) return;
  *epoch = *epoch + 1u;
  if (!all_ok) {
    atomicExch(err, 1);
    return;
  }
  // first max over ranks in rank (= index) order; the loser's best and every
  // rank's second feed the top-2 gap, as k_argmax's merge
  float b = -INFINITY, s = -INFINITY;
  int idx = 0x7fffffff;
  for (int r = 0; r < p.world; ++r) {
    const float rb = rb_s[r];
    const int ri = ri_s[r];
    const float rs = rs_s[r];
    const bool wins = rb > b || (rb == b && ri < idx);
    if (wins) {
      s = fmaxf(fmaxf(s, rs), b);
      b = rb;
      idx = ri;
    } else {
      s = fmaxf(fmaxf(s, rs), rb);
    }
  }
  if (idx == 0x7fffffff) {  // every logit NaN
    idx = 0;
    st->err = 1;
  }
  st->next_token = idx;
  st->best = b;
  st->gap = b - s;
  if (st->auto_advance) {
    if (history && st->history_len < history_cap) history[st->history_len] = idx;
    st->history_len = st->history_len + 1;
    st->token = idx;
    st->pos = st->pos + 1;
  }
}

}  // namespace

void tp_xchg(const TpPeers& p, int nx, int x, int rows, const unsigned* step, float* sum_out, TpXchg* out) {
  TpXchg t{};
  const int par = x & 1;
  for (int d = 0; d < p.world; ++d)
    t.dst[d] = reinterpret_cast<uint64_t*>(p.base[d] + TpLayout::part_offset(par, p.rank, (size_t)rows));
  uint8_t* own = p.base[p.rank];
  for (int r = 0; r < p.world; ++r)
    t.src[r] = reinterpret_cast<const uint64_t*>(own + TpLayout::part_offset(par, r, (size_t)rows));
  t.sum_out = sum_out;
  t.step = step;
  t.world = p.world;
  t.nx = nx;
  t.x = x;
  t.rows = rows;
  *out = t;
}

cudaError_t launch_tp_finalize(const TpXchg& t, const float* base, int* err, cudaStream_t st) {
  if (t.world < 1 || t.world > kTpMaxWorld || (t.world & (t.world - 1)) || !t.sum_out || !t.step || !t.src[0])
    return cudaErrorInvalidValue;
  return launch_k(k_tp_finalize, dim3(1), dim3(1024), 0, st, true, t, base, err);
}

cudaError_t launch_tp_step(unsigned* step, cudaStream_t st) {
  return launch_k(k_tp_step, dim3(1), dim3(32), 0, st, true, step);
}

cudaError_t launch_tp_sample_merge(const TpPeers& p, StepState* st, int* history, int history_cap, unsigned* epoch,
                                   int* err, cudaStream_t s) {
  if (p.world < 1 || p.world > kTpMaxWorld) return cudaErrorInvalidValue;
  return launch_k(k_tp_sample_merge, dim3(1), dim3(32), 0, s, true, p, st, history, history_cap, epoch, err);
}

}  // namespace mcpo
