// tp.cu -- tensor-parallel exchange kernels and descriptors (see tp.cuh).
//
// The hidden-vector exchanges after the row-parallel o and down GEMVs are
// fused into those GEMVs (push epilogue) and the GEMV that consumes them
// (summing prologue); the protocol is in tp_proto.h.  What remains here:
// the step counter and the sampler merge.  The merge uses a flag per rank:
// a kernel publishes its epoch with a system-scope release store to its own
// flag, then acquires every peer's flag, bounded by 1 s of globaltimer; peer
// data is read with uncached loads.
#include "tp.cuh"

#include <math.h>

#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0: publish epoch e and wait for every peer's; false on timeout.
__device__ bool publish_and_wait(const TpPeers& p, unsigned e) {
  __threadfence_system();
  st_release_sys(p.flag[p.rank], e);
  const uint64_t t0 = gtimer();
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    unsigned it = 0;
    while (ld_acquire_sys(p.flag[r]) < e) {
      if ((++it & 255u) == 0 && (gtimer() - t0 > 1000000000ull || it > (1u << 24))) return false;
    }
  }
  return true;
}

// The consumer half of an exchange on its own (the step without an lm_head):
// thread 0 waits for every rank's partial, then out = base + rank-order sum.
__global__ void __launch_bounds__(1024) k_tp_finalize(const TpXchg t, const float* base, int* err) {
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) {
    const uint32_t target = tp_target(tp_exchange_index(*t.step, (uint32_t)t.nx, (uint32_t)t.x), (uint32_t)t.rows);
    ok_s = tp_wait_all(
        t.arrive, t.world, target, [](const uint32_t* p) { return ld_acquire_sys(p); }, [] { return gtimer(); },
        1000000000ull);
    if (!ok_s && err) atomicExch(err, 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < t.rows; i += blockDim.x)
    t.sum_out[i] = tp_rank_sum(base[i], t.world, [&](int r) { return __ldcv(t.src[r] + i); });
  pdl_launch_dependents();
}

__global__ void k_tp_step(unsigned* step) {
  pdl_wait();
  if (threadIdx.x == 0) *step = *step + 1u;
  pdl_launch_dependents();
}

__global__ void k_tp_sample_merge(const TpPeers p, StepState* st, int* history, int history_cap, unsigned* epoch,
                                  int* err) {
  pdl_wait();
  if (threadIdx.x != 0) return;
  const unsigned e = *epoch + 1u;
  *epoch = e;
  if (!publish_and_wait(p, e)) {
    atomicExch(err, 1);
    return;
  }
  // first max over ranks in rank (= index) order; the loser's best and every
  // rank's second feed the top-2 gap, as k_argmax's merge
  float b = -INFINITY, s = -INFINITY;
  int idx = 0x7fffffff;
  for (int r = 0; r < p.world; ++r) {
    const float rb = __ldcv(p.top[r]);
    const int ri = __float_as_int(__ldcv(p.top[r] + 1));
    const float rs = __ldcv(p.top[r] + 2);
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
  for (int d = 0; d < p.world; ++d) {
    t.dst[d] = reinterpret_cast<float*>(p.base[d] + TpLayout::part_offset(par, p.rank, (size_t)rows));
    t.dst_arrive[d] = reinterpret_cast<unsigned*>(p.base[d] + TpLayout::arrive_offset((size_t)rows)) + p.rank;
  }
  uint8_t* own = p.base[p.rank];
  for (int r = 0; r < p.world; ++r)
    t.src[r] = reinterpret_cast<const float*>(own + TpLayout::part_offset(par, r, (size_t)rows));
  t.arrive = reinterpret_cast<const unsigned*>(own + TpLayout::arrive_offset((size_t)rows));
  t.sum_out = sum_out;
  t.step = step;
  t.world = p.world;
  t.nx = nx;
  t.x = x;
  t.rows = rows;
  *out = t;
}

cudaError_t launch_tp_finalize(const TpXchg& t, const float* base, int* err, cudaStream_t st) {
  if (t.world < 1 || t.world > kTpMaxWorld || !t.sum_out || !t.step || !t.arrive) return cudaErrorInvalidValue;
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
