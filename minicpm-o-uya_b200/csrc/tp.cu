// tp.cu -- tensor-parallel exchange kernels (see tp.cuh).
//
// Protocol per exchange: every rank runs the same sequence of exchanges, so
// a per-rank epoch counter (advanced by each exchange kernel) names the
// exchange.  A kernel first publishes its epoch with a system-scope release
// store to its own flag (the partials it publishes were written by earlier
// kernels of the same stream), then acquires every peer's flag, bounded by
// 1 s of globaltimer; peer data is read with uncached loads.  Two partial
// buffers alternate per exchange: a rank writes buffer b for exchange e+2
// only after exchange e+1, which every peer entered after finishing its reads
// of exchange e.
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

__global__ void __launch_bounds__(1024) k_tp_reduce_add(const TpPeers p, int buf, float* hidden, int n,
                                                        unsigned* epoch, int* err) {
  __shared__ unsigned e_s;
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) {
    const unsigned e = *epoch + 1u;
    ok_s = publish_and_wait(p, e) ? 1 : 0;
    e_s = e;
    if (!ok_s) atomicExch(err, 1);
  }
  __syncthreads();
  if (ok_s) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float t = __ldcv(p.part[0][buf] + i);
      for (int r = 1; r < p.world; ++r) t = __fadd_rn(t, __ldcv(p.part[r][buf] + i));
      hidden[i] = __fadd_rn(hidden[i], t);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *epoch = e_s;  // advanced even on a timeout: the error word ends the run
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

cudaError_t launch_tp_reduce_add(const TpPeers& p, int buf, float* hidden, int n, unsigned* epoch, int* err,
                                 cudaStream_t st) {
  if (p.world < 1 || p.world > kTpMaxWorld || buf < 0 || buf > 1) return cudaErrorInvalidValue;
  return launch_k(k_tp_reduce_add, dim3(1), dim3(1024), 0, st, true, p, buf, hidden, n, epoch, err);
}

cudaError_t launch_tp_sample_merge(const TpPeers& p, StepState* st, int* history, int history_cap, unsigned* epoch,
                                   int* err, cudaStream_t s) {
  if (p.world < 1 || p.world > kTpMaxWorld) return cudaErrorInvalidValue;
  return launch_k(k_tp_sample_merge, dim3(1), dim3(32), 0, s, true, p, st, history, history_cap, epoch, err);
}

}  // namespace mcpo
