// noalloc.cu -- decode attention over caller-owned device buffers, with its
// split-K scratch in a fixed static device array instead of allocated memory.
//
// For hosts that must not allocate device memory while they run: a serving
// loop that has already reserved all of its memory, a caller inside a
// memory-pool arena, or a process that allocates only before it starts.
// cudaMalloc may synchronise the device and fail late under memory
// pressure; this entry calls no allocator (neither CUDA's nor any library's).
//
// Set-up happens on the first call made while a device is current, once per
// device: cudaGetSymbolAddress for that device's copy of the scratch array
// and the kernels' shared-memory opt-in.  Make that first call before any
// stream capture.  Every call clears the split counters (they must start at
// zero) and the error word with one asynchronous memset on the caller's
// stream, then launches.  A bounded wait inside the kernel that gives up
// (only a fault elsewhere on the device makes one) raises that error word;
// the call has returned by then, so it is not reported to the caller, and
// the output of such a call is undefined.
// The scratch is one array per device, so calls that overlap on the GPU
// (two streams, or two host threads) race on it; serialise them.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "attention.cuh"
#include "common.cuh"
#include "minicpmo_gpu.h"

namespace mcpo {
namespace {

constexpr size_t kCounterBytes = (size_t)MINICPMO_NOALLOC_MAX_KV_HEADS * 4;
constexpr size_t kErrBytes = 256;  // the kernel's error word, padded to keep the partials 256-byte aligned
constexpr size_t kPartialBytes = (size_t)MINICPMO_NOALLOC_PARTIAL_BYTES;
constexpr int kMaxDevices = 64;

// [counters: MAX_KV_HEADS x u32][error word, padded][partial sums: PARTIAL_BYTES]
static __device__ __align__(256) unsigned char g_attn_scratch[kCounterBytes + kErrBytes + kPartialBytes];

std::mutex g_setup_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {};

int put_error(char* err, size_t cap, const char* fmt, ...) {
  if (err && cap) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, cap, fmt, ap);
    va_end(ap);
  }
  return 0;
}

// The scratch address for the current device, set up on first use.
unsigned char* scratch_for_current_device(char* err, size_t cap) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return put_error(err, cap, "error: no_alloc attention: cudaGetDevice: %s", cudaGetErrorString(e)), nullptr;
  if (dev < 0 || dev >= kMaxDevices)
    return put_error(err, cap, "error: no_alloc attention: device %d beyond %d", dev, kMaxDevices), nullptr;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_ptr[dev]) return g_scratch_ptr[dev];
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_attn_scratch);
  if (e != cudaSuccess || !p)
    return put_error(err, cap, "error: no_alloc attention: cudaGetSymbolAddress: %s", cudaGetErrorString(e)), nullptr;
  e = attention_init();
  if (e != cudaSuccess)
    return put_error(err, cap, "error: no_alloc attention: kernel set-up: %s", cudaGetErrorString(e)), nullptr;
  g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
  return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace mcpo

using namespace mcpo;

extern "C" int minicpmo_gpu_attention_no_alloc(const float* q, const void* k_cache, const void* v_cache, int kv_f16,
                                               size_t pos, size_t head_count, size_t kv_head_count, size_t head_dim,
                                               size_t context_capacity, float* dst, void* stream, char* error,
                                               size_t error_cap) {
  if (!q || !k_cache || !v_cache || !dst) return put_error(error, error_cap, "error: no_alloc attention: null buffer");
  if (head_count == 0 || kv_head_count == 0 || head_dim == 0 || context_capacity == 0)
    return put_error(error, error_cap, "error: no_alloc attention: zero dimension");
  if (!(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim <= 32))
    return put_error(error, error_cap, "error: no_alloc attention: head_dim must be 64, 128, 256 or <= 32 (got %zu)",
                     head_dim);
  if (head_count < kv_head_count)
    return put_error(error, error_cap, "error: no_alloc attention: %zu heads fewer than %zu kv heads", head_count,
                     kv_head_count);
  if (head_count % kv_head_count != 0 || head_count / kv_head_count > 8)
    return put_error(error, error_cap, "error: no_alloc attention: %zu heads over %zu kv heads (need a group of <= 8)",
                     head_count, kv_head_count);
  if (pos >= context_capacity || context_capacity > 2147483647u)
    return put_error(error, error_cap, "error: no_alloc attention: pos %zu outside context %zu", pos, context_capacity);
  if (kv_head_count > (size_t)MINICPMO_NOALLOC_MAX_KV_HEADS)
    return put_error(error, error_cap, "error: no_alloc attention: %zu kv heads exceed the limit of %d", kv_head_count,
                     MINICPMO_NOALLOC_MAX_KV_HEADS);
  const int n_split = attn_n_split((int)kv_head_count);
  const int n_blocks = attn_n_blocks((int)context_capacity);
  const size_t need = attn_partial_floats((int)head_count, n_blocks, (int)head_dim) * 4;
  if (need > kPartialBytes)
    return put_error(error, error_cap,
                     "error: no_alloc attention: needs %zu scratch bytes (%zu heads x %d blocks of 32 positions x %zu), "
                     "limit %zu",
                     need, head_count, n_blocks, (size_t)attn_part_stride((int)head_dim) * 4, kPartialBytes);

  if (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15)
    return put_error(error, error_cap, "error: no_alloc attention: K/V caches must be 16-byte aligned");
  unsigned char* scratch = scratch_for_current_device(error, error_cap);
  if (!scratch) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned* counters = reinterpret_cast<unsigned*>(scratch);
  int* err_word = reinterpret_cast<int*>(scratch + kCounterBytes);
  cudaError_t e = cudaMemsetAsync(counters, 0, kCounterBytes + sizeof(int), st);
  if (e != cudaSuccess) return put_error(error, error_cap, "error: no_alloc attention: counter clear: %s", cudaGetErrorString(e));

  AttnArgs a{};
  a.q = q;
  a.fuse_norm_rope_append = 0;
  a.k_cache = const_cast<void*>(k_cache);
  a.v_cache = const_cast<void*>(v_cache);
  a.kv_f16 = kv_f16 ? 1 : 0;
  a.pos_ptr = nullptr;
  a.pos_static = (int)pos;
  a.n_head = (int)head_count;
  a.n_kv = (int)kv_head_count;
  a.head_dim = (int)head_dim;
  a.ctx = (int)context_capacity;
  a.n_split = n_split;
  a.scale = 1.0f / sqrtf((float)head_dim);
  a.partial = reinterpret_cast<float*>(scratch + kCounterBytes + kErrBytes);
  a.counters = counters;
  a.out = dst;
  a.out_q8 = nullptr;
  a.err = err_word;
  e = launch_attention(a, st);
  if (e != cudaSuccess) return put_error(error, error_cap, "error: no_alloc attention: launch: %s", cudaGetErrorString(e));
  return 1;
}
