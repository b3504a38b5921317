// gemm.cu -- batched decode projections (config: all linear weights Q8_0,
// up to 32 independent sequences) on the sm_100a tensor cores (tcgen05).
//
// Batch-1 decode is a weight stream and runs on dp4a (gemv.cu); with 32
// sequences the same stream carries 32x the arithmetic, which dp4a cannot
// keep up with, so the weights are dequantised to f16 into tensor memory and
// multiplied on the tensor cores with f32 accumulation in tensor memory:
//
//   warp 0      weight producer: per 256-value K-tile, one bulk copy of the
//               tile's Q8_0 bytes (the weights are re-tiled at upload so
//               that the 128 rows x 8 blocks of a (row tile, K-tile) pair
//               are one 34816-byte block), started before the dependency
//               wait (the weights do not depend on the previous kernel);
//   warp 21     activation producer: per K-tile one bulk copy of the f16
//               activation tile (N x 256, already in the operand layout),
//               after the dependency wait;
//   warps 5..20 dequantise: thread = (row, quarter of the K-tile), q * d in
//               f16 (int8 -> f16 exactly via the 0x6400 exponent trick, one
//               rounding in the multiply), stored into the A stage in tensor
//               memory (lane = row, tcgen05.st) -- no shared-memory operand;
//   warps 1..4  MMA issue, one elected thread per warp and quarter q of
//               every K-tile: tcgen05.mma kind::f16 (M = 128, N = sequences,
//               K = 16) with A read from tensor memory, into the quarter's
//               own 128 x N f32 accumulator in tensor memory; stages are
//               released with tcgen05.commit.  A thread's MMAs follow one
//               another about 230 cycles apart at any N (measured on the
//               B200), while MMAs issued by different warps overlap, so four
//               issuers carry four times the MMA rate of one;
//   epilogue    warps 5..20 read the four accumulators with tcgen05.ld (lane
//               = row, each warp a quarter of the sequence columns), add them
//               in quarter order and store / add Y, or, with K split over
//               several CTAs, write partial sums that the last CTA of the row
//               tile adds in split order (deterministic).
//
// All waits are bounded (mbarrier try_wait with an iteration limit); a wait
// that gives up raises the error word and a shared abort flag, the other
// roles stop at their next wait, and the CTA still waits (bounded) for its
// copies and MMAs in flight before it frees tensor memory and exits.
//
// Arithmetic: the result differs from the reference's f32-activation CPU
// path (qwen3.uya:1200-1231) by the f16 rounding of the dequantised weights
// and of the activations (relative 2^-11 each), far inside the 1e-3 matvec
// tolerance.
#include "gemm.cuh"

#include <cuda_fp16.h>
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "gemv.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace mcpo {

namespace {

constexpr int kRawStages = 4;   // Q8_0 weight tiles in flight
constexpr int kActStages = 4;   // f16 activation tiles in flight
constexpr int kAStages = 8;     // f16 operand quarter-tiles (128 rows x 64 K) in tensor memory: two K-tiles
constexpr int kRowPiece = 272;  // bytes of 256 values of one Q8_0 row
constexpr int kRawBytes = kGemmTileRows * kRowPiece;     // 34816
constexpr int kIssuers = 4;   // MMA issuing warps, one per 64-value quarter of a K-tile
constexpr int kDqWarps = 16;  // dequantising / epilogue warps: 4 per quarter of a K-tile
constexpr int kDq0 = 1 + kIssuers;  // first dequantising warp
// the activation producer: a warp of its own, because a lane blocked in a
// wait (the dependency wait, an mbarrier try_wait) holds up the other
// divergent paths of its warp -- here the weight copies
constexpr int kActWarp = kDq0 + kDqWarps;
constexpr int kThreads = (kActWarp + 1) * 32;
// Tensor memory: one 128 x N f32 accumulator per issuer (quarter q's in
// columns [qN, qN + N)); A stage s (128 rows x 64 f16, two per 32-bit
// column) in columns [128 + 32s, 160 + 32s) -- quarter q of K-tile i in
// stage q + 4 (i & 1), so the dequantising warps run a K-tile ahead of the
// MMAs.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = kIssuers * kGemmMaxN;

__host__ __device__ constexpr size_t act_bytes(int N) { return (size_t)N * kGemmKTile * 2; }

// Shared memory: [raw stages][activation stages][barriers][tmem addr][abort]
struct GemmSmem {
  __host__ __device__ static size_t raw_off() { return 0; }
  __host__ __device__ static size_t act_off() { return raw_off() + (size_t)kRawStages * kRawBytes; }
  __host__ __device__ static size_t bar_off(int N) { return act_off() + (size_t)kActStages * act_bytes(N); }
  __host__ __device__ static size_t bytes(int N) {
    return bar_off(N) + 8 * (2 * kRawStages + 2 * kActStages + 2 * kAStages + 1) + 16 + 1024;
  }
};

// ---- tcgen05 primitives (the shared ones are in tcgen05.cuh) ----

// Instruction descriptor for kind::f16: f16 A and B (K-major), f32
// accumulator, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kGemmTileRows >> 4) << 24);
}

// D (+)= A * B with A (128 x 16 f16, lane = row) in tensor memory at tmem_a.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit tensor-memory columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }






// NC (4 or 8) consecutive f32 accumulator columns of this thread's lane.
template <int NC>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, float (&v)[NC]) {
  static_assert(NC == 4 || NC == 8, "4 or 8 columns");
  uint32_t r[NC];
  if constexpr (NC == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
  } else {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < NC; ++i) v[i] = __uint_as_float(r[i]);
}

// Two signed bytes (positions 0,1 or 2,3 of w, already xor 0x80) as f16x2
// exactly: 0x6400 | u is 1024 + u, minus 1152 gives u - 128 = q.
__device__ __forceinline__ __half2 q8x2_to_h2(uint32_t wx, uint32_t sel) {
  const uint32_t b = __byte_perm(wx, 0x64646464u, sel);
  __half2 h;
  memcpy(&h, &b, 4);
  return __hsub2(h, __float2half2_rn(1152.0f));
}

// Row r's 64 values [64qt, 64qt + 64) of the staged K-tile (Q8_0 blocks
// 2qt, 2qt+1: 17 words at [qt][i][r]) -> 32 words of two f16 values in K
// order (word c holds values 2c, 2c+1).
__device__ __forceinline__ void dequant_quarter(const uint8_t* raw, uint32_t (&outw)[32], int r, int qt) {
  uint32_t w[17];
  const uint32_t* src = reinterpret_cast<const uint32_t*>(raw) + (size_t)qt * 17 * kGemmTileRows + r;
#pragma unroll
  for (int i = 0; i < 17; ++i) w[i] = src[(size_t)i * kGemmTileRows];
  // block scales (bytes 0-1 and 34-35) before the sign flip of the quants
  __half2 d2[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int db = 34 * j;
    const uint16_t dbits = (uint16_t)((w[db >> 2] >> (8 * (db & 3))) & 0xffffu);
    __half d;
    memcpy(&d, &dbits, 2);
    d2[j] = __half2half2(d);
  }
#pragma unroll
  for (int i = 0; i < 17; ++i) w[i] ^= 0x80808080u;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int db = 34 * j;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int b = db + 2 + 8 * c + 2 * p;  // first byte of the pair (even, same word as b+1)
        const __half2 v = __hmul2(q8x2_to_h2(w[b >> 2], (b & 3) ? 0x4342u : 0x4140u), d2[j]);
        memcpy(&outw[(4 * j + c) * 4 + p], &v, 4);
      }
    }
  }
}

template <int N>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_q80(const GemmArgs a) {
  // The tensor-core operand tiles are addressed from a 1024-byte aligned
  // shared-memory base (the dynamic region itself is only guaranteed 16-byte
  // alignment when device code is linked separately); the launch reserves
  // the 1 KB of slack.
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* raw_st = smem + GemmSmem::raw_off();
  uint8_t* act_st = smem + GemmSmem::act_off();
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + GemmSmem::bar_off(N));
  uint64_t* raw_empty = raw_full + kRawStages;
  uint64_t* x_full = raw_empty + kRawStages;
  uint64_t* x_empty = x_full + kActStages;
  uint64_t* a_full = x_empty + kActStages;
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* acc_full = a_empty + kAStages;
  uint32_t* tmem_s = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_s + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int row0 = tile * kGemmTileRows;
  const int kt_total = a.K / kGemmKTile;
  const int kt0 = (int)((long long)split * kt_total / a.ksplit);
  const int kt1 = (int)((long long)(split + 1) * kt_total / a.ksplit);
  const int nkt = kt1 - kt0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kDqWarps);  // released by the dequantising warps
    }
    for (int i = 0; i < kActStages; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], kIssuers);  // released by the issuers' MMA commits
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&a_full[i], kDqWarps / 4);  // the four warps of one group
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(acc_full, kIssuers);
    *abort_s = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_s, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_s;

  if (warp == 0) {
    // ---- weight producer (lane 0): the weights do not depend on the
    // previous kernel, so it starts at once and runs ahead as far as its
    // ring allows; the activation tiles come from warp kActWarp after the
    // dependency wait, on a ring of their own.
    if (lane == 0) {
      // this row tile's block list in its segment
      int R = row0;
      const uint8_t* wseg = a.seg[0].w;
      if (a.nseg > 1 && R >= a.seg[0].rows) {
        R -= a.seg[0].rows;
        wseg = a.seg[1].w;
        if (a.nseg > 2 && R >= a.seg[1].rows) {
          R -= a.seg[1].rows;
          wseg = a.seg[2].w;
        }
      }
      const uint8_t* wtile = wseg + (size_t)(R / kGemmTileRows) * kt_total * kRawBytes;
      const uint64_t policy = l2_evict_first_policy();
      int issued = 0;
      for (int i = 0; i < nkt; ++i) {
        const int s = i % kRawStages;
        if (i >= kRawStages && !gwait(&raw_empty[s], (uint32_t)((i / kRawStages) - 1) & 1u, a.err, abort_s)) break;
        mbar_arrive_expect_tx(&raw_full[s], (uint32_t)kRawBytes);
        bulk_load_hint(raw_st + (size_t)s * kRawBytes, wtile + (size_t)(kt0 + i) * kRawBytes, kRawBytes, &raw_full[s],
                       policy);
        issued = i + 1;
      }
      for (int i = issued > kRawStages ? issued - kRawStages : 0; i < issued; ++i)
        if (!mbar_wait(&raw_full[i % kRawStages], (uint32_t)(i / kRawStages) & 1u, a.err)) break;
    }
    __syncwarp();
  } else if (warp == kActWarp) {
    if (lane == 0) {
      pdl_wait();
      int issued = 0;
      for (int i = 0; i < nkt; ++i) {
        const int s = i % kActStages;
        if (i >= kActStages && !gwait(&x_empty[s], (uint32_t)((i / kActStages) - 1) & 1u, a.err, abort_s)) break;
        mbar_arrive_expect_tx(&x_full[s], (uint32_t)act_bytes(N));
        bulk_load(act_st + (size_t)s * act_bytes(N), a.x + (size_t)(kt0 + i) * act_bytes(N), (uint32_t)act_bytes(N),
                  &x_full[s]);
        issued = i + 1;
      }
      for (int i = issued > kActStages ? issued - kActStages : 0; i < issued; ++i)
        if (!mbar_wait(&x_full[i % kActStages], (uint32_t)(i / kActStages) & 1u, a.err)) break;
    }
    __syncwarp();
  } else if (warp < kDq0) {
    // ---- MMA issuers: lane 0 of warp 1 + q issues quarter q of every K-tile ----
    if (lane == 0) {
      const int q = warp - 1;
      const uint32_t idesc = umma_idesc_f16(N);
      const uint32_t sbo = 128, lbo_b = (N / 8) * 128;
      const uint32_t acc = tmem + (uint32_t)(q * N);
      for (int i = 0; i < nkt; ++i) {
        const int s = i % kActStages;
        if (!gwait(&x_full[s], (uint32_t)(i / kActStages) & 1u, a.err, abort_s)) break;
        const int sa = q + 4 * (i & 1);
        if (!gwait(&a_full[sa], (uint32_t)(i >> 1) & 1u, a.err, abort_s)) break;
        tc_fence_after();
        const uint32_t a_tm = tmem + kTmemA + (uint32_t)sa * 32;  // 4 columns of K per 8 values
        const uint32_t b_base = smem_addr(act_st + (size_t)s * act_bytes(N)) + (uint32_t)(q * 8) * lbo_b;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t bd = umma_desc(b_base + kk * 2 * lbo_b, lbo_b, sbo);
          umma_f16_ts(acc, a_tm + (uint32_t)kk * 8, bd, idesc, (i | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&a_empty[sa]);
        umma_commit(&x_empty[s]);
      }
      // after every MMA issued, on every path: the epilogue reads the
      // accumulators (or, on abort, only waits) before tensor memory is freed
      umma_commit(acc_full);
    }
    __syncwarp();
  } else {
    // ---- dequantising warps, then the epilogue (waits warp-uniform).  Warp
    // w belongs to group h = (w-5)/4, which converts quarter h of every
    // K-tile (A stages h and h+4 alternate: while the tensor cores read one,
    // the group fills the other) for rows 32*(w%4) .. +31 (= its
    // tensor-memory lane quarter); in the epilogue it takes sequence columns
    // [h*N/4, h*N/4 + N/4).
    const int h = (warp - kDq0) >> 2;
    const int r = ((warp & 3) << 5) | lane;
    for (int i = 0; i < nkt; ++i) {
      const int s = i % kRawStages;
      if (!__all_sync(0xffffffffu, gwait(&raw_full[s], (uint32_t)(i / kRawStages) & 1u, a.err, abort_s))) break;
      bool ok = true;
      {
        const int qt = h, sa = qt + 4 * (i & 1);
        if (i > 1 && !__all_sync(0xffffffffu, gwait(&a_empty[sa], (uint32_t)(((i >> 1) - 1) & 1), a.err, abort_s))) {
          ok = false;
        } else {
          uint32_t aw[32];
          dequant_quarter(raw_st + (size_t)s * kRawBytes, aw, r, qt);
          tc_fence_after();  // after the MMAs that read this stage before (a_empty)
          tmem_st32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + kTmemA + (uint32_t)sa * 32, aw);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[sa]);
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[s]);
    }
    const bool go = __all_sync(0xffffffffu, mbar_wait(acc_full, 0u, a.err) && !*abort_s);
    tc_fence_after();
    constexpr int NH = N / 4;
    const int c0 = h * NH;
    float v[NH];
#pragma unroll
    for (int c = 0; c < NH; ++c) v[c] = 0.0f;
    if (go) {
      const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)c0;
#pragma unroll
      for (int q = 0; q < kIssuers; ++q) {
        float u[NH];
        tmem_ldn<NH>(taddr + (uint32_t)(q * N), u);
#pragma unroll
        for (int c = 0; c < NH; ++c) v[c] = q == 0 ? u[c] : __fadd_rn(v[c], u[c]);
      }
    }
    const int row = row0 + r;
    if (a.ksplit <= 1) {
      if (go)
#pragma unroll
        for (int n = 0; n < NH; ++n) {
          if (c0 + n < a.n_valid) {
            float* y = a.y + (size_t)(c0 + n) * a.ldy + row;
            *y = a.epi == kGemmAdd ? __fadd_rn(*y, v[n]) : v[n];
          }
        }
    } else {
      // partial sums, then the last CTA of this row tile adds them in split
      // order; the named barrier spans the epilogue warps on every path
      __shared__ unsigned ticket_s;
#pragma unroll
      for (int n = 0; n < NH; ++n) a.partial[((size_t)split * N + c0 + n) * a.rows_total + row] = v[n];
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kDqWarps * 32) : "memory");
      if (warp == kDq0 && lane == 0) ticket_s = atomicAdd(&a.counters[tile], 1u);
      asm volatile("bar.sync 1, %0;" ::"n"(kDqWarps * 32) : "memory");
      if (ticket_s == (unsigned)(a.ksplit - 1)) {
        __threadfence();
        // sums in split order; every split's values are loaded before the adds
        float sum[NH];
#pragma unroll
        for (int n = 0; n < NH; ++n) sum[n] = 0.0f;
        for (int sp = 0; sp < a.ksplit; ++sp) {
          float pv[NH];
#pragma unroll
          for (int n = 0; n < NH; ++n) pv[n] = __ldcg(a.partial + ((size_t)sp * N + c0 + n) * a.rows_total + row);
#pragma unroll
          for (int n = 0; n < NH; ++n) sum[n] = __fadd_rn(sum[n], pv[n]);
        }
#pragma unroll
        for (int n = 0; n < NH; ++n) {
          if (c0 + n < a.n_valid) {
            float* y = a.y + (size_t)(c0 + n) * a.ldy + row;
            *y = a.epi == kGemmAdd ? __fadd_rn(*y, sum[n]) : sum[n];
          }
        }
        if (warp == kDq0 && lane == 0) a.counters[tile] = 0u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- activation producers (f16 operand layout) ----

__global__ void k_pack_x16(const float* __restrict__ x, int ld, int n_valid, int K, int N, uint8_t* __restrict__ x16) {
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.y;
  if (n >= n_valid) return;
  for (int k = (blockIdx.x * blockDim.x + threadIdx.x) * 8; k < K; k += gridDim.x * blockDim.x * 8) {
    const float* src = x + (size_t)n * ld + k;
    uint32_t o[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const __half2 h = __floats2half2_rn(src[2 * p], src[2 * p + 1]);
      memcpy(&o[p], &h, 4);
    }
    *reinterpret_cast<uint4*>(x16 + gemm_x_offset(n, k, N)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// One CTA (256 threads) per sequence: sum of squares in the order of
// gpu_shim.c:694-718 (256 strided partial sums, halving tree), then
// x * inv * w into the operand layout.
__global__ void __launch_bounds__(256) k_rmsnorm_x16(const float* __restrict__ x, int ld, const void* __restrict__ w,
                                                     int w_dtype, int K, float eps, int N, uint8_t* __restrict__ x16) {
  __shared__ float part[256];
  __shared__ float inv_s;
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x, t = threadIdx.x;
  const float* xr = x + (size_t)n * ld;
  float p = 0.0f;
  for (int i = t; i < K; i += 256) p = __fadd_rn(p, __fmul_rn(xr[i], xr[i]));
  part[t] = p;
  __syncthreads();
  for (int stride = 128; stride >= 32; stride >>= 1) {
    if (t < stride) part[t] = __fadd_rn(part[t], part[t + stride]);
    __syncthreads();
  }
  if (t < 32) {
    float v = part[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
    if (t == 0) inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)K), eps)));
  }
  __syncthreads();
  const float inv = inv_s;
  for (int k = t * 8; k < K; k += 256 * 8) {
    uint32_t o[4];
#pragma unroll
    for (int p2 = 0; p2 < 4; ++p2) {
      const int i = k + 2 * p2;
      const float a0 = __fmul_rn(__fmul_rn(xr[i], inv), load_weight(w, w_dtype, i));
      const float a1 = __fmul_rn(__fmul_rn(xr[i + 1], inv), load_weight(w, w_dtype, i + 1));
      const __half2 h = __floats2half2_rn(a0, a1);
      memcpy(&o[p2], &h, 4);
    }
    *reinterpret_cast<uint4*>(x16 + gemm_x_offset(n, k, N)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void k_swiglu_x16(const float* __restrict__ gu, int F, int n_valid, int N, uint8_t* __restrict__ x16) {
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.y;
  if (n >= n_valid) return;
  const float* g = gu + (size_t)n * 2 * F;
  const float* u = g + F;
  for (int k = (blockIdx.x * blockDim.x + threadIdx.x) * 8; k < F; k += gridDim.x * blockDim.x * 8) {
    uint32_t o[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const __half2 h = __floats2half2_rn(silu_mul_det(g[k + 2 * p], u[k + 2 * p]),
                                          silu_mul_det(g[k + 2 * p + 1], u[k + 2 * p + 1]));
      memcpy(&o[p], &h, 4);
    }
    *reinterpret_cast<uint4*>(x16 + gemm_x_offset(n, k, N)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// GGUF Q8_0 rows [rows][K/32 * 34 bytes] -> one contiguous 34816-byte block
// per (row tile, K-tile), laid out [quarter 4][word 17][row 128] in 32-bit
// words: quarter qt of row r is the 68 bytes of Q8_0 blocks 2qt, 2qt+1 of
// that row's 256 values, and the 32 rows a warp converts together read
// consecutive words (no shared-memory bank conflicts).  One thread per word.
__global__ void k_gemm_tile_weights(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows, int K) {
  const int kt_total = K / kGemmKTile;
  const size_t row_bytes = (size_t)(K / 32) * 34;
  const size_t nwords = (size_t)rows * row_bytes / 4;
  constexpr int kBlockWords = kRawBytes / 4;  // 8704
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < nwords; e += (size_t)gridDim.x * blockDim.x) {
    const size_t blk = e / kBlockWords;
    const int within = (int)(e % kBlockWords);
    const int qt = within / (17 * kGemmTileRows);
    const int i = (within / kGemmTileRows) % 17;
    const int r = within % kGemmTileRows;
    const size_t tile = blk / kt_total, kt = blk % kt_total;
    const uint8_t* p = src + (tile * kGemmTileRows + r) * row_bytes + kt * kRowPiece + (size_t)qt * 68 + (size_t)i * 4;
    uint32_t w;
    memcpy(&w, p, 4);  // 4-byte aligned: row_bytes, 272 and 68 are multiples of 4
    reinterpret_cast<uint32_t*>(dst)[e] = w;
  }
}

}  // namespace

cudaError_t launch_gemm_tile_weights(const uint8_t* src, uint8_t* dst, int rows, int K, cudaStream_t st) {
  if (rows <= 0 || rows % kGemmTileRows || K <= 0 || K % kGemmKTile) return cudaErrorInvalidValue;
  k_gemm_tile_weights<<<148 * 16, 256, 0, st>>>(src, dst, rows, K);
  return cudaGetLastError();
}

int gemm_pick_ksplit(int tiles, int ktiles, int sms) {
  // one CTA per SM: minimise waves x K-tiles per CTA (the critical path);
  // matrices with a wave of row tiles or more are not split (partial sums
  // would add traffic for nothing)
  if (tiles >= sms || sms <= 0) return 1;
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= 8 && s <= ktiles; ++s) {
    const long long waves = ((long long)tiles * s + sms - 1) / sms;
    const long long cost = waves * ((ktiles + s - 1) / s);
    if (best_cost < 0 || cost < best_cost) best_cost = cost, best = s;
  }
  return best;
}

cudaError_t gemm_init() {
  cudaError_t e = cudaFuncSetAttribute(k_gemm_q80<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)GemmSmem::bytes(16));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_gemm_q80<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GemmSmem::bytes(32));
  return e;
}

cudaError_t launch_gemm_q80(const GemmArgs& a, cudaStream_t st, bool pdl) {
  if (a.N != 16 && a.N != 32) return cudaErrorInvalidValue;
  if (a.K <= 0 || a.K % kGemmKTile || a.n_valid < 1 || a.n_valid > a.N || a.nseg < 1 || a.nseg > kGemmMaxSegs)
    return cudaErrorInvalidValue;
  int rows = 0;
  for (int i = 0; i < a.nseg; ++i) {
    if (a.seg[i].rows <= 0 || a.seg[i].rows % kGemmTileRows || !a.seg[i].w) return cudaErrorInvalidValue;
    rows += a.seg[i].rows;
  }
  if (rows != a.rows_total || a.ksplit < 1 || a.ksplit > a.K / kGemmKTile) return cudaErrorInvalidValue;
  if (a.ksplit > 1 && (!a.partial || !a.counters)) return cudaErrorInvalidValue;
  const dim3 grid(a.rows_total / kGemmTileRows, a.ksplit);
  if (a.N == 16) return launch_k(k_gemm_q80<16>, grid, dim3(kThreads), GemmSmem::bytes(16), st, pdl, a);
  return launch_k(k_gemm_q80<32>, grid, dim3(kThreads), GemmSmem::bytes(32), st, pdl, a);
}

cudaError_t launch_pack_x16(const float* x, int ld, int n_valid, int K, int N, uint8_t* x16, cudaStream_t st,
                            bool pdl) {
  if (K % 8 || n_valid > N) return cudaErrorInvalidValue;
  const int per = (K / 8 + 127) / 128;
  return launch_k(k_pack_x16, dim3(per < 1 ? 1 : per, n_valid), dim3(128), 0, st, pdl, x, ld, n_valid, K, N, x16);
}

cudaError_t launch_rmsnorm_x16(const float* x, int ld, const void* w, int w_dtype, int n_valid, int K, float eps,
                               int N, uint8_t* x16, cudaStream_t st, bool pdl) {
  if (K % 8 || n_valid > N) return cudaErrorInvalidValue;
  return launch_k(k_rmsnorm_x16, dim3(n_valid), dim3(256), 0, st, pdl, x, ld, w, w_dtype, K, eps, N, x16);
}

cudaError_t launch_swiglu_x16(const float* gu, int F, int n_valid, int N, uint8_t* x16, cudaStream_t st, bool pdl) {
  if (F % 8 || n_valid > N) return cudaErrorInvalidValue;
  const int per = (F / 8 + 127) / 128;
  return launch_k(k_swiglu_x16, dim3(per < 1 ? 1 : per, n_valid), dim3(128), 0, st, pdl, gu, F, n_valid, N, x16);
}

}  // namespace mcpo
