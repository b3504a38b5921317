// tp_protocol_harness.cpp -- the tensor-parallel exchange protocol of the
// decode step (minicpm-o-uya_b200/csrc/tp_proto.h, the same header the CUDA
// kernels use) run by host threads over shared memory.  TEST CODE: built by
// tests/test_tp_host.py with the host compiler.
//
// Each of `world` threads plays a rank.  Per step it runs `nx` exchanges:
// it stores its partial vector, every value with the exchange's tag in one
// 64-bit word, into its slot of every rank's buffer (the slot of the
// exchange's parity), then waits (bounded) value by value for every rank's
// word to carry the tag and checks the rank-order sum value by value.  The
// words are written and read with relaxed 64-bit atomics, as the kernels'
// st/ld.relaxed.sys: no fence or release orders them.  A rank can be
// "killed" at the start of a step (it leaves between steps, as a crashed
// process would); the others must then give up after the wait limit and
// report the error instead of hanging.
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <random>
#include <thread>
#include <vector>

#include "tp_proto.h"

using namespace mcpo;

namespace {

struct RankBuf {
  std::unique_ptr<std::atomic<uint64_t>[]> part;  // [2][kTpMaxWorld][rows] tagged words
};

uint32_t bits_of(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  return b;
}

float float_of(uint32_t b) {
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

float value(int rank, uint32_t index, int i) {
  // distinct per (rank, exchange, element), exact in f32
  return (float)((rank + 1) * 1000 + (int)(index % 977u)) + (float)(i % 64) * 0.25f;
}

uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

}  // namespace

// Steps first_step .. first_step + steps - 1 (a large first_step runs the
// exchange index, and with it the tag, across its wraparound).
extern "C" int tp_harness_run(int world, unsigned first_step, int steps, int nx, int rows, int kill_rank,
                              int kill_step, unsigned long long limit_ns, int max_skew_us, unsigned seed, int* status,
                              int* mismatches) {
  if (world < 1 || world > kTpMaxWorld || nx < 2 || (nx & 1) || rows < 1 || steps < 1 || first_step < 1) return 0;
  std::vector<RankBuf> buf(world);
  const size_t words = (size_t)2 * kTpMaxWorld * rows;
  for (auto& b : buf) {
    b.part.reset(new std::atomic<uint64_t>[words]);
    for (size_t i = 0; i < words; ++i) b.part[i].store(0);
  }
  auto slot = [&](int dst, int par, int src) { return &buf[dst].part[((size_t)par * kTpMaxWorld + src) * rows]; };
  std::vector<std::thread> th;
  for (int r = 0; r < world; ++r) {
    status[r] = -1;
    mismatches[r] = 0;
    th.emplace_back([&, r] {
      std::mt19937 rng(seed * 131u + (unsigned)r);
      std::uniform_int_distribution<int> skew(0, max_skew_us);
      for (int k = 0; k < steps; ++k) {
        const uint32_t step = first_step + (uint32_t)k;
        if (r == kill_rank && k + 1 == kill_step) {
          status[r] = 2;
          return;
        }
        for (int x = 0; x < nx; ++x) {
          const uint32_t index = tp_exchange_index(step, (uint32_t)nx, (uint32_t)x);
          const int par = tp_parity(index);
          const uint32_t tag = tp_tag(index);
          for (int d = 0; d < world; ++d) {
            std::atomic<uint64_t>* s = slot(d, par, r);
            for (int i = 0; i < rows; ++i)
              s[i].store(tp_ll_pack(bits_of(value(r, index, i)), tag), std::memory_order_relaxed);
          }
          if (max_skew_us > 0) std::this_thread::sleep_for(std::chrono::microseconds(skew(rng)));
          const uint64_t deadline = now_ns() + limit_ns;
          bool ok = true;
          for (int i = 0; i < rows && ok; ++i) {
            const float base = (float)(i % 7);
            const float got = tp_rank_sum(base, world, [&](int src) {
              return float_of(tp_ll_wait(
                  reinterpret_cast<const uint64_t*>(slot(r, par, src) + i), tag,
                  [](const uint64_t* p) {
                    return reinterpret_cast<const std::atomic<uint64_t>*>(p)->load(std::memory_order_relaxed);
                  },
                  now_ns, deadline, &ok));
            });
            const float want = tp_rank_sum(base, world, [&](int src) { return value(src, index, i); });
            if (ok && std::memcmp(&got, &want, sizeof(float)) != 0) ++mismatches[r];
          }
          if (!ok) {
            status[r] = 1;
            return;
          }
        }
      }
      status[r] = 0;
    });
  }
  for (auto& t : th) t.join();
  return 1;
}
