// gemm_plan.h - host-side tile/split planning for the tcgen05 GEMM core.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace pgb {

struct GemmPlan {
  bool swap;     // true: MMA M side = output features (decode)
  int bn;        // MMA N (32, 64, 128 or 256)
  int kblocks;   // ceil(K / 64)
  int splits;    // K splits per tile
  int p_tiles;
  int q_tiles;
  int units;     // p_tiles * q_tiles * splits
  int grid;      // persistent CTAs
  size_t partial_bytes;  // split-K scratch (0 when splits == 1)
  size_t counter_bytes;  // tile counters (aligned)
};

// Plan y[T, N] = x[T, K] . W[N, K]^T on a device with `sms` SMs.
// max_partial_bytes caps the split-K scratch (SIZE_MAX: no cap).
GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_partial_bytes);

// Scratch layout used by the column GEMM: [status word | counters | partials].
constexpr size_t kWsHeaderBytes = 256;
inline size_t col_workspace_bytes(const GemmPlan& p) {
  return kWsHeaderBytes + p.counter_bytes + p.partial_bytes;
}

}  // namespace pgb
