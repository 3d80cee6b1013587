// gemm_plan.h - host-side tile and work-decomposition planning for the
// tcgen05 GEMM core.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace pgb {

struct GemmPlan {
  bool swap;      // true: MMA M side = output features (decode)
  int bn;         // MMA N (32, 64, 128 or 256)
  int kblocks;    // ceil(K / 64)
  int p_tiles;
  int q_tiles;
  int tiles;      // p_tiles * q_tiles
  int dp_rounds;  // whole tiles per CTA (round-robin part)
  int sk_first;   // first stream-K tile (== tiles: none)
  int grid;       // CTAs taking part in the GEMM
  int sk_grid;    // CTAs taking part in the stream-K part (<= its k-blocks)
  int max_contrib;        // partial slabs per stream-K tile
  size_t partial_bytes;   // partial scratch (0 without stream-K)
  size_t counter_bytes;   // tile counters (aligned)
};

// Plan y[T, N] = x[T, K] . W[N, K]^T on a device with `sms` SMs.
// max_partial_bytes caps the stream-K scratch (SIZE_MAX: no cap); a plan
// that would exceed it falls back to whole tiles. all_streamk puts every
// tile of a decode shape in the stream-K part (no round-robin whole tiles).
GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_partial_bytes, bool all_streamk = false);

// Scratch layout used by the column GEMM: [status word | counters | partials].
constexpr size_t kWsHeaderBytes = 256;
inline size_t col_workspace_bytes(const GemmPlan& p) {
  return kWsHeaderBytes + p.counter_bytes + p.partial_bytes;
}

}  // namespace pgb
