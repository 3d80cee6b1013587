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
  int dp_rounds;  // rounds of whole tiles [0, split_first), round-robin over `grid` CTAs
  int split_first;  // first split tile (== tiles: none)
  int grid;       // CTAs that take work (the launch may be wider)
  int split_ctas; // CTAs [0, split_ctas) take one split segment after their whole tiles
  int nsplit;     // k-ranges per split tile (1: no split tiles)
  size_t exchange_bytes;  // split-K exchange area (0 without split tiles)
  size_t counter_bytes;   // per-split-tile counters (aligned)
  double est_us;  // cost-model estimate of the chosen decomposition
  bool pair;      // CTA pairs (cta_group::2, column kernels only). Prefill: 256 x 256 tiles, the
                  // other fields describe single-CTA tiles. Decode (swap): the fields count pairs
                  // and 256-row weight tiles; each split tile has two exchange halves.
};

// Plan y[T, N] = x[T, K] . W[N, K]^T on a device with `sms` SMs.
// max_exchange_bytes caps the split-K exchange area (SIZE_MAX: no cap).
// The cheapest candidate under a measured-rate cost model is returned.
GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_exchange_bytes);

// The plan the column kernels run: plan_gemm's, or for 256-token decode
// batches the same decomposition over CTA pairs (256 weight rows per pair
// tile, half the batch's tokens per CTA), which the row-parallel kernels do
// not use.
GemmPlan plan_gemm_col(int T, int N, int K, int sms, size_t max_exchange_bytes);

// Scratch layout used by the column GEMM: [status word | split-tile counters
// | exchange area]. The counter region has one size and place for every
// plan, so the exchange area of one shape (f32 partials, left as they are)
// never lies under the counters of another shape that shares the workspace.
// The first kWsHeaderBytes + kWsCounterBytes bytes must be zero before the
// first call; the kernels leave them zero. The exchange area is written
// before it is read.
constexpr size_t kWsHeaderBytes = 256;
constexpr size_t kWsIndexErrorOffset = 4;  // second int of the header: RoPE index errors (no wait polls it)
constexpr size_t kWsCounterBytes = 8192;  // 8 bytes per split tile: up to 1024 split tiles
inline size_t col_workspace_bytes(const GemmPlan& p) {
  return kWsHeaderBytes + kWsCounterBytes + p.exchange_bytes;
}

// Split-K scratch of one column GEMM launch: status word, per-split-tile
// counters (zero at rest) and the f32 exchange area.
struct ColScratch {
  int* status;
  uint32_t* ctr;
  size_t ctr_bytes;
  float* xchg;
  size_t xchg_bytes;
};

// The scratch inside a column workspace of ws_bytes (>= kWsHeaderBytes + kWsCounterBytes).
inline ColScratch col_scratch(uint8_t* ws, size_t ws_bytes) {
  ColScratch sc;
  sc.status = reinterpret_cast<int*>(ws);
  sc.ctr = reinterpret_cast<uint32_t*>(ws + kWsHeaderBytes);
  sc.ctr_bytes = kWsCounterBytes;
  sc.xchg = reinterpret_cast<float*>(ws + kWsHeaderBytes + kWsCounterBytes);
  sc.xchg_bytes = ws_bytes > kWsHeaderBytes + kWsCounterBytes ? ws_bytes - kWsHeaderBytes - kWsCounterBytes : 0;
  return sc;
}

// Plain column GEMM y = x . w^T (+ bias), 16-bit dtype, on caller-provided
// scratch, planned for `sms` SMs with the exchange capped at the scratch's
// size (gemm_col.cu). Used by the one-rank row-parallel path.
int col_gemm_on_scratch(const void* x, const void* w, const void* bias, void* y, int T, int N, int K, int dtype,
                        const ColScratch& sc, void* stream);

}  // namespace pgb
