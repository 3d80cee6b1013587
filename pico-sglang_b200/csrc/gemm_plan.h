// gemm_plan.h - host-side tile and work-decomposition planning for the
// tcgen05 GEMM core.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace pgb {

// Co-resident clusters of each size for one GEMM kernel configuration
// (cudaOccupancyMaxActiveClusters); 0 = size not usable.
struct ClusterCaps {
  int max_active[9] = {};
};

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
  int csk;        // cluster split-K cluster size (0: not used)
  int n_clusters; // clusters launched when csk > 1
  size_t partial_bytes;   // partial scratch (0 without stream-K)
  size_t counter_bytes;   // tile counters (aligned)
  double est_us;  // cost-model estimate of the chosen decomposition
};

// Plan y[T, N] = x[T, K] . W[N, K]^T on a device with `sms` SMs.
//  - max_partial_bytes caps the stream-K scratch (SIZE_MAX: no cap);
//  - all_streamk: the stream-K candidate covers every tile (the fused
//    row-parallel kernel, whose decode phases read per-tile partials);
//  - caps: cluster sizes usable for cluster split-K (nullptr: none);
//  - fused_row: cost the candidates for the fused row-parallel kernel.
// The cheapest candidate under a measured-rate cost model is returned.
GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_partial_bytes, bool all_streamk = false,
                   const ClusterCaps* caps = nullptr, bool fused_row = false);

// Cluster capacities measured on B200 (148 SMs, one CTA of ~216 KB shared
// memory per SM), scaled to `sms`; used where no device can be queried.
ClusterCaps nominal_cluster_caps(int sms);

// Scratch layout used by the column GEMM: [status word | counters | partials].
constexpr size_t kWsHeaderBytes = 256;
inline size_t col_workspace_bytes(const GemmPlan& p) {
  return kWsHeaderBytes + p.counter_bytes + p.partial_bytes;
}

}  // namespace pgb
