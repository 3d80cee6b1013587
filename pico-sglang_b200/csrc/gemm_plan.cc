// gemm_plan.cc - choose orientation, tile width and work decomposition.
//
// Decode shapes (T <= 256) stream every weight byte once from HBM: the MMA
// M side is filled with 128 weight rows (swap orientation) and the token
// side is only as wide as the batch. Three decompositions compete under a
// cost model built from rates measured on B200 (one 16 KB weight k-block per
// 0.32 us per SM from HBM; one 128x256x64 MMA k-block per 0.38 us):
//   whole tiles      round-robin, no reduction; idle SMs when tiles < SMs;
//   stream-K hybrid  whole tiles for full waves, equal k-block ranges for the
//                    rest, partials reduced in global memory after a grid
//                    barrier (~3 us plus the partial traffic);
//   cluster split-K  clusters of C CTAs split each tile's K range and sum on
//                    chip through distributed shared memory (~0.6 us per
//                    32-token chunk); fewer SMs when tiles do not fill the
//                    co-resident clusters.
// Prefill shapes (T > 256) are tensor-bound with many 128 x 256 tiles: whole
// tiles round-robin.
#include "gemm_plan.h"

#include <algorithm>
#include <cmath>

namespace pgb {

namespace {
int div_up(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

int bn_for_tokens(int T) {
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}

constexpr double kKbHbmUs = 0.32;     // one 16 KB weight k-block per SM
constexpr double kKbMma256Us = 0.38;  // one 128 x 256 x 64 MMA k-block
constexpr double kBarrierUs = 3.0;    // grid barrier after the main loop
constexpr double kChunkUs = 0.6;      // cluster hand-off of one 32-token chunk
constexpr double kL2BytesPerUs = 4.0e6;

double kb_us(int bn) { return std::max(kKbHbmUs, kKbMma256Us * bn / 256.0); }
}  // namespace

ClusterCaps nominal_cluster_caps(int sms) {
  ClusterCaps c;
  const int b200[9] = {0, 148, 74, 45, 33, 0, 22, 0, 15};
  for (int i = 1; i <= 8; ++i) c.max_active[i] = b200[i] * sms / 148;
  return c;
}

GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_partial_bytes, bool all_streamk,
                   const ClusterCaps* caps, bool fused_row) {
  GemmPlan p{};
  p.kblocks = div_up(K, 64);
  if (T <= 256) {
    p.swap = true;
    p.bn = bn_for_tokens(T);
    p.p_tiles = div_up(N, 128);
    p.q_tiles = 1;
  } else {
    p.swap = false;
    p.bn = 256;
    p.p_tiles = div_up(T, 128);
    p.q_tiles = div_up(N, 256);
  }
  p.tiles = p.p_tiles * p.q_tiles;
  p.counter_bytes = 0;

  auto whole_tiles = [&](GemmPlan& q) {
    const int G = std::min(sms, std::max(q.tiles, 1));
    q.grid = G;
    q.sk_grid = 0;
    q.dp_rounds = div_up(q.tiles, G);
    q.sk_first = q.tiles;
    q.max_contrib = 1;
    q.partial_bytes = 0;
    q.csk = 0;
    q.n_clusters = 0;
    q.est_us = q.dp_rounds * q.kblocks * kb_us(q.bn);
  };

  if (!p.swap) {
    whole_tiles(p);
    return p;
  }

  const double t_kb = kb_us(p.bn);
  GemmPlan best = p;
  whole_tiles(best);

  // Stream-K hybrid (partials are token-major: swap orientation only).
  {
    GemmPlan q = p;
    q.csk = 0;
    q.n_clusters = 0;
    q.grid = sms;
    q.dp_rounds = all_streamk ? 0 : q.tiles / sms;
    q.sk_first = q.dp_rounds * sms;
    const long long sk_tiles = q.tiles - q.sk_first;
    bool ok = true;
    if (sk_tiles > 0) {
      const long long total = sk_tiles * q.kblocks;
      q.sk_grid = static_cast<int>(std::min<long long>(q.grid, total));
      const long long per_cta = total / q.sk_grid;  // >= 1: no empty stream-K range
      long long mc = div_up(q.kblocks, per_cta) + 1;
      mc = std::min<long long>({mc, q.sk_grid, static_cast<long long>(q.kblocks)});
      q.max_contrib = static_cast<int>(mc);
      q.partial_bytes = static_cast<size_t>(sk_tiles) * q.max_contrib * 128u * q.bn * 4u;
      ok = q.partial_bytes <= max_partial_bytes && total * q.sk_grid < (1LL << 31);
      const double avg_ctb = static_cast<double>(total) / q.sk_grid > 0
                                 ? std::min<double>(mc, q.kblocks / (static_cast<double>(total) / q.sk_grid) + 1.0)
                                 : 1.0;
      const double traffic = 2.0 * sk_tiles * avg_ctb * 128.0 * T * 4.0;
      q.est_us = q.dp_rounds * q.kblocks * t_kb + std::ceil(static_cast<double>(total) / q.sk_grid) * t_kb +
                 kBarrierUs + traffic / kL2BytesPerUs / sms * 8.0;
    } else {
      q.sk_grid = 0;
      q.max_contrib = 1;
      q.partial_bytes = 0;
      q.est_us = q.dp_rounds * q.kblocks * t_kb;
    }
    if (ok && q.est_us < best.est_us) best = q;
  }

  // Cluster split-K.
  if (caps != nullptr) {
    for (int C : {2, 3, 4, 6, 8}) {
      const int maxc = caps->max_active[C];
      if (maxc <= 0 || p.kblocks < C) continue;
      GemmPlan q = p;
      q.csk = C;
      q.n_clusters = std::min(maxc, q.tiles);
      q.grid = q.n_clusters * C;
      q.sk_grid = 0;
      q.dp_rounds = 0;
      q.sk_first = q.tiles;
      q.max_contrib = 1;
      q.partial_bytes = 0;
      const int rounds = div_up(q.tiles, q.n_clusters);
      q.est_us = rounds * div_up(q.kblocks, C) * t_kb + rounds * (q.bn / 32) * kChunkUs;
      if (fused_row) q.est_us -= 0.0;  // one source per element in the reduce phase, like whole tiles
      if (q.est_us < best.est_us) best = q;
    }
  }
  (void)fused_row;
  return best;
}

}  // namespace pgb
