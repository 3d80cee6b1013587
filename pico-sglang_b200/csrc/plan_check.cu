// plan_check.cu - host-side verification of the GEMM work decomposition.
//
// Replays, on the CPU, the segment sequence every CTA of a planned launch
// walks (the same SegIter the kernels use) and checks that the plan covers
// every (tile, k-block) exactly once and that stream-K contributor indices
// and counts agree with the actual coverage and stay inside the reserved
// partial slabs. Used by the CPU tests; no device is touched.
#include <vector>

#include "gemm_plan.h"
#include "gemm_sm100.cuh"
#include "host_common.h"

namespace {
constexpr size_t kSplitScratchBytesForPlan = 32u << 20;  // the communicator's stream-K scratch
}

extern "C" int pgb_check_work_plan(int T, int N, int K, int sms, int all_streamk, int launch_grid,
                                   int clusters) {
  using namespace pgb;
  if (T <= 0 || N <= 0 || K <= 0 || sms <= 0)
    return set_error(PGB_ERR_INVALID, "check_work_plan: bad arguments");
  const ClusterCaps caps = nominal_cluster_caps(sms);
  const GemmPlan p = plan_gemm(T, N, K, sms, SIZE_MAX, all_streamk != 0, clusters ? &caps : nullptr,
                               all_streamk != 0);
  GemmShape g{};
  g.T = T;
  g.N = N;
  g.K = K;
  g.kblocks = p.kblocks;
  g.p_tiles = p.p_tiles;
  g.q_tiles = p.q_tiles;
  g.tiles = p.tiles;
  g.dp_rounds = p.dp_rounds;
  g.sk_first = p.sk_first;
  g.grid = p.grid;
  g.sk_grid = p.sk_grid;
  g.max_contrib = p.max_contrib;
  g.csk = p.csk;
  g.n_clusters = p.n_clusters;
  // A cluster split-K launch has exactly n_clusters * csk CTAs.
  const int grid = p.csk > 1 ? p.grid : (launch_grid > 0 ? launch_grid : p.grid);
  if (grid < p.grid) return set_error(PGB_ERR_INVALID, "check_work_plan: launch grid below plan grid");
  std::vector<int> cover(static_cast<size_t>(p.tiles) * p.kblocks, 0);
  std::vector<int> ctb_seen(static_cast<size_t>(p.tiles) * ((p.csk > 1 ? p.csk : p.max_contrib) + 1), 0);
  std::vector<int> ctb_count(p.tiles, 0);
  for (int c = 0; c < grid; ++c) {
    SegIter it(g, c);
    Seg s;
    while (it.next(g, s)) {
      if (s.tile < 0 || s.tile >= p.tiles || s.kb0 < 0 || s.kb1 > p.kblocks || s.kb0 >= s.kb1)
        return set_error(PGB_ERR_STATE, "cta %d: bad segment tile %d [%d, %d)", c, s.tile, s.kb0, s.kb1);
      if (s.p != s.tile % p.p_tiles || s.q != s.tile / p.p_tiles)
        return set_error(PGB_ERR_STATE, "cta %d: tile coordinates disagree", c);
      for (int kb = s.kb0; kb < s.kb1; ++kb) ++cover[static_cast<size_t>(s.tile) * p.kblocks + kb];
      if (s.nctb != tile_contributors(g, s.tile))
        return set_error(PGB_ERR_STATE, "tile %d: segment says %d contributors, formula %d", s.tile, s.nctb,
                         tile_contributors(g, s.tile));
      if (s.contrib < 0 || s.contrib >= s.nctb)
        return set_error(PGB_ERR_STATE, "tile %d: contributor %d of %d", s.tile, s.contrib, s.nctb);
      if (p.csk <= 1 && s.tile >= p.sk_first && s.contrib >= p.max_contrib)
        return set_error(PGB_ERR_STATE, "tile %d: contributor %d beyond %d slabs", s.tile, s.contrib,
                         p.max_contrib);
      if (p.csk <= 1 && s.tile < p.sk_first && (s.nctb != 1 || s.kb0 != 0 || s.kb1 != p.kblocks))
        return set_error(PGB_ERR_STATE, "round-robin tile %d split", s.tile);
      const int slots = p.csk > 1 ? p.csk : p.max_contrib;
      const size_t key = static_cast<size_t>(s.tile) * (slots + 1) + std::min(s.contrib, slots);
      if (ctb_seen[key]++ != 0)
        return set_error(PGB_ERR_STATE, "tile %d: contributor %d appears twice", s.tile, s.contrib);
      ++ctb_count[s.tile];
    }
  }
  for (size_t i = 0; i < cover.size(); ++i)
    if (cover[i] != 1)
      return set_error(PGB_ERR_STATE, "tile %zu k-block %zu covered %d times", i / p.kblocks, i % p.kblocks,
                       cover[i]);
  for (int t = 0; t < p.tiles; ++t)
    if (ctb_count[t] != tile_contributors(g, t))
      return set_error(PGB_ERR_STATE, "tile %d: %d contributors seen, formula %d", t, ctb_count[t],
                       tile_contributors(g, t));
  const size_t need = static_cast<size_t>(p.tiles - p.sk_first) * p.max_contrib * 128u * p.bn * 4u;
  if (p.csk > 1 && (p.kblocks < p.csk || p.grid != p.n_clusters * p.csk))
    return set_error(PGB_ERR_STATE, "cluster split-K plan with %d k-blocks over %d CTAs per cluster",
                     p.kblocks, p.csk);
  if (p.csk <= 1 && p.sk_first < p.tiles && need > p.partial_bytes)
    return set_error(PGB_ERR_STATE, "partials need %zu bytes, plan reserves %zu", need, p.partial_bytes);
  return PGB_OK;
}

extern "C" int pgb_describe_plan(int T, int N, int K, int sms, int fused_row, int clusters, char* out,
                                 size_t out_bytes) {
  using namespace pgb;
  if (out == nullptr || out_bytes == 0) return set_error(PGB_ERR_INVALID, "describe_plan: no buffer");
  const ClusterCaps caps = nominal_cluster_caps(sms);
  const GemmPlan p = plan_gemm(T, N, K, sms, fused_row ? kSplitScratchBytesForPlan : SIZE_MAX, fused_row != 0,
                               clusters ? &caps : nullptr, fused_row != 0);
  snprintf(out, out_bytes,
           "swap=%d bn=%d tiles=%d kblocks=%d grid=%d dp_rounds=%d sk_first=%d sk_grid=%d max_contrib=%d "
           "csk=%d n_clusters=%d partial_bytes=%zu est_us=%.2f",
           p.swap ? 1 : 0, p.bn, p.tiles, p.kblocks, p.grid, p.dp_rounds, p.sk_first, p.sk_grid, p.max_contrib,
           p.csk, p.n_clusters, p.partial_bytes, p.est_us);
  return PGB_OK;
}
