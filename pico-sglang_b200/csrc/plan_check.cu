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

extern "C" int pgb_check_work_plan(int T, int N, int K, int sms, int all_streamk, int launch_grid) {
  using namespace pgb;
  if (T <= 0 || N <= 0 || K <= 0 || sms <= 0)
    return set_error(PGB_ERR_INVALID, "check_work_plan: bad arguments");
  const GemmPlan p = plan_gemm(T, N, K, sms, SIZE_MAX, all_streamk != 0);
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
  const int grid = launch_grid > 0 ? launch_grid : p.grid;
  if (grid < p.grid) return set_error(PGB_ERR_INVALID, "check_work_plan: launch grid below plan grid");
  std::vector<int> cover(static_cast<size_t>(p.tiles) * p.kblocks, 0);
  std::vector<int> ctb_seen(static_cast<size_t>(p.tiles) * (p.max_contrib + 1), 0);
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
      if (s.tile >= p.sk_first && s.contrib >= p.max_contrib)
        return set_error(PGB_ERR_STATE, "tile %d: contributor %d beyond %d slabs", s.tile, s.contrib,
                         p.max_contrib);
      if (s.tile < p.sk_first && (s.nctb != 1 || s.kb0 != 0 || s.kb1 != p.kblocks))
        return set_error(PGB_ERR_STATE, "round-robin tile %d split", s.tile);
      const size_t key = static_cast<size_t>(s.tile) * (p.max_contrib + 1) + std::min(s.contrib, p.max_contrib);
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
  if (p.sk_first < p.tiles && need > p.partial_bytes)
    return set_error(PGB_ERR_STATE, "partials need %zu bytes, plan reserves %zu", need, p.partial_bytes);
  return PGB_OK;
}
