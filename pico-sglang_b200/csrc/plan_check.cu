// plan_check.cu - host-side verification of the GEMM work decomposition.
//
// Replays, on the CPU, the segment sequence every CTA of a planned launch
// walks (the same SegIter the kernels use) and checks that the plan covers
// every (tile, k-block) exactly once, that each split tile has exactly
// nsplit CTAs with distinct k-range indices, that the split columns of every
// split tile partition its real tokens, and that the exchange area and the
// gathered pieces fit what the plan and the pipeline ring reserve. Used by
// the CPU tests; no device is touched.
#include <vector>

#include "comm.h"
#include "gemm_plan.h"
#include "gemm_sm100.cuh"
#include "host_common.h"

namespace {
pgb::GemmPlan plan_for(int T, int N, int K, int sms, int fused_row) {
  return fused_row ? pgb::plan_gemm(T, N, K, sms, pgb::kSplitScratchBytes) : pgb::plan_gemm_col(T, N, K, sms, SIZE_MAX);
}
}  // namespace

// all_streamk selects the fused row-parallel kernel's plan (its exchange area
// is the communicator's); launch_grid > 0 replays a launch wider than the
// plan's grid (the row kernel launches one CTA per SM). `clusters` is unused.
extern "C" int pgb_check_work_plan(int T, int N, int K, int sms, int all_streamk, int launch_grid,
                                   int clusters) {
  using namespace pgb;
  (void)clusters;
  if (T <= 0 || N <= 0 || K <= 0 || sms <= 0)
    return set_error(PGB_ERR_INVALID, "check_work_plan: bad arguments");
  const GemmPlan p = plan_for(T, N, K, sms, all_streamk);
  GemmShape g{};
  g.T = T;
  g.N = N;
  g.K = K;
  g.kblocks = p.kblocks;
  g.p_tiles = p.p_tiles;
  g.q_tiles = p.q_tiles;
  g.tiles = p.tiles;
  g.dp_rounds = p.dp_rounds;
  g.split_first = p.split_first;
  g.grid = p.grid;
  g.split_ctas = p.split_ctas;
  g.nsplit = p.nsplit;
  const int grid = launch_grid > 0 ? launch_grid : p.grid;
  if (grid < p.grid) return set_error(PGB_ERR_INVALID, "check_work_plan: launch grid below plan grid");
  if (p.grid > sms) return set_error(PGB_ERR_STATE, "plan grid %d above %d SMs", p.grid, sms);
  if (p.split_ctas != (p.tiles - p.split_first) * p.nsplit || p.split_ctas > p.grid)
    return set_error(PGB_ERR_STATE, "split CTAs %d for %d split tiles of %d on a grid of %d", p.split_ctas,
                     p.tiles - p.split_first, p.nsplit, p.grid);
  if (p.nsplit > 1 && (p.nsplit > p.kblocks || !p.swap))
    return set_error(PGB_ERR_STATE, "split of %d over %d k-blocks (swap %d)", p.nsplit, p.kblocks, p.swap);
  std::vector<int> cover(static_cast<size_t>(p.tiles) * p.kblocks, 0);
  std::vector<int> seen(static_cast<size_t>(p.tiles) * (p.nsplit + 1), 0);
  for (int c = 0; c < grid; ++c) {
    SegIter it(g, c);
    Seg s;
    int nseg = 0, nsplit_seg = 0;
    while (it.next(g, s)) {
      ++nseg;
      if (s.tile < 0 || s.tile >= p.tiles || s.kb0 < 0 || s.kb1 > p.kblocks || s.kb0 >= s.kb1)
        return set_error(PGB_ERR_STATE, "cta %d: bad segment tile %d [%d, %d)", c, s.tile, s.kb0, s.kb1);
      if (s.p != s.tile % p.p_tiles || s.q != s.tile / p.p_tiles)
        return set_error(PGB_ERR_STATE, "cta %d: tile coordinates disagree", c);
      for (int kb = s.kb0; kb < s.kb1; ++kb) ++cover[static_cast<size_t>(s.tile) * p.kblocks + kb];
      if (s.nctb != tile_contributors(g, s.tile))
        return set_error(PGB_ERR_STATE, "tile %d: segment says %d CTAs, formula %d", s.tile, s.nctb,
                         tile_contributors(g, s.tile));
      if (s.contrib < 0 || s.contrib >= s.nctb)
        return set_error(PGB_ERR_STATE, "tile %d: k-range %d of %d", s.tile, s.contrib, s.nctb);
      if (s.tile < p.split_first && (s.nctb != 1 || s.kb0 != 0 || s.kb1 != p.kblocks))
        return set_error(PGB_ERR_STATE, "whole tile %d split", s.tile);
      if (s.nctb > 1) {
        ++nsplit_seg;
        // A split segment is the CTA's last: its ring then holds the gathered pieces.
        Seg rest;
        SegIter probe = it;
        if (probe.next(g, rest)) return set_error(PGB_ERR_STATE, "cta %d: segment after its split segment", c);
      }
      const size_t key = static_cast<size_t>(s.tile) * (p.nsplit + 1) + std::min(s.contrib, p.nsplit);
      if (seen[key]++ != 0) return set_error(PGB_ERR_STATE, "tile %d: k-range %d twice", s.tile, s.contrib);
    }
    if (nsplit_seg > 1) return set_error(PGB_ERR_STATE, "cta %d: %d split segments", c, nsplit_seg);
    (void)nseg;
  }
  for (size_t i = 0; i < cover.size(); ++i)
    if (cover[i] != 1)
      return set_error(PGB_ERR_STATE, "tile %zu k-block %zu covered %d times", i / p.kblocks, i % p.kblocks,
                       cover[i]);
  // Split columns partition the real tokens of every split tile.
  for (int t = p.split_first; t < p.tiles; ++t) {
    const int q = t / p.p_tiles;
    const int V = std::min(p.bn, T - q * p.bn);
    int prev = 0;
    for (int r = 0; r < p.nsplit; ++r) {
      int c0, c1;
      split_cols(p.bn, V, p.nsplit, r, c0, c1);
      if (c0 != prev || c1 < c0) return set_error(PGB_ERR_STATE, "tile %d: split columns of %d not contiguous", t, r);
      prev = c1;
    }
    if (prev != V) return set_error(PGB_ERR_STATE, "tile %d: split columns cover %d of %d tokens", t, prev, V);
  }
  const size_t need = static_cast<size_t>(p.tiles - p.split_first) * p.nsplit * 128u * p.bn * 4u;
  if (p.nsplit > 1 && need > p.exchange_bytes)
    return set_error(PGB_ERR_STATE, "exchange needs %zu bytes, plan reserves %zu", need, p.exchange_bytes);
  if (p.counter_bytes < static_cast<size_t>(p.tiles - p.split_first) * 8u)
    return set_error(PGB_ERR_STATE, "counters need %d bytes, plan reserves %zu", (p.tiles - p.split_first) * 8,
                     p.counter_bytes);
  // Counters live in a fixed region: the column workspace's, or the
  // communicator's for the row kernel.
  const size_t region = all_streamk ? kTileCounterBytes : kWsCounterBytes;
  if (p.counter_bytes > region)
    return set_error(PGB_ERR_STATE, "counters need %zu bytes, the region holds %zu", p.counter_bytes, region);
  // The gathered pieces must fit the smallest ring of this tile width.
  const size_t ring = gemm_ring_bytes(p.bn);
  if (p.nsplit > 1 && split_recv_bytes(p.bn, p.nsplit) > ring)
    return set_error(PGB_ERR_STATE, "split of %d gathers %zu bytes, ring holds %zu", p.nsplit,
                     split_recv_bytes(p.bn, p.nsplit), ring);
  return PGB_OK;
}

extern "C" int pgb_describe_plan(int T, int N, int K, int sms, int fused_row, int clusters, char* out,
                                 size_t out_bytes) {
  using namespace pgb;
  (void)clusters;
  if (out == nullptr || out_bytes == 0) return set_error(PGB_ERR_INVALID, "describe_plan: no buffer");
  const GemmPlan p = plan_for(T, N, K, sms, fused_row);
  snprintf(out, out_bytes,
           "swap=%d bn=%d tiles=%d kblocks=%d grid=%d dp_rounds=%d split_first=%d split_ctas=%d nsplit=%d "
           "exchange_bytes=%zu est_us=%.2f pair=%d",
           p.swap ? 1 : 0, p.bn, p.tiles, p.kblocks, p.grid, p.dp_rounds, p.split_first, p.split_ctas, p.nsplit,
           p.exchange_bytes, p.est_us, (p.pair && !fused_row) ? 1 : 0);
  return PGB_OK;
}
