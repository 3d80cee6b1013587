// gemm_plan.cc - choose orientation, tile width and work decomposition.
//
// Decode shapes (T <= 256) stream every weight byte once from HBM: the MMA
// M side is filled with 128 weight rows (swap orientation) and the token
// side is only as wide as the batch. Whole tiles are dealt round-robin for
// as many full waves as the tile count allows; the tiles of the ragged last
// wave are split along K into S equal k-ranges on S CTAs each ("split
// tail"), so every SM streams about the same number of weight k-blocks. The
// S CTAs of a split tile reduce-scatter their f32 partials through L2 (see
// split_reduce_tile). S is chosen under a cost model built from rates
// measured on B200: one 16 KB weight k-block per 0.32 us per SM from HBM,
// one 128 x 256 x 64 MMA k-block per 0.38 us, and the exchange's fixed cost
// plus its bytes at the per-SM bulk-copy rate.
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

constexpr double kKbHbmUs = 0.32;          // one 16 KB weight k-block per SM
constexpr double kKbMma256Us = 0.38;       // one 128 x 256 x 64 MMA k-block
constexpr double kSplitFixedUs = 2.0;      // publish, wait for the tile's CTAs, bulk copy, sum
constexpr double kExchangeBytesPerUs = 6.0e4;  // partial bytes one SM stores + loads per us
constexpr int kMaxSplit = 8;

double kb_us(int bn) { return std::max(kKbHbmUs, kKbMma256Us * bn / 256.0); }
}  // namespace

GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_exchange_bytes) {
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
  const double t_kb = kb_us(p.bn);

  // Whole tiles only.
  p.grid = std::min(sms, std::max(p.tiles, 1));
  p.dp_rounds = div_up(p.tiles, p.grid);
  p.split_first = p.tiles;
  p.split_ctas = 0;
  p.nsplit = 1;
  p.exchange_bytes = 0;
  p.counter_bytes = 0;
  p.est_us = p.dp_rounds * p.kblocks * t_kb;
  // Prefill: the column kernel runs these tiles on CTA pairs (256 x 256 per
  // pair, cta_group::2), which load a third less per MMA than one CTA.
  p.pair = !p.swap;
  if (!p.swap) return p;

  // Short reductions at wide batches (T > 64, at most 32 k-blocks: the
  // row-parallel GEMMs at TP >= 2): 64-token tiles without a split, when they
  // fit one wave and fill at least two thirds of it. Each weight tile is then read by ceil(T / 64) CTAs (from L2
  // after the first), which costs less than the split exchange here and more
  // for longer reductions (measured on B200 at T = 256, N = 4096: K = 2048
  // 12.5 us against 15.5 us for 4-way split 256-token tiles; K = 4096 21.8
  // against 19.0 us).
  if (T > 64 && p.kblocks <= 32) {
    GemmPlan q = p;
    q.bn = 64;
    q.q_tiles = div_up(T, 64);
    q.tiles = q.p_tiles * q.q_tiles;
    if (q.tiles <= sms && 3 * q.tiles >= 2 * sms) {
      q.grid = q.tiles;
      q.dp_rounds = 1;
      q.split_first = q.tiles;
      q.est_us = q.kblocks * 0.3;
      return q;
    }
  }

  // Split tail: full waves of whole tiles, the rest split S ways.
  const int full = p.tiles / sms;
  const int rem = p.tiles - full * sms;
  GemmPlan best = p;
  if (rem > 0) {
    const int s_max = std::min({kMaxSplit, sms / rem, p.kblocks});
    for (int S = 2; S <= s_max; ++S) {
      GemmPlan q = p;
      q.dp_rounds = full;
      q.split_first = full * sms;
      q.grid = full > 0 ? sms : rem * S;
      q.split_ctas = rem * S;
      q.nsplit = S;
      q.exchange_bytes = static_cast<size_t>(rem) * S * 128u * q.bn * 4u;
      q.counter_bytes = (static_cast<size_t>(rem) * 8u + 255u) / 256u * 256u;
      if (q.exchange_bytes > max_exchange_bytes) continue;
      const double moved = 2.0 * (S - 1.0) / S * 128.0 * std::min(T, q.bn) * 4.0;
      q.est_us = full * q.kblocks * t_kb + div_up(q.kblocks, S) * t_kb + kSplitFixedUs + moved / kExchangeBytesPerUs;
      if (q.est_us < best.est_us) best = q;
    }
  }
  return best;
}

GemmPlan plan_gemm_col(int T, int N, int K, int sms, size_t max_exchange_bytes) {
  const GemmPlan base = plan_gemm(T, N, K, sms, max_exchange_bytes);
  if (!base.swap || base.bn != 256 || base.q_tiles != 1 || N < 512) return base;
  // Pairs are the unit of work: a 256-row weight tile per pair, its MMA
  // bound at one 256 x 256 x 64 k-block per 0.36 us (each CTA loads 32 KB
  // per k-block, which L2 sustains), the split tail as for single CTAs.
  constexpr double kKbPairUs = 0.36;
  const int units = sms / 2;
  GemmPlan p = base;
  p.pair = true;
  p.bn = 256;
  p.p_tiles = div_up(N, 256);
  p.q_tiles = 1;
  p.tiles = p.p_tiles;
  p.grid = std::min(units, p.tiles);
  p.dp_rounds = div_up(p.tiles, p.grid);
  p.split_first = p.tiles;
  p.split_ctas = 0;
  p.nsplit = 1;
  p.exchange_bytes = 0;
  p.counter_bytes = 0;
  p.est_us = p.dp_rounds * p.kblocks * kKbPairUs;
  const int full = p.tiles / units;
  const int rem = p.tiles - full * units;
  GemmPlan best = p;
  if (rem > 0) {
    const int s_max = std::min({kMaxSplit, units / rem, p.kblocks});
    for (int S = 2; S <= s_max; ++S) {
      GemmPlan q = p;
      q.dp_rounds = full;
      q.split_first = full * units;
      q.grid = full > 0 ? units : rem * S;
      q.split_ctas = rem * S;
      q.nsplit = S;
      q.exchange_bytes = static_cast<size_t>(rem) * 2u * S * 128u * 256u * 4u;
      q.counter_bytes = (static_cast<size_t>(rem) * 2u * 8u + 255u) / 256u * 256u;
      if (q.exchange_bytes > max_exchange_bytes) continue;
      const double moved = 2.0 * (S - 1.0) / S * 128.0 * std::min(T, 256) * 4.0;
      q.est_us = full * q.kblocks * kKbPairUs + div_up(q.kblocks, S) * kKbPairUs + kSplitFixedUs +
                 moved / kExchangeBytesPerUs;
      if (q.est_us < best.est_us) best = q;
    }
  }
  // The single-CTA plan stays when the pairs cannot cover the SMs as well.
  return best.est_us <= base.est_us ? best : base;
}

}  // namespace pgb
