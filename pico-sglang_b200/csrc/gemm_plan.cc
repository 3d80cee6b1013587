// gemm_plan.cc - choose orientation, tile width and work decomposition.
//
// Decode shapes (T <= 256) stream every weight byte once from HBM. The MMA
// M side is filled with 128 weight rows (swap orientation) and the token
// side is only as wide as the batch, rounded up to 32. The tiles' k-blocks
// are then split evenly over the SMs (stream-K), so every SM streams the
// same number of bytes and none idles while others finish a last wave.
// Prefill shapes (T > 256) are tensor-bound and have many 128 x 256 tiles;
// with at least four waves of tiles, whole tiles are dealt round-robin.
#include "gemm_plan.h"

#include <algorithm>

namespace pgb {

namespace {
int div_up(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

int bn_for_tokens(int T) {
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}
}  // namespace

GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_partial_bytes, bool all_streamk) {
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
  p.sk_grid = 0;
  p.max_contrib = 1;
  p.partial_bytes = 0;
  // Round-robin whole tiles for every full wave; stream-K (swap orientation
  // only: its partials are token-major) for the remainder.
  const int G = std::min(sms, std::max(p.tiles, 1));
  if (p.swap) {
    p.grid = sms;
    p.dp_rounds = all_streamk ? 0 : p.tiles / sms;
    p.sk_first = p.dp_rounds * sms;
    const long long sk_tiles = p.tiles - p.sk_first;
    if (sk_tiles > 0) {
      const long long total = sk_tiles * p.kblocks;
      p.sk_grid = static_cast<int>(std::min<long long>(p.grid, total));
      const long long per_cta = total / p.sk_grid;  // >= 1: no empty stream-K range
      long long mc = div_up(p.kblocks, per_cta) + 1;
      mc = std::min<long long>({mc, p.sk_grid, static_cast<long long>(p.kblocks)});
      p.max_contrib = static_cast<int>(mc);
      p.partial_bytes = static_cast<size_t>(sk_tiles) * p.max_contrib * 128u * p.bn * 4u;
      if (p.partial_bytes <= max_partial_bytes) return p;
    } else {
      return p;
    }
  }
  // Whole tiles only.
  p.grid = G;
  p.sk_grid = 0;
  p.dp_rounds = div_up(p.tiles, G);
  p.sk_first = p.tiles;
  p.max_contrib = 1;
  p.partial_bytes = 0;
  return p;
}

}  // namespace pgb
