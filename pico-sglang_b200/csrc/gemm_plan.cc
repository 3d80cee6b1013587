// gemm_plan.cc - choose orientation, tile width and split-K factor.
//
// Decode shapes (T <= 256) are weight-streaming: every weight byte is read
// once from HBM, so the plan fills the MMA M side with 128 weight rows
// (swap) and splits K until the number of work units covers the SMs with
// little wave quantisation. Prefill shapes are tensor-bound and use
// 128 x 256 token x feature tiles without split-K.
#include "gemm_plan.h"

#include <algorithm>
#include <cmath>

namespace pgb {

namespace {
constexpr double kHbmBytesPerSec = 6.5e12;   // measured copy bandwidth class of B200
constexpr double kSmBytesPerSec = 60e9;      // sustained TMA stream of one SM
constexpr double kSplitFixedSec = 0.4e-6;    // counter handshake + extra epilogue pass

int div_up(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

int bn_for_tokens(int T) {
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}
}  // namespace

GemmPlan plan_gemm(int T, int N, int K, int sms, size_t max_partial_bytes) {
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
  const long long pq = static_cast<long long>(p.p_tiles) * p.q_tiles;
  p.splits = 1;
  if (p.swap && pq < 4LL * sms) {
    // Bytes one unit streams: its weight rows (HBM) and token rows (L2),
    // plus the f32 partial written and read back when split.
    const double w_row_bytes = 128.0 * 64.0 * 2.0;           // per k-block
    const double x_row_bytes = static_cast<double>(p.bn) * 64.0 * 2.0;
    double best = 1e30;
    const int max_s = std::min(p.kblocks, 16);
    for (int s = 1; s <= max_s; ++s) {
      const size_t part = (s > 1) ? static_cast<size_t>(pq) * s * 128u * p.bn * 4u : 0u;
      if (part > max_partial_bytes) break;
      const long long units = pq * s;
      const double kb_per_unit = static_cast<double>(p.kblocks) / s;
      const double unit_bytes = kb_per_unit * (w_row_bytes + x_row_bytes) +
                                (s > 1 ? 2.0 * 128.0 * p.bn * 4.0 : 0.0);
      const double total = static_cast<double>(pq) * p.kblocks * w_row_bytes +
                           (s > 1 ? static_cast<double>(units) * 2.0 * 128.0 * p.bn * 4.0 : 0.0);
      const long long waves = (units + sms - 1) / sms;
      const double t = std::max(total / kHbmBytesPerSec, waves * unit_bytes / kSmBytesPerSec) +
                       (s > 1 ? kSplitFixedSec : 0.0);
      if (t < best * 0.98) {
        best = t;
        p.splits = s;
      }
    }
  }
  p.units = static_cast<int>(pq * p.splits);
  p.grid = std::min(p.units, sms);
  p.partial_bytes = p.splits > 1 ? static_cast<size_t>(pq) * p.splits * 128u * p.bn * 4u : 0u;
  p.counter_bytes = (static_cast<size_t>(pq) * 4u + 255u) / 256u * 256u;
  return p;
}

}  // namespace pgb
