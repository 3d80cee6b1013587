// gemm_sm100.cuh - persistent, warp-specialised tcgen05 GEMM core.
//
// Computes the products of the tensor-parallel linear layers,
//   y[T, N] = x[T, K] . W[N, K]^T      (x, W row-major bf16/f16, f32 accumulate)
// which is what LinearTPImpl.forward (python/picosgl/layers/linear.py:23-27)
// obtains from F.linear / cuBLAS.
//
// Roles inside one 192-thread CTA (one CTA per SM, persistent over tiles):
//   warp 0, one lane : TMA producer. Streams A and B k-blocks (64 wide,
//                      128-byte swizzle) into a STAGES-deep shared ring.
//   warp 1, one lane : MMA issuer. tcgen05.mma (M=128, N=BN, K=16) into one of
//                      two TMEM accumulators, so the epilogue of tile i
//                      overlaps the main loop of tile i+1. Warp 1 also owns the
//                      TMEM allocation.
//   warps 2..5       : epilogue. TMEM -> registers (tcgen05.ld 32x32b), split-K
//                      combine, then the mode-specific store.
//
// Tile orientation. The MMA M side (128 rows, "P") and N side (BN rows, "Q")
// are assigned per problem shape:
//   SWAP = false : P = tokens, Q = output features  (prefill; T large)
//   SWAP = true  : P = output features, Q = tokens  (decode; T <= 256), so the
//                  128-row MMA side is always filled by weight rows and the
//                  token side is only as wide as the batch.
//
// Split tiles (see GemmShape): the CTAs that share a tile's K range
// reduce-scatter their f32 partials through L2 (split_reduce_tile); every
// output element is summed in split order, so the result does not depend on
// timing.
#pragma once

#include "sm100.cuh"

namespace pgb {

constexpr int kBlockK = 64;          // k-block: one 128-byte swizzle atom of 16-bit elements
constexpr int kTileP = 128;          // MMA M
constexpr int kGemmThreads = 192;    // 6 warps
constexpr int kEpiThreads = 128;     // warps 2..5
constexpr int kMaxRanks = 8;

// Everything the GEMM loop needs to know about the problem.
//
// Work decomposition. The output is cut into tiles of 128 (P) x BN (Q); a
// tile's reduction dimension is `kblocks` k-blocks of 64. Tiles
// [0, split_first) are whole tiles dealt round-robin: CTA c computes tiles
// c, c + grid, ... (dp_rounds of them at most). Tiles [split_first, tiles)
// are split tiles: split tile u is cut into nsplit equal k-ranges, and CTA
// c < split_ctas takes k-range c % nsplit of split tile c / nsplit after its
// whole tiles, so every SM streams about the same number of k-blocks and no
// SM idles through a ragged last wave. The nsplit CTAs of a split tile are
// co-resident (cooperative launch) and reduce-scatter their partials through
// the exchange area (split_reduce_tile).
struct GemmShape {
  int T, N, K;
  int kblocks;      // ceil(K / 64)
  int p_tiles;      // tiles along the MMA M side
  int q_tiles;      // tiles along the MMA N side
  int tiles;        // p_tiles * q_tiles
  int dp_rounds;    // whole tiles per CTA at most
  int split_first;  // first split tile (== tiles: none)
  int grid;         // CTAs that take work (<= gridDim.x)
  int split_ctas;   // (tiles - split_first) * nsplit
  int nsplit;       // k-ranges per split tile
  float* xchg;      // exchange area [tiles - split_first][nsplit][BN tokens][128 features] f32
  uint32_t* ctr;    // per split tile: {published, finished} counters, zero at rest
  int* status;      // device status word (first error wins)
  uint64_t wait_ns; // budget for every intra-kernel wait
  int glu;          // gated mode: N = gated width I, the weight is [gate; up] of 2I rows
};

// One contiguous piece of a tile's reduction handled by this CTA.
struct Seg {
  int tile, p, q;
  int kb0, kb1;   // k-block range [kb0, kb1)
  int contrib;    // index of this CTA among the tile's CTAs (its k-range)
  int nctb;       // number of CTAs sharing the tile (1 = whole tile)
};

// Iterates the segments of CTA `cta` in order: its whole tiles, then its
// split segment. All roles of a CTA walk the same sequence. Host-callable so
// the decomposition can be checked without a GPU.
struct SegIter {
  int cta, round, split_done;
  __host__ __device__ __forceinline__ SegIter(const GemmShape& g, int cta_) {
    cta = cta_;
    round = cta < g.grid ? 0 : g.dp_rounds;
    split_done = cta < g.split_ctas ? 0 : 1;
  }
  __device__ __forceinline__ explicit SegIter(const GemmShape& g) : SegIter(g, static_cast<int>(blockIdx.x)) {}
  __host__ __device__ __forceinline__ bool next(const GemmShape& g, Seg& s) {
    while (round < g.dp_rounds) {
      s.tile = cta + round * g.grid;
      ++round;
      if (s.tile < g.split_first) {
        s.kb0 = 0;
        s.kb1 = g.kblocks;
        s.contrib = 0;
        s.nctb = 1;
        s.p = s.tile % g.p_tiles;
        s.q = s.tile / g.p_tiles;
        return true;
      }
      round = g.dp_rounds;  // ragged last round: no more whole tiles
    }
    if (split_done) return false;
    split_done = 1;
    const int S = g.nsplit, j = cta % S;
    s.tile = g.split_first + cta / S;
    s.kb0 = j * g.kblocks / S;
    s.kb1 = (j + 1) * g.kblocks / S;
    s.contrib = j;
    s.nctb = S;
    s.p = s.tile % g.p_tiles;
    s.q = s.tile / g.p_tiles;
    return true;
  }
};

// Number of CTAs sharing `tile` (1 for whole tiles).
__host__ __device__ __forceinline__ int tile_contributors(const GemmShape& g, int tile) {
  return tile >= g.split_first ? g.nsplit : 1;
}

// Weight tile of segment s, k-block kb, into dst (the A operand in the swap
// orientation, B otherwise). In gated mode (g.glu) the weight is the merged
// [gate; up] matrix of 2 * g.N rows (LinearColParallelMerged's layout,
// python/picosgl/layers/linear.py:45-56) and a tile is two boxes of half
// height: gate rows r0 .. and the up rows g.N + r0 .. of the same output
// features, stacked. Both halves are whole 1024-byte swizzle atoms, so the
// stacked boxes have the layout of one full-height box.
template <int BN, bool SWAP>
__device__ __forceinline__ void load_weight_tile(const GemmShape& g, const CUtensorMap* tm, uint64_t* bar,
                                                 uint8_t* dst, int kb, const Seg& s, uint64_t hint) {
  constexpr int kRows = SWAP ? kTileP : BN;
  const int t = SWAP ? s.p : s.q;
  if (!g.glu) {
    tma_load_2d(tm, bar, dst, kb * kBlockK, t * kRows, hint);
    return;
  }
  const int r0 = t * (kRows / 2);
  tma_load_2d(tm, bar, dst, kb * kBlockK, r0, hint);
  tma_load_2d(tm, bar, dst + (kRows / 2) * kBlockK * 2, kb * kBlockK, g.N + r0, hint);
}

// EXTRA: bytes of an epilogue-policy region after the barriers (0: none).
template <int BN, int STAGES, int EXTRA = 0>
struct GemmSmem {
  static constexpr int kABytes = kTileP * kBlockK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kBlockK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
  // Layout (from a 1024-byte aligned base): A ring, B ring, barriers, extra.
  static constexpr int kOffA = 0;
  static constexpr int kOffB = STAGES * kABytes;
  static constexpr int kOffEpi = kOffB + STAGES * kBBytes;
  static constexpr int kEpiBytes = 32 * kTileP * 2;  // 32 tokens x 128 features, 16-bit
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  static constexpr int kBarBytes = 8 * (2 * STAGES + 6) + 64;
  static constexpr int kOffExtra = kOffBar + kBarBytes;
  static constexpr int kBytes = kOffExtra + EXTRA + 1024;  // + alignment slack
};

// CTAs per SM a GEMM kernel of tile width BN is built for. Narrow decode
// tiles (BN <= 64) fit two CTAs per SM, so the next kernel in the stream
// (programmatic dependent launch) becomes resident next to this one, sets up
// and requests its first weight stages while this kernel finishes its tail.
__host__ __device__ constexpr int gemm_ctas_per_sm(int bn) { return bn <= 64 ? 2 : 1; }

// Pipeline depth that fills the shared-memory budget for a tile width:
// ~100 KB of ring when two CTAs share an SM, ~200 KB otherwise (room is left
// for the epilogue tile and the barriers).
__host__ __device__ constexpr int gemm_stages_for(int bn) {
  return ((gemm_ctas_per_sm(bn) == 2 ? 100 : 200) * 1024) / (kTileP * kBlockK * 2 + bn * kBlockK * 2) > 12
             ? 12
             : ((gemm_ctas_per_sm(bn) == 2 ? 100 : 200) * 1024) / (kTileP * kBlockK * 2 + bn * kBlockK * 2);
}
template <int BN>
constexpr int gemm_stages() {
  return gemm_stages_for(BN);
}

// Bytes of the pipeline ring of a tile width (A and B stages).
__host__ __device__ constexpr size_t gemm_ring_bytes(int bn) {
  return static_cast<size_t>(gemm_stages_for(bn)) * static_cast<size_t>(kTileP + bn) * kBlockK * 2u;
}

// Split-K column runs. A split tile's real tokens are cut into nsplit runs of
// whole units, one per CTA; each CTA sums the S partials of its run. Units of
// 32 tokens (one epilogue chunk) when the largest run's gather area fits the
// ring, else 4-token groups (S = 7 at BN = 256, S >= 7 at BN <= 64): with
// 32-token units every chunk of the partial is wholly one CTA's, which the
// epilogue moves with constant-offset loads and stores.
__host__ __device__ constexpr size_t split_recv_bytes_unit(int BN, int S, int unit) {
  return static_cast<size_t>(S) * static_cast<size_t>(((BN + unit - 1) / unit + S - 1) / S) *
         static_cast<size_t>(unit) * 128u * 4u;
}
__host__ __device__ constexpr int split_unit(int BN, int S) {
  return split_recv_bytes_unit(BN, S, 32) <= gemm_ring_bytes(BN) ? 32 : 4;
}

// Token columns [c0, c1) of a split tile of width BN (tile-relative, V real
// tokens) that split r of S owns: runs of split_unit tokens, cut evenly.
__host__ __device__ __forceinline__ void split_cols(int BN, int V, int S, int r, int& c0, int& c1) {
  const int unit = split_unit(BN, S);
  const int G = (V + unit - 1) / unit;
  c0 = (r * G / S) * unit;
  c1 = ((r + 1) * G / S) * unit;
  c0 = c0 < V ? c0 : V;
  c1 = c1 < V ? c1 : V;
}

// Bytes of a split CTA's gather area in its ring: S slots (its own and the
// others' pieces) of its largest column run, 128 f32 per column.
__host__ __device__ constexpr size_t split_recv_bytes(int BN, int S) {
  return split_recv_bytes_unit(BN, S, split_unit(BN, S));
}

struct GemmCtl {
  uint64_t* full;       // [STAGES]
  uint64_t* empty;      // [STAGES]
  uint64_t* acc_full;   // [2]
  uint64_t* acc_empty;  // [2]
  uint64_t* drain;      // [1] used only when unwinding after a timeout
  uint32_t* tmem_base;
  int* abort;
  int* flag;
  uint8_t* a;
  uint8_t* b;
  uint16_t* epi;  // [32][128] staging tile of the swap-orientation epilogue
  uint64_t* xchg; // split tiles: the others' pieces have landed in the ring
  uint8_t* extra; // the epilogue policy's region (GemmSmem EXTRA bytes)
};

template <int BN, int STAGES, int EXTRA = 0>
__device__ __forceinline__ GemmCtl gemm_carve_smem(uint8_t* raw) {
  using L = GemmSmem<BN, STAGES, EXTRA>;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  GemmCtl c;
  c.a = base + L::kOffA;
  c.b = base + L::kOffB;
  c.epi = reinterpret_cast<uint16_t*>(base + L::kOffEpi);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::kOffBar);
  c.full = bars;
  c.empty = bars + STAGES;
  c.acc_full = bars + 2 * STAGES;
  c.acc_empty = bars + 2 * STAGES + 2;
  c.drain = bars + 2 * STAGES + 4;
  c.xchg = bars + 2 * STAGES + 5;
  c.tmem_base = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);
  c.abort = reinterpret_cast<int*>(c.tmem_base + 1);
  c.flag = c.abort + 1;
  c.extra = base + L::kOffExtra;
  return c;
}

// Weight tiles of the first STAGES k-blocks of this CTA into fresh stages
// (no wait needed), issued by thread 0 right after the barriers are
// initialised, before TMEM allocation and before the predecessor kernel
// has finished. Returns how many stages were armed; gemm_producer adds
// their activation tiles after pdl_wait().
template <int BN, int STAGES, bool SWAP>
__device__ __forceinline__ int gemm_prefetch_weights(const GemmShape& g, const GemmCtl& c,
                                                     const CUtensorMap* tm_a, const CUtensorMap* tm_b,
                                                     uint64_t hint_w) {
  using L = GemmSmem<BN, STAGES>;
  int pre = 0;
  SegIter it0(g);
  Seg s0;
  while (pre < STAGES && it0.next(g, s0)) {
    for (int kb = s0.kb0; kb < s0.kb1 && pre < STAGES; ++kb, ++pre) {
      mbar_arrive_expect_tx(&c.full[pre], L::kStageBytes);
      if (SWAP)
        load_weight_tile<BN, SWAP>(g, tm_a, &c.full[pre], c.a + pre * L::kABytes, kb, s0, hint_w);
      else
        load_weight_tile<BN, SWAP>(g, tm_b, &c.full[pre], c.b + pre * L::kBBytes, kb, s0, hint_w);
    }
  }
  return pre;
}

// Producer: one thread. The weight operand (A in the swap orientation, B
// otherwise) does not depend on the previous kernel, so the first STAGES
// k-blocks' weight tiles are requested before pdl_wait(); the activation
// tiles of those stages follow once the predecessor has finished, then the
// steady-state loop streams both. after_wait() runs right after pdl_wait().
template <int BN, int STAGES, bool SWAP, typename AfterWait>
__device__ __forceinline__ void gemm_producer(const GemmShape& g, const GemmCtl& c,
                                              const CUtensorMap* tm_a, const CUtensorMap* tm_b,
                                              uint64_t hint_a, uint64_t hint_b, int pre,
                                              AfterWait&& after_wait) {
  using L = GemmSmem<BN, STAGES>;
  auto load_w = [&](int stage, int kb, const Seg& s) {
    if (SWAP)
      load_weight_tile<BN, SWAP>(g, tm_a, &c.full[stage], c.a + stage * L::kABytes, kb, s, hint_a);
    else
      load_weight_tile<BN, SWAP>(g, tm_b, &c.full[stage], c.b + stage * L::kBBytes, kb, s, hint_b);
  };
  auto load_x = [&](int stage, int kb, const Seg& s) {
    if (SWAP)
      tma_load_2d(tm_b, &c.full[stage], c.b + stage * L::kBBytes, kb * kBlockK, s.q * BN, hint_b);
    else
      tma_load_2d(tm_a, &c.full[stage], c.a + stage * L::kABytes, kb * kBlockK, s.p * kTileP, hint_a);
  };
  int issued[STAGES];
#pragma unroll
  for (int i = 0; i < STAGES; ++i) issued[i] = i < pre ? 0 : -1;
  (void)load_w;
  pdl_wait();
  after_wait();
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  int n_issued = 0;
  SegIter it(g);
  Seg tc;
  while (ok && it.next(g, tc)) {
    for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
      if (n_issued < pre) {
        load_x(stage, kb, tc);  // stage armed above
      } else {
        if (!mbar_wait(&c.empty[stage], phase ^ 1u, g.wait_ns, c.abort)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&c.full[stage], L::kStageBytes);
        load_w(stage, kb, tc);
        load_x(stage, kb, tc);
      }
      trace(n_issued < 200 ? n_issued : 1023);
      ++n_issued;
      issued[stage] = static_cast<int>(phase);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  if (!ok) {
    record_error(g.status, kDevTimeoutPipeline);
    *reinterpret_cast<volatile int*>(c.abort) = 1;
    // Let every load already in flight land before the CTA can retire.
    for (int i = 0; i < STAGES; ++i)
      if (issued[i] >= 0) (void)mbar_wait(&c.full[i], static_cast<uint32_t>(issued[i]), 10000000ull, nullptr);
  }
}

// MMA issuer: one thread.
template <int BN, int STAGES>
__device__ __forceinline__ void gemm_mma(const GemmShape& g, const GemmCtl& c, uint32_t idesc) {
  using L = GemmSmem<BN, STAGES>;
  // The first activation tiles arrive only after the predecessor kernel has
  // finished; start the bounded waits from there.
  pdl_wait();
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  const uint32_t tmem = *c.tmem_base;
  bool ok = true;
  bool any_commit = false;
  int n_full = 0;
  SegIter it(g);
  Seg tc;
  while (ok && it.next(g, tc)) {
    if (!mbar_wait(&c.acc_empty[acc], acc_phase ^ 1u, g.wait_ns, c.abort)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * BN);
    for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
      if (!mbar_wait(&c.full[stage], phase, g.wait_ns, c.abort)) {
        ok = false;
        break;
      }
      trace(n_full < 200 ? 200 + n_full : 1023);
      ++n_full;
      tc_fence_after();
      const uint64_t da = umma_desc_sw128_kmajor(smem_u32(c.a + stage * L::kABytes));
      const uint64_t db = umma_desc_sw128_kmajor(smem_u32(c.b + stage * L::kBBytes));
#pragma unroll
      for (int k = 0; k < kBlockK / 16; ++k) {
        // Advancing K by 16 elements = 32 bytes = 2 units of the address field.
        umma_f16_ss(d_tmem, da + static_cast<uint64_t>(2 * k), db + static_cast<uint64_t>(2 * k),
                    idesc, (kb > tc.kb0 || k > 0) ? 1u : 0u);
      }
      umma_commit(&c.empty[stage]);
      any_commit = true;
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (!ok) break;
    umma_commit(&c.acc_full[acc]);
    trace(404);
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1u;
    }
  }
  if (!ok) {
    record_error(g.status, kDevTimeoutPipeline);
    *reinterpret_cast<volatile int*>(c.abort) = 1;
    if (any_commit) {
      // No MMA may still read shared memory or write TMEM when the CTA
      // leaves: a commit tracks every earlier MMA of this thread.
      umma_commit(c.drain);
      (void)mbar_wait(c.drain, 0u, 10000000ull, nullptr);
    }
  }
}

// Epilogue helpers --------------------------------------------------------

// TMEM address of (lane quarter of this warp, column col) in accumulator acc.
__device__ __forceinline__ uint32_t epi_taddr(uint32_t tmem, int acc, int bn, int col) {
  const uint32_t quarter = static_cast<uint32_t>((threadIdx.x >> 5) & 3);
  return tmem + ((quarter * 32u) << 16) + static_cast<uint32_t>(acc * bn + col);
}

// Row of the 128-row tile owned by this epilogue thread (= its TMEM lane).
__device__ __forceinline__ int epi_row() {
  return static_cast<int>(((threadIdx.x >> 5) & 3) * 32 + (threadIdx.x & 31));
}

template <typename IO>
__device__ __forceinline__ IO f32_to_io(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 f32_to_io<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half f32_to_io<__half>(float v) {
  return __float2half_rn(v);
}
template <typename IO>
__device__ __forceinline__ float io_to_f32(IO v);
template <>
__device__ __forceinline__ float io_to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float io_to_f32<__half>(__half v) {
  return __half2float(v);
}

// Pack 8 f32 into 8 16-bit values (16 bytes).
template <typename IO>
__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 out;
  uint16_t h[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    IO t = f32_to_io<IO>(v[j]);
    h[j] = *reinterpret_cast<uint16_t*>(&t);
  }
  out.x = static_cast<uint32_t>(h[0]) | (static_cast<uint32_t>(h[1]) << 16);
  out.y = static_cast<uint32_t>(h[2]) | (static_cast<uint32_t>(h[3]) << 16);
  out.z = static_cast<uint32_t>(h[4]) | (static_cast<uint32_t>(h[5]) << 16);
  out.w = static_cast<uint32_t>(h[6]) | (static_cast<uint32_t>(h[7]) << 16);
  return out;
}

template <typename IO>
__device__ __forceinline__ void unpack8(uint4 u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint16_t lo = static_cast<uint16_t>(w[j] & 0xFFFFu), hi = static_cast<uint16_t>(w[j] >> 16);
    v[2 * j] = io_to_f32<IO>(*reinterpret_cast<IO*>(&lo));
    v[2 * j + 1] = io_to_f32<IO>(*reinterpret_cast<IO*>(&hi));
  }
}

// SiLU in f32 as the reference's activation computes it: silu_and_mul
// (python/picosgl/layers/activation.py:9-12) runs flashinfer's act_and_mul
// kernel, which evaluates x / (1 + exp(-x)) with the fast exponential and
// multiplies by the up value in f32.
__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + __expf(-x)); }

// The same with the quotient from the fast reciprocal (__fdividef: at most
// 2 ulp from the IEEE quotient for denominators up to 2^126, 0 beyond, where
// the quotient is below 2^-100). The GEMM epilogues use it: the IEEE division
// made the gated epilogue the longest part of a wide tile.
__device__ __forceinline__ float silu_f32_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// out[e] = silu(gate[e]) * up[e] for 8 packed 16-bit values, rounded once.
template <typename IO, bool FAST>
__device__ __forceinline__ uint4 silu_mul8(uint4 gate, uint4 up) {
  float gv[8], uv[8];
  unpack8<IO>(gate, gv);
  unpack8<IO>(up, uv);
#pragma unroll
  for (int e = 0; e < 8; ++e) gv[e] = (FAST ? silu_f32_fast(gv[e]) : silu_f32(gv[e])) * uv[e];
  return pack8<IO>(gv);
}

// Row of the merged weight (and bias) that tile row `row` of swap-orientation
// tile p holds, or -1 past the end. Gated mode: rows 0..63 are the gate rows
// of output features p * 64 .., rows 64..127 the up rows of the same features.
template <bool GLU>
__device__ __forceinline__ int swap_weight_row(const GemmShape& g, int p, int row) {
  if constexpr (GLU) {
    const int f = p * (kTileP / 2) + (row & (kTileP / 2 - 1));
    return f < g.N ? (row < kTileP / 2 ? f : g.N + f) : -1;
  } else {
    const int n = p * kTileP + row;
    return n < g.N ? n : -1;
  }
}

// Load 32 accumulator columns [col, col + 32) of accumulator acc.
template <int BN>
__device__ __forceinline__ void epi_load_chunk(uint32_t tmem, int acc, int col, float* v) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(epi_taddr(tmem, acc, BN, col), r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// Swap orientation: this thread holds v[j] = out(tile row `row`, token
// t0 + j), j < 32. Stage the 32 x 128 block, rounded to IO, through shared
// memory as epi[token j][tile row] so it can leave as 16-byte pieces of token
// rows. All 128 epilogue threads call this together; a readout follows.
template <typename IO>
__device__ __forceinline__ void swap_stage(uint16_t* epi, const float* v) {
  const int row = epi_row();
  named_bar_sync(1, kEpiThreads);  // previous chunk fully read
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    IO h = f32_to_io<IO>(v[j]);
    epi[j * kTileP + row] = *reinterpret_cast<uint16_t*>(&h);
  }
  named_bar_sync(1, kEpiThreads);
}

// Index of this thread among the 128 epilogue threads.
__device__ __forceinline__ int epi_tid() { return static_cast<int>(threadIdx.x) - (kGemmThreads - kEpiThreads); }

// Readout of a staged chunk: emit(t, n0, piece) receives the 8 consecutive
// features [n0, n0 + 8) of token t = t0 + j, for tokens in [t_lo, t_hi) and
// n0 < N (tile row r is feature n_base + r).
template <typename Emit>
__device__ __forceinline__ void swap_readout(const uint16_t* epi, int t0, int t_lo, int t_hi, int n_base, int N,
                                             Emit&& emit) {
  const int tid = epi_tid();
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int idx = tid + k * kEpiThreads;  // 512 pieces: 32 tokens x 16 pieces
    const int j = idx >> 4, piece = idx & 15;
    const int t = t0 + j, n0 = n_base + piece * 8;
    if (t >= t_lo && t < t_hi && n0 < N) emit(t, n0, *reinterpret_cast<const uint4*>(epi + j * kTileP + piece * 8));
  }
}

// Gated readout: tile rows 0..63 hold gate and rows 64..127 up values of the
// 64 features [n_base, n_base + 64), already rounded to IO by swap_stage (the
// reference materialises gate_up in IO); a piece is silu(gate) * up.
template <typename IO, typename Emit>
__device__ __forceinline__ void swap_readout_glu(const uint16_t* epi, int t0, int t_lo, int t_hi, int n_base, int N,
                                                 Emit&& emit) {
  const int tid = epi_tid();
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int idx = tid + k * kEpiThreads;  // 256 pieces: 32 tokens x 8 pieces
    const int j = idx >> 3, piece = idx & 7;
    const int t = t0 + j, n0 = n_base + piece * 8;
    const uint16_t* src = epi + j * kTileP + piece * 8;
    if (t >= t_lo && t < t_hi && n0 < N)
      emit(t, n0, silu_mul8<IO, true>(*reinterpret_cast<const uint4*>(src),
                                      *reinterpret_cast<const uint4*>(src + kTileP / 2)));
  }
}

// swap_stage followed by the plain readout.
template <typename IO, typename Emit>
__device__ __forceinline__ void swap_epilogue_store(uint16_t* epi, const float* v, int t0, int t_lo, int t_hi,
                                                    int n_base, int N, Emit&& emit) {
  swap_stage<IO>(epi, v);
  swap_readout(epi, t0, t_lo, t_hi, n_base, N, emit);
}

// Split tile (swap orientation), called by the 128 epilogue threads of each
// of the tile's nsplit CTAs with its partial accumulator `acc` over its own
// k-range. The tile's real token columns are cut into nsplit runs
// (split_cols), one per CTA. Each CTA
//   1. stores its partial for the columns the other CTAs own into its slab of
//      the exchange area (token-major f32: a warp writes 128 contiguous bytes
//      per token) and publishes it with one release on the tile's counter;
//   2. once all nsplit CTAs have published, bulk-copies (cp.async.bulk, off
//      the load/store unit) the others' pieces of its own columns into its
//      pipeline ring, which is idle after its last MMA;
//   3. sums its columns in split order (its own values were parked in its
//      ring in step 1), adds this thread's row bias `bias_v` once and hands
//      each 32-token chunk to store_chunk(v, t0, t_lo, t_hi) (all 128
//      threads together, as the whole-tile epilogue does: v[j] is token
//      t0 + j, tokens outside [t_lo, t_hi) are not stored);
//   4. bumps the tile's second counter; the last CTA to finish resets both,
//      so the counters are zero again for the next launch.
// Returns false (and records an error) if a wait runs out.
template <int BN, typename StoreChunk>
__device__ __forceinline__ bool split_reduce_tile(const GemmShape& g, const Seg& sg, const GemmCtl& c, uint32_t tmem,
                                                  int acc, float bias_v, StoreChunk&& store_chunk) {
  const int S = sg.nctb, j = sg.contrib, u = sg.tile - g.split_first;
  const int row = epi_row();
  const int tid = static_cast<int>(threadIdx.x) - (kGemmThreads - kEpiThreads);
  const int t_base = sg.q * BN;
  const int V = min(BN, g.T - t_base);
  const size_t slab = static_cast<size_t>(BN) * kTileP;
  uint32_t* ctr = g.ctr + 2 * u;
  int my0, my1;
  split_cols(BN, V, S, j, my0, my1);
  bool ok = true;

  // 1. This CTA's partial: the other CTAs' columns to its exchange slab, its
  //    own columns to slot j of the gather area in its ring (idle after the
  //    last MMA), laid out [S][n_mine][128] f32.
  const int n_mine = my1 - my0;
  float* recv = reinterpret_cast<float*>(c.a);
  float* mine = g.xchg + static_cast<size_t>(u * S + j) * slab;
  float* own = recv + static_cast<size_t>(j) * n_mine * kTileP + row;
  if (tid == 0) trace(400);
#pragma unroll 1
  for (int cb = 0; cb < V; cb += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(epi_taddr(tmem, acc, BN, cb), r);
    tmem_ld_wait();
    if (tid == 0 && cb < 128) trace(405 + (cb >> 4));
    const int nv = min(32, V - cb);  // real tokens in this chunk
    if (cb >= my0 && cb + nv <= my1) {
      // Every real token of the chunk is this CTA's: park them in its slot
      // of the gather area.
      float* o = own + static_cast<size_t>(cb - my0) * kTileP;
      if (nv == 32) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) o[jj * kTileP] = __uint_as_float(r[jj]);
      } else if (nv <= 8) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          if (jj < nv) o[jj * kTileP] = __uint_as_float(r[jj]);
      } else {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          if (jj < nv) o[jj * kTileP] = __uint_as_float(r[jj]);
      }
    } else if (cb + nv <= my0 || cb >= my1) {
      // Every real token of the chunk is other CTAs': to this CTA's slab.
      float* m = mine + static_cast<size_t>(cb) * kTileP + row;
      if (nv == 32) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) __stcg(m + jj * kTileP, __uint_as_float(r[jj]));
      } else if (nv <= 8) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          if (jj < nv) __stcg(m + jj * kTileP, __uint_as_float(r[jj]));
      } else {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          if (jj < nv) __stcg(m + jj * kTileP, __uint_as_float(r[jj]));
      }
    } else {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int col = cb + jj;
        const float x = __uint_as_float(r[jj]);
        const bool is_mine = col >= my0 && col < my1;
        if (is_mine) own[static_cast<size_t>(col - my0) * kTileP] = x;
        if (!is_mine && col < V) __stcg(mine + static_cast<size_t>(col) * kTileP + row, x);
      }
    }
    if (tid == 0 && cb < 128) trace(406 + (cb >> 4));
  }
  // bar.sync, then one gpu-scope release: every thread's stores are ordered
  // before the publication.
  if (tid == 0) trace(402);
  named_bar_sync(1, kEpiThreads);
  if (tid == 0) {
    trace(403);
    atom_add_acqrel_gpu(ctr, 1u);
    trace(1011);
  }

  // 2. Gather the other CTAs' pieces of this CTA's columns into their slots.
  if (n_mine > 0) {
    if (tid == 0) {
      int okw = 1;
      Deadline d(g.wait_ns);
      volatile int* st = g.status;
      while (ld_acquire_gpu(ctr) < static_cast<uint32_t>(S)) {
        if (d.expired()) {
          record_error(g.status, kDevTimeoutGrid);
          okw = 0;
          break;
        }
        if ((d.n & 255u) == 0u && *st != 0) {
          okw = 0;
          break;
        }
      }
      if (okw) {
        fence_proxy_async_global();  // the bulk copies read what the acquire made visible
        const uint32_t piece = static_cast<uint32_t>(n_mine) * kTileP * 4u;
        mbar_arrive_expect_tx(c.xchg, piece * static_cast<uint32_t>(S - 1));
        for (int q = 0; q < S; ++q) {
          if (q == j) continue;
          bulk_g2s(recv + static_cast<size_t>(q) * n_mine * kTileP,
                   g.xchg + static_cast<size_t>(u * S + q) * slab + static_cast<size_t>(my0) * kTileP, piece, c.xchg);
        }
        if (!mbar_wait(c.xchg, 0u, g.wait_ns, nullptr)) {
          record_error(g.status, kDevTimeoutPipeline);
          okw = 0;
        }
      }
      *c.flag = okw;
      trace(1012);
    }
    named_bar_sync(1, kEpiThreads);
    ok = *reinterpret_cast<volatile int*>(c.flag) != 0;
  }

  // 3. Sum the S slots in split order, add the bias, round, store. Shared
  //    memory only and branch-free: token indices past this CTA's run are
  //    clamped (those lanes of the staging tile are not emitted).
  if (ok && n_mine > 0) {
    const float* base = recv + row;
#pragma unroll 1
    for (int c0 = 0; c0 < n_mine; c0 += 32) {
      if (tid == 0 && c0 == 0) trace(1014);
      const int lim = n_mine - 1 - c0;
      float v[32];
      const float* s0 = base + static_cast<size_t>(c0) * kTileP;
      if (lim >= 31) {
        // A full chunk: constant offsets.
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) v[jj] = s0[jj * kTileP];
#pragma unroll 1
        for (int q = 1; q < S; ++q) {
          const float* sq = base + (static_cast<size_t>(q) * n_mine + c0) * kTileP;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) v[jj] += sq[jj * kTileP];
        }
      } else if (lim < 8) {
        // A short run (decode batches of up to 8 tokens): 8 columns at most;
        // tokens past it read as 0 (those lanes of the staging tile are not
        // emitted).
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) v[jj] = 0.f;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          if (jj <= lim) v[jj] = s0[jj * kTileP];
#pragma unroll 1
        for (int q = 1; q < S; ++q) {
          const float* sq = base + (static_cast<size_t>(q) * n_mine + c0) * kTileP;
#pragma unroll
          for (int jj = 0; jj < 8; ++jj)
            if (jj <= lim) v[jj] += sq[jj * kTileP];
        }
      } else {
        // The run's last, partial chunk: tokens past it read as 0 (those
        // lanes of the staging tile are not emitted).
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) v[jj] = jj <= lim ? s0[jj * kTileP] : 0.f;
#pragma unroll 1
        for (int q = 1; q < S; ++q) {
          const float* sq = base + (static_cast<size_t>(q) * n_mine + c0) * kTileP;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (jj <= lim) v[jj] += sq[jj * kTileP];
        }
      }
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) v[jj] += bias_v;
      if (tid == 0 && c0 == 0) trace(1015);
      store_chunk(v, t_base + my0 + c0, t_base + my0, t_base + my1);
      if (tid == 0 && c0 == 0) trace(1016);
    }
  }

  // 4. The last CTA of the tile to finish resets its counters. Relaxed: each
  //    CTA's poll of the first counter and its gather have completed before
  //    its increment (program order, bar.sync), so the reset cannot reach a
  //    wait still in progress, and the next launch sees it across the kernel
  //    boundary. No release is needed, so the output stores need not drain
  //    first.
  named_bar_sync(1, kEpiThreads);
  if (tid == 0) {
    trace(1013);
    const uint32_t old = atom_add_relaxed_gpu(ctr + 1, 1u);
    if (old == static_cast<uint32_t>(S) - 1u) {
      ctr[0] = 0u;
      ctr[1] = 0u;
    }
  }
  return ok;
}

}  // namespace pgb
