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
// Shared tiles (stream-K, see GemmShape): a CTA that covers only part of a
// tile's K range stores its f32 partial; after a grid barrier all warps sum
// the partials of every shared tile in contributor order.
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
// [0, sk_first) are whole tiles dealt round-robin: CTA c computes tiles
// c, c + grid, ... (dp_rounds of them at most). Tiles [sk_first, tiles) are
// stream-K tiles: their k-blocks are laid end to end and CTA c takes the
// contiguous range [c*total/grid, (c+1)*total/grid) of them, cut at tile
// boundaries into segments. With sk_first = dp_rounds * grid every CTA
// streams the same number of k-blocks (+-1), so no SM idles while others
// finish a last partial wave. A stream-K tile shared by several CTAs is
// finished after a grid barrier (cooperative launch) by all warps together,
// adding the contributors' f32 partials in contributor order, so the result
// does not depend on timing.
//
// Cluster split-K (csk > 1) replaces both: the grid is made of clusters of
// csk CTAs, cluster c computes tiles c, c + n_clusters, ..., and CTA r of the
// cluster streams k-blocks [r*kblocks/csk, (r+1)*kblocks/csk) of each. The
// csk partial accumulators are summed through distributed shared memory
// (cluster_reduce_tile), so no partial leaves the chip.
struct GemmShape {
  int T, N, K;
  int kblocks;      // ceil(K / 64)
  int p_tiles;      // tiles along the MMA M side
  int q_tiles;      // tiles along the MMA N side
  int tiles;        // p_tiles * q_tiles
  int dp_rounds;    // whole tiles per CTA before the stream-K part
  int sk_first;     // first stream-K tile (== tiles: no stream-K part)
  int grid;         // CTAs taking part in the round-robin part (<= gridDim.x)
  int sk_grid;      // CTAs taking part in the stream-K part, <= grid and <=
                    // its k-block count, so every stream-K range is non-empty
  int max_contrib;  // partial slabs reserved per stream-K tile
  int csk;          // > 1: cluster split-K with this cluster size (see SegIter)
  int n_clusters;   // clusters in the launch when csk > 1
  float* ws;        // partials [tiles - sk_first][max_contrib][BN tokens][128 features] f32
  int* status;      // device status word (first error wins); the grid
                    // barrier's counters follow it at +64 and +128 bytes
  uint64_t wait_ns; // budget for every intra-kernel wait
};

// One contiguous piece of a tile's reduction handled by this CTA.
struct Seg {
  int tile, p, q;
  int kb0, kb1;   // k-block range [kb0, kb1)
  int contrib;    // index of this CTA among the tile's contributors
  int nctb;       // number of contributors (1 = this CTA owns the whole tile)
};

// CTA whose stream-K range contains stream-K k-block u.
__host__ __device__ __forceinline__ int streamk_cta_of(long long u, long long total, int grid) {
  return static_cast<int>(((u + 1) * grid - 1) / total);
}

__host__ __device__ __forceinline__ long long streamk_total(const GemmShape& g) {
  return static_cast<long long>(g.tiles - g.sk_first) * g.kblocks;
}

// Iterates the segments of CTA `cta` in order: its whole tiles, then its
// stream-K range. All roles of a CTA walk the same sequence. Host-callable
// so the decomposition can be checked without a GPU.
struct SegIter {
  long long u, u1, total;
  int t, round, cta;
  int ckb0, ckb1;  // cluster split-K: this CTA's k-range of every tile
  __host__ __device__ __forceinline__ SegIter(const GemmShape& g, int cta_) {
    cta = cta_;
    if (g.csk > 1) {
      const int cl = cta / g.csk, r = cta % g.csk;
      t = cl < g.n_clusters ? cl : g.tiles;
      ckb0 = r * g.kblocks / g.csk;
      ckb1 = (r + 1) * g.kblocks / g.csk;
      round = 0;
      u = u1 = total = 0;
      return;
    }
    ckb0 = ckb1 = 0;
    total = streamk_total(g);
    round = 0;
    t = cta;
    if (cta < g.sk_grid && total > 0) {
      u = total * cta / g.sk_grid;
      u1 = total * (cta + 1) / g.sk_grid;
    } else {  // no stream-K part, or a CTA beyond the stream-K grid
      u = u1 = 0;
    }
    if (cta >= g.grid) round = g.dp_rounds;
  }
  __device__ __forceinline__ explicit SegIter(const GemmShape& g) : SegIter(g, static_cast<int>(blockIdx.x)) {}
  __host__ __device__ __forceinline__ bool next(const GemmShape& g, Seg& s) {
    if (g.csk > 1) {
      if (t >= g.tiles) return false;
      s.tile = t;
      s.kb0 = ckb0;
      s.kb1 = ckb1;
      s.contrib = cta % g.csk;
      s.nctb = g.csk;
      s.p = t % g.p_tiles;
      s.q = t / g.p_tiles;
      t += g.n_clusters;
      return true;
    }
    if (round < g.dp_rounds) {
      s.tile = t + round * g.grid;
      ++round;
      if (s.tile < g.sk_first) {
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
    if (u >= u1) return false;
    const int rel = static_cast<int>(u / g.kblocks);
    s.tile = g.sk_first + rel;
    s.kb0 = static_cast<int>(u - static_cast<long long>(rel) * g.kblocks);
    const long long rem = u1 - u;
    s.kb1 = rem < static_cast<long long>(g.kblocks - s.kb0) ? s.kb0 + static_cast<int>(rem) : g.kblocks;
    u += s.kb1 - s.kb0;
    const long long first = static_cast<long long>(rel) * g.kblocks;
    const int c0 = streamk_cta_of(first, total, g.sk_grid);
    const int c1 = streamk_cta_of(first + g.kblocks - 1, total, g.sk_grid);
    s.contrib = cta - c0;
    s.nctb = c1 - c0 + 1;
    s.p = s.tile % g.p_tiles;
    s.q = s.tile / g.p_tiles;
    return true;
  }
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kTileP * kBlockK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kBlockK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
  // Layout (from a 1024-byte aligned base): A ring, B ring, barriers.
  static constexpr int kOffA = 0;
  static constexpr int kOffB = STAGES * kABytes;
  static constexpr int kOffEpi = kOffB + STAGES * kBBytes;
  static constexpr int kEpiBytes = 32 * kTileP * 2;  // 32 tokens x 128 features, 16-bit
  static constexpr int kOffRed = kOffEpi + kEpiBytes;
  static constexpr int kRedBytes = 32 * kTileP * 4;  // cluster split-K chunk: 32 tokens x 128 f32
  static constexpr int kOffBar = kOffRed + kRedBytes;
  static constexpr int kBarBytes = 8 * (2 * STAGES + 7) + 64;
  static constexpr int kBytes = kOffBar + kBarBytes + 1024;  // + alignment slack
};

// Pipeline depth that fills the shared-memory budget for a tile width.
template <int BN>
constexpr int gemm_stages() {
  constexpr int kBudget = 200 * 1024;  // leaves room for the epilogue tiles and barriers
  constexpr int kStage = kTileP * kBlockK * 2 + BN * kBlockK * 2;
  return kBudget / kStage > 12 ? 12 : kBudget / kStage;
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
  float* red;     // [32][128] f32 chunk exchanged by cluster split-K
  uint64_t* red_ready;  // all csk chunks of the cluster are written
  uint64_t* red_free;   // all csk CTAs finished reading this CTA's chunk
};

template <int BN, int STAGES>
__device__ __forceinline__ GemmCtl gemm_carve_smem(uint8_t* raw) {
  using L = GemmSmem<BN, STAGES>;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  GemmCtl c;
  c.a = base + L::kOffA;
  c.b = base + L::kOffB;
  c.epi = reinterpret_cast<uint16_t*>(base + L::kOffEpi);
  c.red = reinterpret_cast<float*>(base + L::kOffRed);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::kOffBar);
  c.full = bars;
  c.empty = bars + STAGES;
  c.acc_full = bars + 2 * STAGES;
  c.acc_empty = bars + 2 * STAGES + 2;
  c.drain = bars + 2 * STAGES + 4;
  c.red_ready = bars + 2 * STAGES + 5;
  c.red_free = bars + 2 * STAGES + 6;
  c.tmem_base = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 7);
  c.abort = reinterpret_cast<int*>(c.tmem_base + 1);
  c.flag = c.abort + 1;
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
        tma_load_2d(tm_a, &c.full[pre], c.a + pre * L::kABytes, kb * kBlockK, s0.p * kTileP, hint_w);
      else
        tma_load_2d(tm_b, &c.full[pre], c.b + pre * L::kBBytes, kb * kBlockK, s0.q * BN, hint_w);
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
      tma_load_2d(tm_a, &c.full[stage], c.a + stage * L::kABytes, kb * kBlockK, s.p * kTileP, hint_a);
    else
      tma_load_2d(tm_b, &c.full[stage], c.b + stage * L::kBBytes, kb * kBlockK, s.q * BN, hint_b);
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

// Load 32 accumulator columns [col, col + 32) of accumulator acc.
template <int BN>
__device__ __forceinline__ void epi_load_chunk(uint32_t tmem, int acc, int col, float* v) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(epi_taddr(tmem, acc, BN, col), r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// Number of CTAs contributing to `tile` (1 for whole tiles).
__host__ __device__ __forceinline__ int tile_contributors(const GemmShape& g, int tile) {
  if (g.csk > 1) return g.csk;
  if (tile < g.sk_first) return 1;
  const long long total = streamk_total(g);
  const long long first = static_cast<long long>(tile - g.sk_first) * g.kblocks;
  return streamk_cta_of(first + g.kblocks - 1, total, g.sk_grid) - streamk_cta_of(first, total, g.sk_grid) + 1;
}

// Token-major f32 partial of stream-K tile `tile`, contributor j, in swap
// orientation: [BN tokens][128 features]. A warp stores 128 contiguous bytes
// per token, and the reduction phase reads 8 consecutive features of a token
// as two float4.
template <int BN>
__device__ __forceinline__ float* partial_tm(const GemmShape& g, int tile, int j) {
  return g.ws + (static_cast<size_t>(tile - g.sk_first) * g.max_contrib + j) * BN * kTileP;
}

// Store this segment's accumulator (acc) as a token-major f32 partial.
// Called by the 128 epilogue threads; tokens >= T are skipped.
template <int BN>
__device__ __forceinline__ void partial_store_tm(const GemmShape& g, const Seg& sg, uint32_t tmem,
                                                 int acc) {
  const int row = epi_row();
  if (sg.contrib < 0 || sg.contrib >= g.max_contrib || sg.tile < g.sk_first) {
    // Never store outside the reserved slabs; report instead.
    if (row == 0) record_error(g.status, kDevBadArgs);
    return;
  }
  float* dst = partial_tm<BN>(g, sg.tile, sg.contrib);
#pragma unroll 1
  for (int col = 0; col < BN; col += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(epi_taddr(tmem, acc, BN, col), r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = sg.q * BN + col + j;
      if (t < g.T) __stcg(dst + static_cast<size_t>(col + j) * kTileP + row, __uint_as_float(r[j]));
    }
  }
}

// Grid-wide barrier for a cooperative launch on one GPU. arrive/gen live in
// global memory and are zero at rest; the last CTA to arrive resets the
// counter and bumps the generation. Bounded: returns false (and records an
// error) when the wait runs out or another CTA already failed.
__device__ __forceinline__ bool grid_barrier_local(uint32_t* arrive, uint32_t* gen, int* status,
                                                   uint64_t wait_ns) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint32_t g0 = ld_acquire_gpu(gen);
    __threadfence();
    const uint32_t old = atom_add_acqrel_gpu(arrive, 1u);
    if (old == gridDim.x - 1) {
      *arrive = 0u;
      __threadfence();
      st_release_gpu(gen, g0 + 1u);
    } else {
      Deadline d(wait_ns);
      volatile int* st = status;
      while (ld_acquire_gpu(gen) == g0) {
        if (d.expired()) {
          record_error(status, kDevTimeoutGrid);
          ok = 0;
          break;
        }
        if ((d.n & 255u) == 0u && *st != 0) {
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Cluster split-K reduction of one tile (swap orientation). Every one of the
// 128 epilogue threads of every CTA of the cluster calls this for the same
// tile, with its own partial accumulator `acc`. Per 32-token chunk: each CTA
// writes its partial to its shared `red` buffer (token-major), signals the
// cluster, then reduces its share of the feature groups over the csk buffers
// in CTA-rank order through DSMEM and hands every finished 4-feature piece to
// emit(t, n0, float4), then signals that it is done reading. `seq` counts
// chunks across tiles (mbarrier parities). Only the epilogue warps take part,
// so the producer and MMA warps keep streaming the next tile meanwhile.
template <int BN, typename Emit4>
__device__ __forceinline__ bool cluster_reduce_tile(const GemmShape& g, const Seg& sg, const GemmCtl& c,
                                                    uint32_t tmem, int acc, uint32_t& seq, Emit4&& emit) {
  const int C = g.csk;
  const int rank = static_cast<int>(blockIdx.x) % C;
  const int row = epi_row();
  const int tid = static_cast<int>(threadIdx.x) - (kGemmThreads - kEpiThreads);
  const int g0 = rank * (kTileP / 4) / C, g1 = (rank + 1) * (kTileP / 4) / C;
  const int ng = g1 - g0;
  bool ok = true;
#pragma unroll 1
  for (int col = 0; col < BN; col += 32) {
    if (seq > 0 && !mbar_wait_cluster(c.red_free, (seq - 1) & 1u, g.wait_ns)) ok = false;
    uint32_t r[32];
    tmem_ld_32x32b_x32(epi_taddr(tmem, acc, BN, col), r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) c.red[j * kTileP + row] = __uint_as_float(r[j]);
    named_bar_sync(1, kEpiThreads);
    // One thread per destination CTA arrives, so the C release-arrives are in
    // flight together; each releases at cluster scope, and the named barrier
    // above orders every thread's buffer writes before it.
    if (tid == 0) trace(1010);
    if (tid < C) mbar_arrive_cluster(dsmem_addr(c.red_ready, tid));
    if (tid == 0) trace(1011);
    if (!mbar_wait_cluster(c.red_ready, seq & 1u, g.wait_ns)) ok = false;
    if (tid == 0) trace(1012);
    if (ok) {
      const int items = 32 * ng;
      for (int it0 = tid; it0 < items; it0 += 2 * kEpiThreads) {
        // Two items per pass: all 2*C DSMEM loads in flight before the adds.
        float4 v[2][8];
        int jj[2], gg[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int it = it0 + k * kEpiThreads;
          jj[k] = it < items ? it / ng : -1;
          gg[k] = it < items ? g0 + it % ng : 0;
          if (jj[k] >= 0) {
            const float* my = c.red + jj[k] * kTileP + gg[k] * 4;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (q < C) v[k][q] = ld_dsmem_f4(dsmem_addr(my, q));
          }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (jj[k] < 0) continue;
          float4 a = v[k][0];
#pragma unroll
          for (int q = 1; q < 8; ++q) {
            if (q < C) {
              a.x += v[k][q].x;
              a.y += v[k][q].y;
              a.z += v[k][q].z;
              a.w += v[k][q].w;
            }
          }
          const int t = sg.q * BN + col + jj[k], n0 = sg.p * kTileP + gg[k] * 4;
          if (t < g.T && n0 < g.N) emit(t, n0, a);
        }
      }
    }
    named_bar_sync(1, kEpiThreads);
    if (tid == 0) trace(1013);
    if (tid < C) mbar_arrive_cluster(dsmem_addr(c.red_free, tid));
    ++seq;
  }
  if (!ok) record_error(g.status, kDevTimeoutPipeline);
  return ok;
}

// Before a CTA of a split-K cluster retires, every CTA of the cluster must
// have finished reading its reduction buffer.
__device__ __forceinline__ void cluster_reduce_drain(const GemmShape& g, const GemmCtl& c, uint32_t seq) {
  if (g.csk > 1 && seq > 0 && !mbar_wait_cluster(c.red_free, (seq - 1) & 1u, g.wait_ns))
    record_error(g.status, kDevTimeoutPipeline);
  if (threadIdx.x == kGemmThreads - kEpiThreads) trace(1014);
}

// Swap orientation: this thread holds v[j] = out(feature p*128 + row,
// token t0 + j), j < 32. Stage the 32 x 128 block through shared memory so
// it leaves as 16-byte pieces of token rows. emit(t, n0, piece) receives
// 8 consecutive features [n0, n0 + 8) of token t. All 128 epilogue threads
// call this together.
template <typename IO, typename Emit>
__device__ __forceinline__ void swap_epilogue_store(uint16_t* epi, const float* v, int t0, int T,
                                                    int n_base, int N, Emit&& emit) {
  const int row = epi_row();
  named_bar_sync(1, kEpiThreads);  // previous chunk fully read
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    IO h = f32_to_io<IO>(v[j]);
    epi[j * kTileP + row] = *reinterpret_cast<uint16_t*>(&h);
  }
  named_bar_sync(1, kEpiThreads);
  const int tid = static_cast<int>(threadIdx.x) - (kGemmThreads - kEpiThreads);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int idx = tid + k * kEpiThreads;  // 512 pieces: 32 tokens x 16 pieces
    const int j = idx >> 4, piece = idx & 15;
    const int t = t0 + j, n0 = n_base + piece * 8;
    if (t < T && n0 < N) emit(t, n0, *reinterpret_cast<const uint4*>(epi + j * kTileP + piece * 8));
  }
}

}  // namespace pgb
