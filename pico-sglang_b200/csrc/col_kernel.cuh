// col_kernel.cuh - the column-parallel GEMM kernel and its epilogue policies.
//
// y = x[T, K] . W^T on the tcgen05 core (gemm_sm100.cuh); what happens to the
// f32 accumulators is the epilogue policy's business:
//   EpiPlain : y[T, N] (+ bias), LinearTPImpl.forward for the column layers
//              (python/picosgl/layers/linear.py:23-27, 45-73);
//   EpiGlu   : silu(gate) * up for the merged [gate; up] weight, GatedMLP's
//              gate_up_proj + act_fn (python/picosgl/layers/mlp.py:43-46);
//   EpiRope  : (qkv_rope.cu) RoPE on q and k heads, q to its tensor and k, v
//              into the paged KV cache (python/picosgl/layers/attention.py:94-117
//              followed by MHAKVCachePool.store_kv).
//
// A policy is a trivially copyable struct passed to the kernel as a
// __grid_constant__ parameter, with (all 128 epilogue threads call each
// member together):
//   static constexpr bool kGlu        weight tiles are gate / up halves
//   static constexpr int kSmemBytes   shared memory the policy needs (c.extra)
//   template <bool SWAP> void prepare(g, c)
//                                     once, before the first accumulator is
//                                     ready (the main loop is still running)
//   float row_bias(g, p, row)         swap orientation: bias of tile row `row`
//   void swap_chunk(g, c, v, p, t0, t_lo, t_hi)
//                                     swap orientation: v[j] is tile row `row`
//                                     of token t0 + j; store tokens [t_lo, t_hi)
//   template <int BN> void nonswap_tile(g, tmem, acc, p, q)
//                                     prefill orientation: the whole tile
#pragma once

#include "gemm_plan.h"
#include "gemm_sm100.cuh"
#include "host_common.h"

namespace pgb {

template <typename IO>
struct EpiPlain {
  static constexpr bool kGlu = false;
  static constexpr int kSmemBytes = 0;
  IO* y;
  const IO* bias;

  template <bool SWAP>
  __device__ __forceinline__ void prepare(const GemmShape&, const GemmCtl&) const {}
  __device__ __forceinline__ float row_bias(const GemmShape& g, int p, int row) const {
    const int n = swap_weight_row<false>(g, p, row);
    return (bias != nullptr && n >= 0) ? io_to_f32<IO>(bias[n]) : 0.f;
  }
  __device__ __forceinline__ void swap_chunk(const GemmShape& g, const GemmCtl& c, const float* v, int p, int t0,
                                             int t_lo, int t_hi) const {
    IO* out = y;
    const int N = g.N;
    swap_stage<IO>(c.epi, v);
    swap_readout(c.epi, t0, t_lo, t_hi, p * kTileP, N, [&](int t, int n0, uint4 piece) {
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * N + n0) = piece;
    });
  }
  // Lane = token t, columns = output features.
  template <int BN>
  __device__ __forceinline__ void nonswap_tile(const GemmShape& g, uint32_t tmem, int acc, int p, int q) const {
    const int t = p * kTileP + epi_row();
#pragma unroll 1
    for (int col = 0; col < BN; col += 32) {
      float v[32];
      epi_load_chunk<BN>(tmem, acc, col, v);
      const int n0 = q * BN + col;
      if (t < g.T) {
        IO* dst = y + static_cast<size_t>(t) * g.N + n0;
        if (bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < g.N) v[j] += io_to_f32<IO>(bias[n0 + j]);
        }
        if (n0 + 32 <= g.N) {
#pragma unroll
          for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst)[j] = pack8<IO>(v + 8 * j);
        } else {
          for (int j = 0; j < 32 && n0 + j < g.N; ++j) dst[j] = f32_to_io<IO>(v[j]);
        }
      }
    }
  }
};

// Gated: g.N is the gated width I, the weight [gate; up] has 2I rows and the
// bias (if any) 2I entries.
template <typename IO>
struct EpiGlu {
  static constexpr bool kGlu = true;
  static constexpr int kSmemBytes = 0;
  IO* y;
  const IO* bias;

  template <bool SWAP>
  __device__ __forceinline__ void prepare(const GemmShape&, const GemmCtl&) const {}
  __device__ __forceinline__ float row_bias(const GemmShape& g, int p, int row) const {
    const int n = swap_weight_row<true>(g, p, row);
    return (bias != nullptr && n >= 0) ? io_to_f32<IO>(bias[n]) : 0.f;
  }
  __device__ __forceinline__ void swap_chunk(const GemmShape& g, const GemmCtl& c, const float* v, int p, int t0,
                                             int t_lo, int t_hi) const {
    IO* out = y;
    const int N = g.N;
    swap_stage<IO>(c.epi, v);
    swap_readout_glu<IO>(c.epi, t0, t_lo, t_hi, p * (kTileP / 2), N, [&](int t, int n0, uint4 piece) {
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * N + n0) = piece;
    });
  }
  // Lane = token t; columns [0, BN/2) are the gate and [BN/2, BN) the up
  // values of output features q * BN/2 ... Each is rounded to IO (the
  // reference materialises gate_up) before silu(gate) * up.
  template <int BN>
  __device__ __forceinline__ void nonswap_tile(const GemmShape& g, uint32_t tmem, int acc, int p, int q) const {
    const int t = p * kTileP + epi_row();
#pragma unroll 1
    for (int col = 0; col < BN / 2; col += 32) {
      float gv[32], uv[32];
      epi_load_chunk<BN>(tmem, acc, col, gv);
      epi_load_chunk<BN>(tmem, acc, BN / 2 + col, uv);
      const int f0 = q * (BN / 2) + col;
      if (t < g.T) {
        if (bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (f0 + j < g.N) {
              gv[j] += io_to_f32<IO>(bias[f0 + j]);
              uv[j] += io_to_f32<IO>(bias[g.N + f0 + j]);
            }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
          gv[j] = silu_f32_fast(io_to_f32<IO>(f32_to_io<IO>(gv[j]))) * io_to_f32<IO>(f32_to_io<IO>(uv[j]));
        IO* dst = y + static_cast<size_t>(t) * g.N + f0;
        if (f0 + 32 <= g.N) {
#pragma unroll
          for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst)[j] = pack8<IO>(gv + 8 * j);
        } else {
          for (int j = 0; j < 32 && f0 + j < g.N; ++j) dst[j] = f32_to_io<IO>(gv[j]);
        }
      }
    }
  }
};

template <typename IO, int BN, bool SWAP, int STAGES, typename Epi>
__global__ void __launch_bounds__(kGemmThreads, gemm_ctas_per_sm(BN))
    col_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    GemmShape g, const __grid_constant__ Epi epi) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_pre;  // stages armed with weight tiles before pdl_wait()
  GemmCtl c = gemm_carve_smem<BN, STAGES, Epi::kSmemBytes>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    trace(1000);
    tma_prefetch_desc(&tm_a);  // descriptor fetch overlaps barrier set-up
    tma_prefetch_desc(&tm_b);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    mbar_init(&c.acc_full[0], 1);
    mbar_init(&c.acc_full[1], 1);
    mbar_init(&c.acc_empty[0], kEpiThreads);
    mbar_init(&c.acc_empty[1], kEpiThreads);
    mbar_init(c.drain, 1);
    mbar_init(c.xchg, 1);
    *c.abort = 0;
    fence_mbar_init();
    trace(1005);
    s_pre = gemm_prefetch_weights<BN, STAGES, SWAP>(g, c, &tm_a, &tm_b,
                                                   SWAP ? l2_policy_evict_first() : l2_policy_evict_last());
    trace(1006);
  }
  if (warp == 1) {
    tmem_alloc(c.tmem_base, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t hw = l2_policy_evict_first();
      const uint64_t hx = l2_policy_evict_last();
      gemm_producer<BN, STAGES, SWAP>(g, c, &tm_a, &tm_b, SWAP ? hw : hx, SWAP ? hx : hw, s_pre, [] {});
    }
  } else if (warp == 1) {
    if (lane == 0) gemm_mma<BN, STAGES>(g, c, umma_idesc_f16(kTileP, BN, std::is_same<IO, __nv_bfloat16>::value));
  } else {
    pdl_wait();  // outputs (and the exchange area) may still be read by the previous kernel
    epi.template prepare<SWAP>(g, c);
    const uint32_t tmem = *c.tmem_base;
    const int row = epi_row();
    int acc = 0;
    uint32_t acc_phase = 0;
    SegIter it(g);
    Seg tc;
    while (it.next(g, tc)) {
      if (!mbar_wait(&c.acc_full[acc], acc_phase, g.wait_ns, c.abort)) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
        break;
      }
      tc_fence_after();
      if (tc.nctb > 1) {
        // Split tile: reduce-scatter with the tile's other CTAs through L2.
        split_reduce_tile<BN>(g, tc, c, tmem, acc, epi.row_bias(g, tc.p, row),
                              [&](const float* v, int t0, int t_lo, int t_hi) {
                                epi.swap_chunk(g, c, v, tc.p, t0, t_lo, t_hi);
                              });
      } else if constexpr (SWAP) {
        // Lane = tile row (output feature), columns = tokens.
        const float b = epi.row_bias(g, tc.p, row);
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          epi_load_chunk<BN>(tmem, acc, col, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += b;
          epi.swap_chunk(g, c, v, tc.p, tc.q * BN + col, 0, g.T);
        }
      } else {
        epi.template nonswap_tile<BN>(g, tmem, acc, tc.p, tc.q);
      }
      tc_fence_before();
      mbar_arrive(&c.acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(*c.tmem_base, 2 * BN);
  }
  if (threadIdx.x == 0) trace(1001);
}

// Prefill shapes on CTA pairs (cta_group::2). A cluster of two CTAs computes
// one 256-token x 256-column output tile with tcgen05.mma.cta_group::2
// (M = 256, N = 256). CTA r of the pair holds tokens [128 r, 128 r + 128) of
// the tile (the MMA's A rows) and weight rows [128 r, 128 r + 128) of its 256
// (the B half; in gated mode the gate rows in the even CTA and the up rows of
// the same 128 features in the odd one). Each CTA loads 32 KB per k-block for
// the same MMA work per SM for which a single CTA's 128 x 256 tile loads
// 48 KB; at these shapes the main loop is bound by L2-to-SM bandwidth.
//
// The even CTA (rank 0) issues every MMA. Both CTAs' TMA loads count their
// bytes on its full barriers, which only it arms (expect_tx of both halves).
// Its commits arrive on the empty and accumulator-full barriers of both CTAs.
// Each CTA's epilogue reads its own TMEM (its 128 token rows x 256 columns)
// through the policy's nonswap_tile and then arrives on the even CTA's
// accumulator-empty barrier (two arrivals per phase). Tiles are dealt to the
// pairs round-robin, tokens fastest, so consecutive pairs share weight
// columns in L2. Every wait is bounded.
constexpr int kPairStages = 6;

template <typename IO, typename Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    col_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                         GemmShape g, const __grid_constant__ Epi epi) {
  using L = GemmSmem<kTileP, kPairStages, Epi::kSmemBytes>;
  extern __shared__ uint8_t smem_raw[];
  GemmCtl c = gemm_carve_smem<kTileP, kPairStages, Epi::kSmemBytes>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(cluster_id_x());
  const int npairs = static_cast<int>(cluster_count_x());
  const int MT = (g.T + 2 * kTileP - 1) / (2 * kTileP);
  const int PT = MT * g.q_tiles;

  if (threadIdx.x == 0) {
    trace(1000);
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    for (int i = 0; i < kPairStages; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    mbar_init(&c.acc_full[0], 1);
    mbar_init(&c.acc_full[1], 1);
    mbar_init(&c.acc_empty[0], 2);
    mbar_init(&c.acc_empty[1], 2);
    mbar_init(c.drain, 1);
    mbar_init(c.xchg, 1);
    *c.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(c.tmem_base, 4 * kTileP);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before any remote arrival or byte count
  tc_fence_after();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // Producer, both CTAs.
      const uint64_t hx = l2_policy_evict_last();
      const uint64_t hw = l2_policy_evict_first();
      const uint32_t full0 = dsmem_addr(&c.full[0], 0);
      pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; ok && u < PT; u += npairs) {
        const int mt = u % MT, nt = u / MT;
        const int xrow = mt * 2 * kTileP + static_cast<int>(rank) * kTileP;
        const int wrow = g.glu ? (rank == 0 ? nt * kTileP : g.N + nt * kTileP)
                               : nt * 2 * kTileP + static_cast<int>(rank) * kTileP;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&c.empty[stage], phase ^ 1u, g.wait_ns, c.abort)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&c.full[stage], 2u * L::kStageBytes);
          const uint32_t fb = full0 + 8u * static_cast<uint32_t>(stage);
          tma_load_2d_pair(&tm_x, fb, c.a + stage * L::kABytes, kb * kBlockK, xrow, hx);
          tma_load_2d_pair(&tm_w, fb, c.b + stage * L::kBBytes, kb * kBlockK, wrow, hw);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // MMA issuer: the even CTA only.
      const uint32_t idesc = umma_idesc_f16(2 * kTileP, 2 * kTileP, std::is_same<IO, __nv_bfloat16>::value);
      const uint32_t tmem = *c.tmem_base;
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true, any = false;
      for (int u = pair; ok && u < PT; u += npairs) {
        if (!mbar_wait_cluster(&c.acc_empty[acc], acc_phase ^ 1u, g.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * 2 * kTileP);
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&c.full[stage], phase, g.wait_ns, c.abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128_kmajor(smem_u32(c.a + stage * L::kABytes));
          const uint64_t db = umma_desc_sw128_kmajor(smem_u32(c.b + stage * L::kBBytes));
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k)
            umma_f16_ss_pair(d, da + static_cast<uint64_t>(2 * k), db + static_cast<uint64_t>(2 * k), idesc,
                             (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_pair_both(&c.empty[stage]);
          any = true;
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_both(&c.acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
        if (any) {
          // No MMA may still read shared memory or write TMEM when the pair
          // leaves: a commit tracks every earlier MMA of this thread.
          umma_commit_pair_local(c.drain);
          (void)mbar_wait(c.drain, 0u, 10000000ull, nullptr);
        }
      }
    }
  } else {
    // Epilogue, both CTAs: this CTA's 128 token rows of each tile.
    pdl_wait();
    epi.template prepare<false>(g, c);
    const uint32_t tmem = *c.tmem_base;
    const uint32_t empty0 = dsmem_addr(&c.acc_empty[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < PT; u += npairs) {
      if (!mbar_wait_cluster(&c.acc_full[acc], acc_phase, g.wait_ns)) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
        break;
      }
      tc_fence_after();
      const int mt = u % MT, nt = u / MT;
      epi.template nonswap_tile<2 * kTileP>(g, tmem, acc, 2 * mt + static_cast<int>(rank), nt);
      tc_fence_before();
      named_bar_sync(1, kEpiThreads);
      if (epi_tid() == 0) mbar_arrive_cluster(empty0 + 8u * static_cast<uint32_t>(acc));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no commit or arrival from the peer is still on its way
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(*c.tmem_base, 4 * kTileP);
  }
  if (threadIdx.x == 0) trace(1001);
}

// Decode batches of 129-256 tokens on CTA pairs (swap orientation). A pair
// tile is 256 weight rows x the batch's 256 token columns: CTA r holds weight
// rows [128 r, 128 r + 128) of it (its own 128-row tile p = 2 pt + r) and
// tokens [128 r, 128 r + 128) of the batch (the B half). Each CTA loads 32 KB
// per k-block where a single CTA of the same work loads 48 KB (the batch's
// 32 KB activation tile dominated). The decomposition (GemmShape) counts
// pairs: whole pair tiles round-robin, then split pair tiles over S pairs.
// Each CTA's accumulator is an ordinary 128-row swap tile, so the epilogue
// and the split-K reduce-scatter run per CTA as in col_gemm_kernel, with the
// split partners being the same-rank CTAs of the tile's S pairs (exchange
// halves 2 u + r). Split partners wait for each other: all pairs of a launch
// must be resident together, which the launcher checks against the occupancy
// of a cluster launch.
template <typename IO, typename Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    col_gemm_pair_swap_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                              GemmShape g, const __grid_constant__ Epi epi) {
  constexpr int BN = 2 * kTileP;  // tokens per pair tile
  using L = GemmSmem<kTileP, kPairStages, Epi::kSmemBytes>;
  extern __shared__ uint8_t smem_raw[];
  GemmCtl c = gemm_carve_smem<kTileP, kPairStages, Epi::kSmemBytes>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(cluster_id_x());

  if (threadIdx.x == 0) {
    trace(1000);
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
    for (int i = 0; i < kPairStages; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    mbar_init(&c.acc_full[0], 1);
    mbar_init(&c.acc_full[1], 1);
    mbar_init(&c.acc_empty[0], 2);
    mbar_init(&c.acc_empty[1], 2);
    mbar_init(c.drain, 1);
    mbar_init(c.xchg, 1);
    *c.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(c.tmem_base, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before any remote arrival or byte count
  tc_fence_after();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // Producer, both CTAs: this CTA's weight rows and token half, bytes
      // counted on the even CTA's full barriers.
      const uint64_t hw = l2_policy_evict_first();
      const uint64_t hx = l2_policy_evict_last();
      const uint32_t full0 = dsmem_addr(&c.full[0], 0);
      pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      SegIter it(g, pair);
      Seg tc;
      while (ok && it.next(g, tc)) {
        Seg mine = tc;
        mine.p = 2 * tc.p + static_cast<int>(rank);
        for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
          if (!mbar_wait(&c.empty[stage], phase ^ 1u, g.wait_ns, c.abort)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&c.full[stage], 2u * L::kStageBytes);
          const uint32_t fb = full0 + 8u * static_cast<uint32_t>(stage);
          uint8_t* a = c.a + stage * L::kABytes;
          if (!g.glu) {
            tma_load_2d_pair(&tm_w, fb, a, kb * kBlockK, mine.p * kTileP, hw);
          } else {
            const int r0 = mine.p * (kTileP / 2);
            tma_load_2d_pair(&tm_w, fb, a, kb * kBlockK, r0, hw);
            tma_load_2d_pair(&tm_w, fb, a + (kTileP / 2) * kBlockK * 2, kb * kBlockK, g.N + r0, hw);
          }
          tma_load_2d_pair(&tm_x, fb, c.b + stage * L::kBBytes, kb * kBlockK, static_cast<int>(rank) * kTileP, hx);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // MMA issuer: the even CTA only.
      const uint32_t idesc = umma_idesc_f16(2 * kTileP, BN, std::is_same<IO, __nv_bfloat16>::value);
      const uint32_t tmem = *c.tmem_base;
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true, any = false;
      SegIter it(g, pair);
      Seg tc;
      while (ok && it.next(g, tc)) {
        if (!mbar_wait_cluster(&c.acc_empty[acc], acc_phase ^ 1u, g.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
          if (!mbar_wait(&c.full[stage], phase, g.wait_ns, c.abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128_kmajor(smem_u32(c.a + stage * L::kABytes));
          const uint64_t db = umma_desc_sw128_kmajor(smem_u32(c.b + stage * L::kBBytes));
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k)
            umma_f16_ss_pair(d, da + static_cast<uint64_t>(2 * k), db + static_cast<uint64_t>(2 * k), idesc,
                             (kb > tc.kb0 || k > 0) ? 1u : 0u);
          umma_commit_pair_both(&c.empty[stage]);
          any = true;
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_both(&c.acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
        if (any) {
          umma_commit_pair_local(c.drain);
          (void)mbar_wait(c.drain, 0u, 10000000ull, nullptr);
        }
      }
    }
  } else {
    // Epilogue, both CTAs: this CTA's 128-row tile of each segment.
    pdl_wait();
    epi.template prepare<true>(g, c);
    const uint32_t tmem = *c.tmem_base;
    const uint32_t empty0 = dsmem_addr(&c.acc_empty[0], 0);
    const int row = epi_row();
    int acc = 0;
    uint32_t acc_phase = 0;
    SegIter it(g, pair);
    Seg tc;
    while (it.next(g, tc)) {
      if (!mbar_wait_cluster(&c.acc_full[acc], acc_phase, g.wait_ns)) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
        break;
      }
      tc_fence_after();
      Seg sv = tc;
      sv.p = 2 * tc.p + static_cast<int>(rank);
      if (tc.nctb > 1) {
        // Exchange half 2 u + r of split pair tile u.
        sv.tile = g.split_first + 2 * (tc.tile - g.split_first) + static_cast<int>(rank);
        split_reduce_tile<BN>(g, sv, c, tmem, acc, epi.row_bias(g, sv.p, row),
                              [&](const float* v, int t0, int t_lo, int t_hi) {
                                epi.swap_chunk(g, c, v, sv.p, t0, t_lo, t_hi);
                              });
      } else {
        const float b = epi.row_bias(g, sv.p, row);
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          epi_load_chunk<BN>(tmem, acc, col, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += b;
          epi.swap_chunk(g, c, v, sv.p, col, 0, g.T);
        }
      }
      tc_fence_before();
      named_bar_sync(1, kEpiThreads);
      if (epi_tid() == 0) mbar_arrive_cluster(empty0 + 8u * static_cast<uint32_t>(acc));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no commit or arrival from the peer is still on its way
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(*c.tmem_base, 2 * BN);
  }
  if (threadIdx.x == 0) trace(1001);
}

// Clusters of two that a pair kernel keeps resident at once on `dev`
// (cudaOccupancyMaxActiveClusters), queried once per kernel and device.
template <typename Kern>
int pair_clusters(Kern kern, const DeviceInfo& dev, int smem_bytes, int* out) {
  static int cached[64];
  static bool have[64];
  if (dev.device >= 0 && dev.device < 64 && have[dev.device]) {
    *out = cached[dev.device];
    return PGB_OK;
  }
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.gridDim = dim3(2 * (dev.sm_count / 2));
  cudaLaunchAttribute cl{};
  cl.id = cudaLaunchAttributeClusterDimension;
  cl.val.clusterDim.x = 2;
  cl.val.clusterDim.y = 1;
  cl.val.clusterDim.z = 1;
  cfg.attrs = &cl;
  cfg.numAttrs = 1;
  int n = 0;
  PGB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
  if (dev.device >= 0 && dev.device < 64) {
    cached[dev.device] = n;
    have[dev.device] = true;
  }
  *out = n;
  return PGB_OK;
}

// Launch the decode pair kernel for a swap plan with p.pair (counted in
// pairs). Same arguments as launch_col.
template <typename IO, typename Epi>
int launch_col_pair_swap(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w, int T, int N, int K,
                         const ColScratch& sc, cudaStream_t stream, const Epi& epi) {
  using L = GemmSmem<kTileP, kPairStages, Epi::kSmemBytes>;
  static_assert(L::kBytes <= 232448, "shared memory budget");
  auto kern = col_gemm_pair_swap_kernel<IO, Epi>;
  if (L::kBytes > dev.max_smem_optin)
    return set_error(PGB_ERR_UNSUPPORTED, "kernel needs %d B shared memory, device allows %d", L::kBytes,
                     dev.max_smem_optin);
  PGB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  if (p.nsplit > 1 && split_recv_bytes(2 * kTileP, p.nsplit) > static_cast<size_t>(kPairStages) * L::kStageBytes)
    return set_error(PGB_ERR_STATE, "col_gemm: split of %d does not fit the pipeline ring", p.nsplit);
  if (p.exchange_bytes > sc.xchg_bytes)
    return set_error(PGB_ERR_INVALID, "col_gemm: split exchange of %zu bytes, scratch holds %zu", p.exchange_bytes,
                     sc.xchg_bytes);
  if (p.counter_bytes > sc.ctr_bytes)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: %d split tiles exceed the counter region",
                     2 * (p.tiles - p.split_first));

  constexpr bool kBf16 = std::is_same<IO, __nv_bfloat16>::value;
  CUtensorMap tm_x, tm_w;
  int rc = make_tmap_2d_16bit(&tm_x, x, K, T, static_cast<uint64_t>(K) * 2, kBlockK, kTileP, kBf16);
  if (rc) return rc;
  constexpr int kWRows = kTileP / (Epi::kGlu ? 2 : 1);
  rc = make_tmap_2d_16bit(&tm_w, w, K, Epi::kGlu ? 2 * N : N, static_cast<uint64_t>(K) * 2, kBlockK, kWRows, kBf16);
  if (rc) return rc;

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
  g.status = sc.status;
  g.ctr = sc.ctr;
  g.xchg = sc.xchg;
  g.wait_ns = 2000000000ull;
  g.glu = Epi::kGlu ? 1 : 0;

  int clusters = 0;
  rc = pair_clusters(kern, dev, L::kBytes, &clusters);
  if (rc) return rc;
  // Split partners spin on each other: every pair of the launch must fit at once.
  if (clusters < p.grid)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: %d CTA pairs planned, %d fit the device", p.grid, clusters);
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cfg.gridDim = dim3(2 * p.grid);
  return launch_ex(cfg, /*cooperative=*/false, 2, kern, tm_w, tm_x, g, epi);
}

// Launch the pair kernel for a prefill plan (p.pair). Same arguments as
// launch_col.
template <typename IO, typename Epi>
int launch_col_pair(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w, int T, int N, int K,
                    const ColScratch& sc, cudaStream_t stream, const Epi& epi) {
  using L = GemmSmem<kTileP, kPairStages, Epi::kSmemBytes>;
  static_assert(L::kBytes <= 232448, "shared memory budget");
  auto kern = col_gemm_pair_kernel<IO, Epi>;
  if (L::kBytes > dev.max_smem_optin)
    return set_error(PGB_ERR_UNSUPPORTED, "kernel needs %d B shared memory, device allows %d", L::kBytes,
                     dev.max_smem_optin);
  PGB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  constexpr bool kBf16 = std::is_same<IO, __nv_bfloat16>::value;
  CUtensorMap tm_x, tm_w;
  int rc = make_tmap_2d_16bit(&tm_x, x, K, T, static_cast<uint64_t>(K) * 2, kBlockK, kTileP, kBf16);
  if (rc) return rc;
  rc = make_tmap_2d_16bit(&tm_w, w, K, Epi::kGlu ? 2 * N : N, static_cast<uint64_t>(K) * 2, kBlockK, kTileP, kBf16);
  if (rc) return rc;

  GemmShape g{};
  g.T = T;
  g.N = N;
  g.K = K;
  g.kblocks = p.kblocks;
  g.p_tiles = p.p_tiles;
  g.q_tiles = p.q_tiles;
  g.tiles = p.tiles;
  g.dp_rounds = p.dp_rounds;
  g.split_first = p.tiles;
  g.grid = p.grid;
  g.split_ctas = 0;
  g.nsplit = 1;
  g.status = sc.status;
  g.ctr = sc.ctr;
  g.xchg = sc.xchg;
  g.wait_ns = 2000000000ull;
  g.glu = Epi::kGlu ? 1 : 0;

  const int pair_tiles = ((T + 2 * kTileP - 1) / (2 * kTileP)) * p.q_tiles;
  int clusters = 0;
  rc = pair_clusters(kern, dev, L::kBytes, &clusters);
  if (rc) return rc;
  if (clusters < 1) return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: no CTA pair fits an SM pair");
  clusters = std::min(clusters, std::min(pair_tiles, dev.sm_count / 2));
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cfg.gridDim = dim3(2 * clusters);
  return launch_ex(cfg, /*cooperative=*/false, 2, kern, tm_x, tm_w, g, epi);
}

// Launch one column kernel. N is the output width g.N; the weight has N rows,
// or 2N ([gate; up]) for a gated policy. sc is the split-K scratch (a column
// workspace, col_scratch(), or a communicator's device-local area).
template <typename IO, int BN, bool SWAP, typename Epi>
int launch_col(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w, int T, int N, int K,
               const ColScratch& sc, cudaStream_t stream, const Epi& epi) {
  constexpr int STAGES = gemm_stages<BN>();
  using L = GemmSmem<BN, STAGES, Epi::kSmemBytes>;
  static_assert(L::kBytes <= 232448, "shared memory budget");
  static_assert(gemm_ctas_per_sm(BN) == 1 || 2 * (L::kBytes + 1024) <= 233472, "two CTAs per SM");
  auto kern = col_gemm_kernel<IO, BN, SWAP, STAGES, Epi>;
  if (L::kBytes > dev.max_smem_optin)
    return set_error(PGB_ERR_UNSUPPORTED, "kernel needs %d B shared memory, device allows %d", L::kBytes,
                     dev.max_smem_optin);
  PGB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  if (p.nsplit > 1 && split_recv_bytes(BN, p.nsplit) > static_cast<size_t>(STAGES) * L::kStageBytes)
    return set_error(PGB_ERR_STATE, "col_gemm: split of %d does not fit the pipeline ring", p.nsplit);
  if (p.exchange_bytes > sc.xchg_bytes)
    return set_error(PGB_ERR_INVALID, "col_gemm: split exchange of %zu bytes, scratch holds %zu", p.exchange_bytes,
                     sc.xchg_bytes);
  if (p.counter_bytes > sc.ctr_bytes)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: %d split tiles exceed the counter region",
                     p.tiles - p.split_first);

  constexpr bool kBf16 = std::is_same<IO, __nv_bfloat16>::value;
  CUtensorMap tm_x, tm_w;
  int rc = make_tmap_2d_16bit(&tm_x, x, K, T, static_cast<uint64_t>(K) * 2, kBlockK, SWAP ? BN : kTileP, kBf16);
  if (rc) return rc;
  constexpr int kWRows = (SWAP ? kTileP : BN) / (Epi::kGlu ? 2 : 1);  // weight box height
  rc = make_tmap_2d_16bit(&tm_w, w, K, Epi::kGlu ? 2 * N : N, static_cast<uint64_t>(K) * 2, kBlockK, kWRows,
                          kBf16);
  if (rc) return rc;

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
  g.status = sc.status;
  g.ctr = sc.ctr;
  g.xchg = sc.xchg;
  g.wait_ns = 2000000000ull;  // 2 s: far beyond any legitimate pipeline stall
  g.glu = Epi::kGlu ? 1 : 0;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  const CUtensorMap& ta = SWAP ? tm_w : tm_x;
  const CUtensorMap& tb = SWAP ? tm_x : tm_w;
  // The CTAs of a split tile wait for each other: cooperative launch.
  return launch_ex(cfg, /*cooperative=*/p.split_ctas > 0, 1, kern, ta, tb, g, epi);
}

// The tile width the plan picked, for one policy.
template <typename IO, typename Epi>
int dispatch_col(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w, int T, int N, int K,
                 const ColScratch& sc, cudaStream_t stream, const Epi& epi) {
  if (p.pair) {
    const int rc = p.swap ? launch_col_pair_swap<IO>(p, dev, x, w, T, N, K, sc, stream, epi)
                          : launch_col_pair<IO>(p, dev, x, w, T, N, K, sc, stream, epi);
    if (rc != PGB_ERR_UNSUPPORTED) return rc;
    // The device cannot keep the pairs resident: the single-CTA plan.
    GemmPlan q = plan_gemm(T, Epi::kGlu ? 2 * N : N, K, dev.sm_count, sc.xchg_bytes);
    q.pair = false;
    return dispatch_col<IO>(q, dev, x, w, T, N, K, sc, stream, epi);
  }
  if (!p.swap) return launch_col<IO, 256, false>(p, dev, x, w, T, N, K, sc, stream, epi);
  switch (p.bn) {
    case 32: return launch_col<IO, 32, true>(p, dev, x, w, T, N, K, sc, stream, epi);
    case 64: return launch_col<IO, 64, true>(p, dev, x, w, T, N, K, sc, stream, epi);
    case 128: return launch_col<IO, 128, true>(p, dev, x, w, T, N, K, sc, stream, epi);
    case 256: return launch_col<IO, 256, true>(p, dev, x, w, T, N, K, sc, stream, epi);
    default: return set_error(PGB_ERR_INVALID, "no kernel for tile width %d", p.bn);
  }
}

}  // namespace pgb
