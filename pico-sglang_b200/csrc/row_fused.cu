// row_fused.cu - row-parallel GEMM + all-reduce + residual-add + RMSNorm in
// one cooperative kernel.
//
// Replaces, per call, the reference sequence
//   LinearRowParallel.forward   y = F.linear(x_local, W_local)         (layers/linear.py:90-97)
//   -> all_reduce(y, "sum")     memcpy + ncclAllReduce + memcpy        (csrc/src/pynccl.cu:95-137)
//   -> RMSNormFused.forward     flashinfer fused_add_rmsnorm           (layers/norm.py:73-75)
//
// Phase 1 (tcgen05 GEMM, persistent): each finished output tile (split
//   tiles reduce-scattered between their CTAs on this GPU) is rounded to the
//   I/O type and stored into the slot region of the rank(s) that reduce its rows:
//   every rank for one-shot, the row owner for two-shot. Remote stores go
//   over NVLink while later tiles are still being multiplied.
// Barrier 0: grid arrival, then a release flag to every rank, then bounded
//   waits for all ranks' flags of this epoch.
// Phase 2: per owned row, sum the ranks' partials in rank order (f32),
//   round to the I/O type (the reference materialises the reduced tensor),
//   add the residual, store the residual, RMS-normalise and store out.
//   Two-shot owners also push both rows to every peer's result region.
// Barrier 1 + phase 3 (two-shot only): copy the other owners' rows in.
//
// On a one-rank communicator the entry point runs the column GEMM and then
// fused_add_rmsnorm instead (faster there, as measured), unless
// pgb_comm_set_one_rank_path asked for this kernel.
#include "comm.h"
#include "gemm_f32.h"
#include "gemm_plan.h"
#include "gemm_sm100.cuh"
#include "host_common.h"
#include "reduce_phases.cuh"

namespace pgb {

constexpr int kRowMaxVec = 8;  // 8 vectors of 8 per thread: width <= 192 * 64 = 12288

struct RowArgs {
  GemmShape g;
  CommDev cm;
  RowSplit rs;
  void* out;
  void* residual;
  const void* norm_w;
  const void* bias;
  float eps;
  int do_norm;
};

template <typename IO>
__device__ __forceinline__ void row_store_partial(const RowArgs& a, uint32_t parity, int t, int n,
                                                  IO val) {
  const int H = a.g.N;
  const size_t src_off = static_cast<size_t>(a.cm.rank) * a.rs.rows_cap * H;
  if (a.rs.oneshot) {
    for (int d = 0; d < a.cm.world; ++d) {
      IO* base = reinterpret_cast<IO*>(a.cm.slots[d] + parity * a.cm.slot_parity_bytes);
      base[src_off + static_cast<size_t>(t) * H + n] = val;
    }
  } else {
    const int o = t / a.rs.rows_per;
    IO* base = reinterpret_cast<IO*>(a.cm.slots[o] + parity * a.cm.slot_parity_bytes);
    base[src_off + static_cast<size_t>(t - o * a.rs.rows_per) * H + n] = val;
  }
}

// 4 consecutive features [n0, n0 + 4) of token t into the reducing rank(s).
template <typename IO>
__device__ __forceinline__ void row_store4(const RowArgs& a, uint32_t parity, int t, int n0, uint2 piece) {
  const int H = a.g.N;
  const size_t src_off = static_cast<size_t>(a.cm.rank) * a.rs.rows_cap * H;
  int d0 = 0, d1 = a.cm.world;
  size_t row = static_cast<size_t>(t);
  if (!a.rs.oneshot) {
    d0 = t / a.rs.rows_per;
    d1 = d0 + 1;
    row = static_cast<size_t>(t - d0 * a.rs.rows_per);
  }
  for (int d = d0; d < d1; ++d) {
    IO* base = reinterpret_cast<IO*>(a.cm.slots[d] + parity * a.cm.slot_parity_bytes);
    *reinterpret_cast<uint2*>(base + src_off + row * H + n0) = piece;
  }
}

// 8 consecutive features [n0, n0 + 8) of token t into the reducing rank(s).
template <typename IO>
__device__ __forceinline__ void row_store_piece(const RowArgs& a, uint32_t parity, int t, int n0,
                                                uint4 piece) {
  const int H = a.g.N;
  const size_t src_off = static_cast<size_t>(a.cm.rank) * a.rs.rows_cap * H;
  int d0 = 0, d1 = a.cm.world;
  size_t row = static_cast<size_t>(t);
  if (!a.rs.oneshot) {
    d0 = t / a.rs.rows_per;
    d1 = d0 + 1;
    row = static_cast<size_t>(t - d0 * a.rs.rows_per);
  }
  for (int d = d0; d < d1; ++d) {
    IO* base = reinterpret_cast<IO*>(a.cm.slots[d] + parity * a.cm.slot_parity_bytes);
    *reinterpret_cast<uint4*>(base + src_off + row * H + n0) = piece;
  }
}

template <typename IO>
__device__ __forceinline__ void row_store_partial_vec32(const RowArgs& a, uint32_t parity, int t,
                                                        int n0, const float* v) {
  const int H = a.g.N;
  const size_t src_off = static_cast<size_t>(a.cm.rank) * a.rs.rows_cap * H;
  uint4 pk[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) pk[j] = pack8<IO>(v + 8 * j);
  int d0 = 0, d1 = a.cm.world;
  size_t row = static_cast<size_t>(t);
  if (!a.rs.oneshot) {
    d0 = t / a.rs.rows_per;
    d1 = d0 + 1;
    row = static_cast<size_t>(t - d0 * a.rs.rows_per);
  }
  for (int d = d0; d < d1; ++d) {
    IO* base = reinterpret_cast<IO*>(a.cm.slots[d] + parity * a.cm.slot_parity_bytes);
    uint4* dst = reinterpret_cast<uint4*>(base + src_off + row * H + n0);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = pk[j];
  }
}

template <typename IO, int BN, bool SWAP, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, gemm_ctas_per_sm(BN))
    row_fused_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     RowArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_pre;  // stages armed with weight tiles before pdl_wait()
  __shared__ uint32_t s_epoch;
  __shared__ uint64_t s_epoch_bar;  // the producer publishes s_epoch after pdl_wait()
  __shared__ float s_red[32];
  GemmCtl c = gemm_carve_smem<BN, STAGES>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const GemmShape& g = a.g;

  if (threadIdx.x == 0) {
    trace(1000);
    tma_prefetch_desc(&tm_a);  // descriptor fetch overlaps barrier set-up
    tma_prefetch_desc(&tm_b);
    mbar_init(&s_epoch_bar, 1);
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
      // The epoch counter is written by the previous call on this stream:
      // read it only once that call has finished.
      gemm_producer<BN, STAGES, SWAP>(g, c, &tm_a, &tm_b, SWAP ? hw : hx, SWAP ? hx : hw, s_pre, [&] {
        s_epoch = comm_begin(a.cm);
        mbar_arrive(&s_epoch_bar);
      });
    }
  } else if (warp == 1) {
    if (lane == 0) gemm_mma<BN, STAGES>(g, c, umma_idesc_f16(kTileP, BN, std::is_same<IO, __nv_bfloat16>::value));
  } else {
    pdl_wait();
    if (!mbar_wait(&s_epoch_bar, 0u, g.wait_ns, nullptr)) record_error(g.status, kDevTimeoutPipeline);
    const uint32_t parity = s_epoch & 1u;
    const uint32_t tmem = *c.tmem_base;
    const int row = epi_row();
    const IO* bias = static_cast<const IO*>(a.bias);
    (void)row;
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
        // Split tile: reduce-scatter with the tile's other CTAs through L2,
        // then store into the slots of the reducing rank(s).
        const int nb = tc.p * kTileP + row;
        const float b = (bias != nullptr && nb < g.N) ? io_to_f32<IO>(bias[nb]) : 0.f;
        split_reduce_tile<BN>(g, tc, c, tmem, acc, b, [&](const float* v, int t0, int t_lo, int t_hi) {
          swap_epilogue_store<IO>(c.epi, v, t0, t_lo, t_hi, tc.p * kTileP, g.N, [&](int t, int n0, uint4 piece) {
            row_store_piece<IO>(a, parity, t, n0, piece);
          });
        });
      } else {
        // Whole tiles: round and store straight into the slots of the
        // rank(s) that reduce these rows.
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          epi_load_chunk<BN>(tmem, acc, col, v);
          if constexpr (SWAP) {
            const int n = tc.p * kTileP + row;
            if (bias != nullptr && n < g.N) {
              const float b = io_to_f32<IO>(bias[n]);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += b;
            }
            swap_epilogue_store<IO>(c.epi, v, tc.q * BN + col, 0, g.T, tc.p * kTileP, g.N,
                                    [&](int t, int n0, uint4 piece) {
                                      row_store_piece<IO>(a, parity, t, n0, piece);
                                    });
          } else {
            const int t = tc.p * kTileP + row;
            const int n0 = tc.q * BN + col;
            if (t < g.T) {
              if (bias != nullptr) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (n0 + j < g.N) v[j] += io_to_f32<IO>(bias[n0 + j]);
              }
              if (n0 + 32 <= g.N) {
                row_store_partial_vec32<IO>(a, parity, t, n0, v);
              } else {
                for (int j = 0; j < 32 && n0 + j < g.N; ++j)
                  row_store_partial<IO>(a, parity, t, n0 + j, f32_to_io<IO>(v[j]));
              }
            }
          }
        }
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

  pdl_wait();
  const uint32_t e = s_epoch;  // published before the barrier above
  const uint32_t parity = e & 1u;
  const bool multi = a.cm.world > 1;
  IO* out = static_cast<IO*>(a.out);
  IO* residual = static_cast<IO*>(a.residual);
  const IO* norm_w = static_cast<const IO*>(a.norm_w);
  // A failure anywhere on this GPU poisons the status; the barriers then
  // stop waiting and the later phases are skipped.
  if (threadIdx.x == 0) trace(1004);
  const bool ok0 = grid_cross_barrier(a.cm, kBarPartials, e, multi);
  if (threadIdx.x == 0) trace(1002);
  if (ok0) {
    const int r0 = a.rs.first(a.cm.rank), r1 = a.rs.last(a.cm.rank);
    // The pipeline ring is idle from here on: it stages the pre-norm rows.
    constexpr size_t kRing = static_cast<size_t>(STAGES) * GemmSmem<BN, STAGES>::kStageBytes;
    // Narrow (decode) tiles never carry more rows than CTAs: only wide tiles
    // build the warp-per-row path.
    bool warp_rows = false;
    if constexpr (BN >= 128) {
      if (r1 - r0 > static_cast<int>(gridDim.x) &&
          static_cast<size_t>(g.N) * (4u * (kGemmThreads / 32) + 2u) <= kRing) {
        reduce_rows_warp<IO>(a.cm, a.rs, parity, r0, r1, g.N, out, residual, norm_w, a.eps, a.do_norm, c.a);
        if (threadIdx.x == 0) trace(1017);
        warp_rows = true;
      }
    }
    if (!warp_rows) {
      float* srow = reinterpret_cast<float*>(c.a);
      int nrow = 0;
      for (int t = r0 + static_cast<int>(blockIdx.x); t < r1; t += gridDim.x, ++nrow) {
        reduce_row<IO, kRowMaxVec>(a.cm, a.rs, parity, t, g.N, out, residual, norm_w, a.eps, a.do_norm, s_red,
                                   srow);
        if (threadIdx.x == 0 && nrow < 3) trace(1017 + nrow);
      }
    }
  }
  if (multi && !a.rs.oneshot) {
    if (threadIdx.x == 0) trace(1008);
    const bool ok2 = grid_cross_barrier(a.cm, kBarResults, e, true);
    if (threadIdx.x == 0) trace(1009);
    if (ok0 && ok2) gather_rows<IO>(a.cm, a.rs, parity, g.N, out, residual, a.do_norm);
  }
  if (threadIdx.x == 0) trace(1003);
  comm_end(a.cm, e);
  if (threadIdx.x == 0) trace(1001);
}

namespace {

template <typename IO, int BN, bool SWAP>
int launch_row(pgb_comm* c, RowArgs args, const void* x, const void* w, cudaStream_t stream) {
  constexpr int STAGES = gemm_stages<BN>();
  using L = GemmSmem<BN, STAGES>;
  static_assert(L::kBytes + 256 <= 232448, "shared memory budget");
  static_assert(static_cast<size_t>(STAGES) * L::kStageBytes >= kGemmThreads * 8 * kRowMaxVec * (4 + 2),
                "the ring holds one f32 row and its norm weights in the row phase");
  auto kern = row_fused_kernel<IO, BN, SWAP, STAGES>;
  PGB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  if (args.g.nsplit > 1 && split_recv_bytes(BN, args.g.nsplit) > static_cast<size_t>(STAGES) * L::kStageBytes)
    return set_error(PGB_ERR_STATE, "row kernel: split of %d does not fit the pipeline ring", args.g.nsplit);
  constexpr bool kBf16 = std::is_same<IO, __nv_bfloat16>::value;
  const int T = args.g.T, N = args.g.N, K = args.g.K;
  CUtensorMap tm_x, tm_w;
  int rc = make_tmap_2d_16bit(&tm_x, x, K, T, static_cast<uint64_t>(K) * 2, kBlockK,
                              SWAP ? BN : kTileP, kBf16);
  if (rc) return rc;
  rc = make_tmap_2d_16bit(&tm_w, w, K, N, static_cast<uint64_t>(K) * 2, kBlockK,
                          SWAP ? kTileP : BN, kBf16);
  if (rc) return rc;

  cudaLaunchConfig_t cfg{};
  // Every SM takes part in the row phase.
  cfg.gridDim = dim3(c->sm_count);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  const CUtensorMap& ta = SWAP ? tm_w : tm_x;
  const CUtensorMap& tb = SWAP ? tm_x : tm_w;
  return launch_ex(cfg, /*cooperative=*/true, 1, kern, ta, tb, args);
}

template <typename IO>
int dispatch_row(pgb_comm* c, const GemmPlan& p, const RowArgs& args, const void* x, const void* w,
                 cudaStream_t s) {
  if (!p.swap) return launch_row<IO, 256, false>(c, args, x, w, s);
  switch (p.bn) {
    case 32: return launch_row<IO, 32, true>(c, args, x, w, s);
    case 64: return launch_row<IO, 64, true>(c, args, x, w, s);
    case 128: return launch_row<IO, 128, true>(c, args, x, w, s);
    case 256: return launch_row<IO, 256, true>(c, args, x, w, s);
    default: return set_error(PGB_ERR_INVALID, "no kernel for tile width %d", p.bn);
  }
}

}  // namespace

// f32 check mode of the fused row op: the partial product in IEEE f32 into
// `out`, the communicator's all-reduce over it, then the f32 fused
// residual-add + RMSNorm - the reference's sequence (linear.py:90-97,
// pynccl.cu:95-137, norm.py:73-75) at f32, as separate launches (not a hot
// path). The bias, if any, is added on every rank before the reduction, as
// in the fused bf16 kernel.
int row_f32(pgb_comm* comm, const void* x_local, const void* w_local, const void* bias, void* residual,
            const void* norm_w, float eps, void* out, int T, int N, int K_local, void* stream) {
  if (x_local == nullptr || w_local == nullptr || out == nullptr)
    return set_error(PGB_ERR_INVALID, "row_gemm: null pointer argument");
  if (norm_w != nullptr && residual == nullptr)
    return set_error(PGB_ERR_INVALID, "row_gemm: norm weight given without residual");
  int rc = launch_gemm_f32(static_cast<const float*>(x_local), static_cast<const float*>(w_local),
                           static_cast<const float*>(bias), static_cast<float*>(out), T, N, K_local,
                           static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  if (comm->world > 1) {
    rc = pgb_all_reduce(comm, out, static_cast<size_t>(T) * N, PGB_F32, PGB_OP_SUM, stream);
    if (rc) return rc;
  }
  if (norm_w != nullptr) rc = pgb_fused_add_rmsnorm(out, residual, norm_w, eps, T, N, PGB_F32, stream);
  return rc;
}

int row_xchg(pgb_comm* comm, const void* x_local, const void* w_local, const void* bias, void* residual,
             const void* norm_w, float eps, void* out, int T, int N, int K_local, int dtype, void* stream);

// Choose one-shot or two-shot for a reduction of `rows` x `width` elements of
// `elem` bytes; returns false if neither fits the communicator buffers.
bool plan_rows(const pgb_comm* c, int rows, int width, int elem, RowSplit* rs) {
  const double row_bytes = static_cast<double>(width) * elem;
  const double S = row_bytes * rows;
  const int n = c->world;
  const bool one_fits = static_cast<double>(n) * S <= static_cast<double>(c->slot_parity_bytes);
  const int rows_per = (rows + n - 1) / n;
  const bool two_fits = static_cast<double>(n) * rows_per * row_bytes <= c->slot_parity_bytes &&
                        2.0 * S <= static_cast<double>(c->result_parity_bytes);
  bool one = (n == 1) || !two_fits;
  if (n > 1 && one_fits && two_fits) {
    // NVLink ~770 GB/s per direction, HBM ~6.5 TB/s, one extra barrier ~2 us.
    const double t_one = (n - 1) * S / 770e9 + n * S / 6.5e12;
    const double t_two = 2.0 * (n - 1) / n * S / 770e9 + S / 6.5e12 + 2e-6;
    one = t_one <= t_two;
  }
  if (one && !one_fits) return false;
  rs->rows = rows;
  rs->oneshot = one ? 1 : 0;
  rs->rows_per = one ? rows : rows_per;
  rs->rows_cap = one ? rows : rows_per;
  return true;
}

// The row op as three launches: the column GEMM into out (on the
// communicator's split scratch), the communicator's all-reduce over it, then
// fused_add_rmsnorm in place. Used when the payload does not fit the
// communicator's buffers (the reference then all-reduces in place,
// csrc/src/pynccl.cu:127-135) and, by default, for prefill batches, where the
// column GEMM runs on CTA pairs and beats the fused kernel's single-CTA tiles
// by more than the exchange overlap gains.
int row_unfused(pgb_comm* comm, const void* x_local, const void* w_local, const void* bias, void* residual,
                const void* norm_w, float eps, void* out, int T, int N, int K_local, int dtype, void* stream) {
  ColScratch sc;
  sc.status = reinterpret_cast<int*>(comm->local + LocalLayout::kStatus);
  sc.ctr = reinterpret_cast<uint32_t*>(comm->local + LocalLayout::kCounters);
  sc.ctr_bytes = kTileCounterBytes;
  sc.xchg = reinterpret_cast<float*>(comm->local + LocalLayout::kPartials);
  sc.xchg_bytes = kSplitScratchBytes;
  int rc = col_gemm_on_scratch(x_local, w_local, bias, out, T, N, K_local, dtype, sc, stream);
  if (rc) return rc;
  if (comm->world > 1) {
    rc = pgb_all_reduce(comm, out, static_cast<size_t>(T) * N, dtype, PGB_OP_SUM, stream);
    if (rc) return rc;
  }
  if (norm_w == nullptr) return PGB_OK;
  return pgb_fused_add_rmsnorm(out, residual, norm_w, eps, T, N, dtype, stream);
}

// Largest batch the default exchange mode runs on the fused kernel.
constexpr int kFusedRowMaxTokens = 256;

}  // namespace pgb

extern "C" int pgb_row_gemm_allreduce_addnorm(pgb_comm* comm, const void* x_local,
                                              const void* w_local, const void* bias,
                                              void* residual, const void* norm_w, float eps,
                                              void* out, int T, int N, int K_local, int dtype,
                                              void* stream) {
  using namespace pgb;
  if (comm == nullptr) return set_error(PGB_ERR_INVALID, "row_gemm: null communicator");
  if (comm->world > 1 && !comm->peers_open)
    return set_error(PGB_ERR_STATE, "row_gemm: peers not opened (call pgb_comm_open_peers)");
  if (T < 0 || N <= 0 || K_local <= 0)
    return set_error(PGB_ERR_INVALID, "row_gemm: bad shape T=%d N=%d K=%d", T, N, K_local);
  if (T == 0) return PGB_OK;
  if (dtype == PGB_F32) return row_f32(comm, x_local, w_local, bias, residual, norm_w, eps, out, T, N, K_local, stream);
  if (dtype != PGB_BF16 && dtype != PGB_F16)
    return set_error(PGB_ERR_INVALID, "row_gemm: unknown dtype %d", dtype);
  if (K_local % 8 != 0 || N % 8 != 0)
    return set_error(PGB_ERR_INVALID, "row_gemm: K=%d and N=%d must be multiples of 8", K_local, N);
  if (N > kGemmThreads * 8 * kRowMaxVec)
    return set_error(PGB_ERR_UNSUPPORTED, "row_gemm: hidden size %d above %d", N,
                     kGemmThreads * 8 * kRowMaxVec);
  if (x_local == nullptr || w_local == nullptr || out == nullptr)
    return set_error(PGB_ERR_INVALID, "row_gemm: null pointer argument");
  if (norm_w != nullptr && residual == nullptr)
    return set_error(PGB_ERR_INVALID, "row_gemm: norm weight given without residual");
  const uintptr_t mis = reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual) |
                        reinterpret_cast<uintptr_t>(norm_w);
  if ((mis & 15u) != 0u)
    return set_error(PGB_ERR_INVALID, "row_gemm: out / residual / norm weight not 16-byte aligned");
  int cur = -1;
  PGB_CUDA_TRY(cudaGetDevice(&cur));
  if (cur != comm->device)
    return set_error(PGB_ERR_INVALID, "row_gemm: current device %d, communicator on %d", cur,
                     comm->device);

  if (comm->world == 1 && !comm->one_rank_fused) {
    // One rank: the all-reduce is the identity (the reference's LinearRowParallel
    // all-reduces only when tp > 1, python/picosgl/layers/linear.py:90-97), so
    // there is nothing to overlap. The column GEMM on the communicator's own
    // split scratch, then fused_add_rmsnorm in place on `out`, beats the fused
    // kernel's grid barrier and row phase here (measured on B200 at T = 1..256:
    // 15.6 vs 18.9 us for o_proj at T = 1, 23.0 vs 29.5 at T = 256).
    return row_unfused(comm, x_local, w_local, bias, residual, norm_w, eps, out, T, N, K_local, dtype, stream);
  }
  if (comm->exchange_mode == PGB_XCHG_AUTO && T > kFusedRowMaxTokens)
    return row_unfused(comm, x_local, w_local, bias, residual, norm_w, eps, out, T, N, K_local, dtype, stream);

  if (comm->exchange_mode == PGB_XCHG_ONESHOT || comm->exchange_mode == PGB_XCHG_TWOSHOT ||
      (comm->exchange_mode == PGB_XCHG_NVLS && comm->nvls)) {
    // Decode shapes on request: the per-piece exchange kernel (row_xchg.cu).
    // Not the default: measured on two B200s it is slower than the barrier
    // kernel below (o_proj T = 256: 42.9 vs 29.7 us; T = 1: 23.4 vs 18.0 us),
    // because every CTA's system-scope fence before its flags costs 2-3 us,
    // where the barrier kernel fences once per rank.
    const int rc = row_xchg(comm, x_local, w_local, bias, residual, norm_w, eps, out, T, N, K_local, dtype, stream);
    if (rc != PGB_ERR_UNSUPPORTED) return rc;
  }
  RowSplit rs;
  if (!plan_rows(comm, T, N, 2, &rs)) {
    // The payload does not fit the communicator's buffers: the chunked
    // all-reduce of the unfused sequence.
    return row_unfused(comm, x_local, w_local, bias, residual, norm_w, eps, out, T, N, K_local, dtype, stream);
  }
  const GemmPlan p = plan_gemm(T, N, K_local, comm->sm_count, kSplitScratchBytes);
  if (p.counter_bytes > kTileCounterBytes)
    return set_error(PGB_ERR_UNSUPPORTED, "row_gemm: too many split tiles (%d)", p.tiles - p.split_first);

  RowArgs args{};
  args.g.T = T;
  args.g.N = N;
  args.g.K = K_local;
  args.g.kblocks = p.kblocks;
  args.g.p_tiles = p.p_tiles;
  args.g.q_tiles = p.q_tiles;
  args.g.tiles = p.tiles;
  args.g.dp_rounds = p.dp_rounds;
  args.g.split_first = p.split_first;
  args.g.grid = p.grid;
  args.g.split_ctas = p.split_ctas;
  args.g.nsplit = p.nsplit;
  args.g.status = reinterpret_cast<int*>(comm->local + LocalLayout::kStatus);
  args.g.ctr = reinterpret_cast<uint32_t*>(comm->local + LocalLayout::kCounters);
  args.g.xchg = reinterpret_cast<float*>(comm->local + LocalLayout::kPartials);
  args.g.wait_ns = 2000000000ull;
  args.cm = comm_dev(comm);
  args.rs = rs;
  args.out = out;
  args.residual = residual;
  args.norm_w = norm_w;
  args.bias = bias;
  args.eps = eps;
  args.do_norm = norm_w != nullptr ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PGB_BF16) return dispatch_row<__nv_bfloat16>(comm, p, args, x_local, w_local, s);
  return dispatch_row<__half>(comm, p, args, x_local, w_local, s);
}

#ifdef PGB_TRACE
extern "C" PGB_API int pgb_debug_set_trace_row(void* buf) {
  cudaError_t e = cudaMemcpyToSymbol(pgb::pgb_trace_buf, &buf, sizeof(buf));
  return e == cudaSuccess ? 0 : 2;
}
#endif
