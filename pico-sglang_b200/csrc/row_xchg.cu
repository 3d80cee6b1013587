// row_xchg.cu - row-parallel GEMM + all-reduce + residual-add + RMSNorm on
// several GPUs for decode shapes, with a feature-slice exchange.
//
// Replaces, per call, the reference sequence
//   LinearRowParallel.forward   y = F.linear(x_local, W_local)         (layers/linear.py:90-97)
//   -> all_reduce(y, "sum")     memcpy + ncclAllReduce + memcpy        (csrc/src/pynccl.cu:95-137)
//   -> RMSNormFused.forward     flashinfer fused_add_rmsnorm           (layers/norm.py:73-75)
// for T <= 256 tokens (the swap orientation of the GEMM core: 128 output
// features x BN tokens per tile).
//
// Every rank runs the same work decomposition, so CTA c computes "piece" k
// (its k-th segment: a whole tile, or its token run of a split tile) of the
// same output region on every rank.
//
// Two-shot (reduce-scatter by feature slices + all-gather of the reduced sum):
//   1. GEMM. Each 16-byte piece of 8 output features of a finished piece
//      (split tiles reduce-scattered on this GPU first, rounded to the I/O
//      type as F.linear rounds) goes to the rank owning that feature slice:
//      rank s owns features [s*F, (s+1)*F) of every 128-feature tile,
//      F = 128 / world. Barrier 0 (every CTA arrives, one system-scope fence
//      and a flag per rank, then every CTA waits for all ranks).
//   2. CTA c on rank s sums its slice of each of its pieces over the ranks in
//      rank order (f32), rounds it (the reference materialises the reduced
//      tensor), and stores it into every rank's y buffer [T][H]. Barrier 1.
//   3. Every rank computes residual += y and out = rmsnorm(residual) for its
//      rows from its own y buffer and its own residual copy: every rank ends
//      bit-identical. The all-gather carries y only, half the bytes of
//      gathering out and residual.
// One-shot (small payloads): step 1 sends the whole piece to every rank,
// step 2 is skipped, and step 3 sums the ranks' pieces itself.
//
// Each reduction step is spread over every CTA that computed a piece (the
// slices follow the GEMM's own decomposition), where the token-row owners of
// row_fused.cu leave most CTAs idle at small T.
//
// Bytes over NVLink per rank: two-shot 2 (n-1)/n T H 2 (the P2P bound),
// one-shot (n-1) T H 2.
#include "comm.h"
#include "gemm_plan.h"
#include "gemm_sm100.cuh"
#include "host_common.h"
#include "reduce_phases.cuh"

namespace pgb {

namespace {

constexpr int kXchgRowMaxVec = 8;  // width <= 192 threads x 8 vectors x 8 elements

struct XchgArgs {
  GemmShape g;
  CommDev cm;
  int nvls;      // NVLink multicast: partials local, reduced in the switch
  uint8_t* nv_uc;  // this device's view of the multicast-bound region
  uint8_t* nv_mc;  // the multicast view (every device of the team)
  uint64_t nv_parity_bytes;  // per parity: [partials | reduced], half each
  int oneshot;
  int fslice;  // two-shot: features of a 128-feature tile owned by each rank (128 / world)
  void* out;
  void* residual;
  const void* norm_w;
  const void* bias;
  float eps;
  int do_norm;
};

// Token range [t0, t1) of piece s (a tile of BN tokens, or one CTA's run of a
// split tile, as split_reduce_tile cuts it).
__device__ __forceinline__ void piece_tokens(const GemmShape& g, const Seg& s, int bn, int& t0, int& t1) {
  const int base = s.q * bn;
  const int V = min(bn, g.T - base);
  if (s.nctb > 1) {
    int c0, c1;
    split_cols(bn, V, s.nctb, s.contrib, c0, c1);
    t0 = base + c0;
    t1 = base + c1;
  } else {
    t0 = base;
    t1 = base + V;
  }
}

// Step 1 store: 8 consecutive features [n0, n0 + 8) of token t of this
// rank's partial.
template <typename IO>
__device__ __forceinline__ void xchg_emit(const XchgArgs& a, uint32_t parity, int t, int n0, uint4 piece) {
  const CommDev& cm = a.cm;
  const int H = a.g.N, T = a.g.T;
  if (a.nvls) {
    // this device's partials [T][H], reduced later through the multicast view
    IO* base = reinterpret_cast<IO*>(a.nv_uc + parity * a.nv_parity_bytes);
    *reinterpret_cast<uint4*>(base + static_cast<size_t>(t) * H + n0) = piece;
    return;
  }
  if (a.oneshot) {
    // slots of every rank: [src rank][T][H]
    const size_t off = (static_cast<size_t>(cm.rank) * T + t) * H + n0;
    for (int d = 0; d < cm.world; ++d) {
      IO* base = reinterpret_cast<IO*>(cm.slots[d] + parity * cm.slot_parity_bytes);
      *reinterpret_cast<uint4*>(base + off) = piece;
    }
  } else {
    // slots of the slice owner s: [src rank][T][H / world], the owner's
    // features of tile p at [p * F, (p + 1) * F).
    const int F = a.fslice, W = H / cm.world;
    const int f = n0 & (kTileP - 1), s = f / F;
    const size_t off = (static_cast<size_t>(cm.rank) * T + t) * W + (n0 >> 7) * F + (f - s * F);
    IO* base = reinterpret_cast<IO*>(cm.slots[s] + parity * cm.slot_parity_bytes);
    *reinterpret_cast<uint4*>(base + off) = piece;
  }
}

template <typename IO, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, gemm_ctas_per_sm(BN))
    row_xchg_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ XchgArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_pre;  // stages armed with weight tiles before pdl_wait()
  __shared__ uint32_t s_epoch;
  __shared__ uint64_t s_epoch_bar;  // the producer publishes s_epoch after pdl_wait()
  __shared__ float s_red[32];
  GemmCtl c = gemm_carve_smem<BN, STAGES>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const GemmShape& g = a.g;
  const CommDev& cm = a.cm;

  if (threadIdx.x == 0) {
    trace(1000);
    tma_prefetch_desc(&tm_a);
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
    s_pre = gemm_prefetch_weights<BN, STAGES, true>(g, c, &tm_a, &tm_b, l2_policy_evict_first());
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
      // The epoch counter is written by the previous call on this stream:
      // read it only once that call has finished.
      gemm_producer<BN, STAGES, true>(g, c, &tm_a, &tm_b, l2_policy_evict_first(), l2_policy_evict_last(), s_pre,
                                      [&] {
                                        s_epoch = comm_begin(cm);
                                        mbar_arrive(&s_epoch_bar);
                                      });
    }
  } else if (warp == 1) {
    if (lane == 0) gemm_mma<BN, STAGES>(g, c, umma_idesc_f16(kTileP, BN, std::is_same<IO, __nv_bfloat16>::value));
  } else {
    // Step 1: GEMM epilogue, pushing every finished piece to its reducer(s).
    pdl_wait();
    if (!mbar_wait(&s_epoch_bar, 0u, g.wait_ns, nullptr)) record_error(g.status, kDevTimeoutPipeline);
    const uint32_t e = s_epoch;
    const uint32_t parity = e & 1u;
    const uint32_t tmem = *c.tmem_base;
    const int row = epi_row();
    const int etid = epi_tid();
    if (etid == 0) trace(1001);
    const IO* bias = static_cast<const IO*>(a.bias);
    int acc = 0, done = 0;  // pieces finished (traces only)
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
      if (etid == 0 && done == 0) trace(1002);
      const int nb = tc.p * kTileP + row;
      const float b = (bias != nullptr && nb < g.N) ? io_to_f32<IO>(bias[nb]) : 0.f;
      auto emit = [&](int t, int n0, uint4 piece) { xchg_emit<IO>(a, parity, t, n0, piece); };
      if (tc.nctb > 1) {
        split_reduce_tile<BN>(g, tc, c, tmem, acc, b, [&](const float* v, int t0, int t_lo, int t_hi) {
          swap_epilogue_store<IO>(c.epi, v, t0, t_lo, t_hi, tc.p * kTileP, g.N, emit);
        });
      } else {
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          epi_load_chunk<BN>(tmem, acc, col, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += b;
          swap_epilogue_store<IO>(c.epi, v, tc.q * BN + col, 0, g.T, tc.p * kTileP, g.N, emit);
        }
      }
      tc_fence_before();
      mbar_arrive(&c.acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      if (etid == 0 && done == 0) trace(1003);
      ++done;
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
  const int n = cm.world, T = g.T, H = g.N;
  IO* out = static_cast<IO*>(a.out);
  IO* residual = static_cast<IO*>(a.residual);
  const IO* norm_w = static_cast<const IO*>(a.norm_w);
  // CTA-uniform: every thread of the CTA takes the same branches below.
  bool ok = __syncthreads_and(*reinterpret_cast<volatile int*>(g.status) == 0) != 0;

  // Barrier 0: every rank's step-1 stores have landed. Every CTA calls each
  // barrier, errors or not, so the arrival counters stay balanced.
  if (a.nvls) fence_proxy_alias();  // unicast stores before multicast reads
  ok = grid_cross_barrier(cm, kBarPartials, e, true) && ok;
  if (threadIdx.x == 0) trace(1004);

  // NVLS: rank s sums the s-th share of the [T][H] partials over every GPU in
  // the switch (f32 accumulation, one rounding) and stores it into every
  // GPU's reduced region with one multicast store.
  if (a.nvls) {
    if (ok) {
      const size_t nvec = static_cast<size_t>(T) * H / 8;
      const size_t per = (nvec + n - 1) / n;
      const size_t v0 = static_cast<size_t>(cm.rank) * per;
      const size_t v1 = v0 + per < nvec ? v0 + per : nvec;
      const uint8_t* part = a.nv_mc + parity * a.nv_parity_bytes;
      uint8_t* red = a.nv_mc + parity * a.nv_parity_bytes + a.nv_parity_bytes / 2;
      const size_t nthr = static_cast<size_t>(gridDim.x) * blockDim.x;
#pragma unroll 1
      for (size_t v = v0 + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < v1; v += nthr) {
        const uint4 sum = std::is_same<IO, __nv_bfloat16>::value ? multimem_ld_reduce_bf16x8(part + v * 16)
                                                                  : multimem_ld_reduce_f16x8(part + v * 16);
        multimem_st_16(red + v * 16, sum);
      }
      fence_proxy_alias();
    }
    ok = grid_cross_barrier(cm, kBarResults, e, true) && ok;
    fence_proxy_alias();  // multicast stores before unicast reads
  }

  // Step 2 (two-shot): reduce this rank's slice of each of this CTA's pieces
  // and store it into every rank's y buffer.
  if (!a.oneshot && !a.nvls) {
    if (ok) {
      const int F = a.fslice, W = H / n, per_tok = F / 8;
      const IO* slots = reinterpret_cast<const IO*>(cm.slots[cm.rank] + parity * cm.slot_parity_bytes);
      const size_t src_stride = static_cast<size_t>(T) * W;
      SegIter it(g);
      Seg sg;
      while (it.next(g, sg)) {
        int t0, t1;
        piece_tokens(g, sg, BN, t0, t1);
        const int items = (t1 - t0) * per_tok;
#pragma unroll 1
        for (int i = threadIdx.x; i < items; i += blockDim.x) {
          const int t = t0 + i / per_tok, f8 = i - (i / per_tok) * per_tok;
          const IO* src = slots + static_cast<size_t>(t) * W + sg.p * F + f8 * 8;
          uint4 sv[PGB_MAX_RANKS];
#pragma unroll
          for (int r = 0; r < PGB_MAX_RANKS; ++r)
            if (r < n) sv[r] = __ldcg(reinterpret_cast<const uint4*>(src + r * src_stride));
          float s8[8], p8[8];
          unpack8_io<IO>(sv[0], s8);
#pragma unroll
          for (int r = 1; r < PGB_MAX_RANKS; ++r) {
            if (r < n) {
              unpack8_io<IO>(sv[r], p8);
#pragma unroll
              for (int j = 0; j < 8; ++j) s8[j] += p8[j];
            }
          }
          const size_t yoff = static_cast<size_t>(t) * H + sg.p * kTileP + cm.rank * F + f8 * 8;
          for (int d = 0; d < n; ++d)
            store8<IO>(reinterpret_cast<IO*>(cm.results[d] + parity * cm.result_parity_bytes) + yoff, s8);
        }
      }
    }
    if (threadIdx.x == 0) trace(1006);
    ok = grid_cross_barrier(cm, kBarResults, e, true) && ok;
  }

  // Step 3: residual add + RMSNorm of the rows this CTA owns.
  if (threadIdx.x == 0) trace(1007);
  const bool warp_rows = T > static_cast<int>(gridDim.x);
  if (ok && (warp_rows || static_cast<int>(blockIdx.x) < T)) {
    const IO* base =
        a.nvls ? reinterpret_cast<const IO*>(a.nv_uc + parity * a.nv_parity_bytes + a.nv_parity_bytes / 2)
        : a.oneshot ? reinterpret_cast<const IO*>(cm.slots[cm.rank] + parity * cm.slot_parity_bytes)
                    : reinterpret_cast<const IO*>(cm.results[cm.rank] + parity * cm.result_parity_bytes);
    const int nsrc = (a.oneshot && !a.nvls) ? n : 1;
    const size_t stride = static_cast<size_t>(T) * H;
    bool done_warp = false;
    if constexpr (BN >= 128) {
      constexpr size_t kRing = static_cast<size_t>(STAGES) * GemmSmem<BN, STAGES>::kStageBytes;
      if (warp_rows && static_cast<size_t>(H) * (4u * (kGemmThreads / 32) + 2u) <= kRing) {
        reduce_rows_warp_src<IO>(
            cm, parity, [&](int t) { return base + static_cast<size_t>(t) * H; }, stride, nsrc, false, 0, T, H, out,
            residual, norm_w, a.eps, a.do_norm, c.a);
        done_warp = true;
      }
    }
    if (!done_warp) {
      float* srow = reinterpret_cast<float*>(c.a);
#pragma unroll 1
      for (int t = blockIdx.x; t < T; t += gridDim.x)
        reduce_row_src<IO, kXchgRowMaxVec>(cm, parity, base + static_cast<size_t>(t) * H, stride, nsrc, false, t, H,
                                           out, residual, norm_w, a.eps, a.do_norm, s_red, srow);
    }
  }
  if (threadIdx.x == 0) trace(1008);
  comm_end(cm, e);
  if (threadIdx.x == 0) trace(1009);
}

template <typename IO, int BN>
int launch_xchg(pgb_comm* comm, const XchgArgs& args, const void* x, const void* w, cudaStream_t stream) {
  constexpr int STAGES = gemm_stages<BN>();
  using L = GemmSmem<BN, STAGES>;
  static_assert(L::kBytes + 256 <= 232448, "shared memory budget");
  static_assert(static_cast<size_t>(STAGES) * L::kStageBytes >= kGemmThreads * 8 * kXchgRowMaxVec * (4 + 2),
                "the ring holds one f32 row and its norm weights in the row phase");
  auto kern = row_xchg_kernel<IO, BN, STAGES>;
  PGB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  if (args.g.nsplit > 1 && split_recv_bytes(BN, args.g.nsplit) > static_cast<size_t>(STAGES) * L::kStageBytes)
    return set_error(PGB_ERR_STATE, "row exchange: split of %d does not fit the pipeline ring", args.g.nsplit);
  constexpr bool kBf16 = std::is_same<IO, __nv_bfloat16>::value;
  const int T = args.g.T, N = args.g.N, K = args.g.K;
  CUtensorMap tm_x, tm_w;
  int rc = make_tmap_2d_16bit(&tm_x, x, K, T, static_cast<uint64_t>(K) * 2, kBlockK, BN, kBf16);
  if (rc) return rc;
  rc = make_tmap_2d_16bit(&tm_w, w, K, N, static_cast<uint64_t>(K) * 2, kBlockK, kTileP, kBf16);
  if (rc) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(comm->sm_count);  // every SM takes part in the row phase
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  return launch_ex(cfg, /*cooperative=*/true, 1, kern, tm_w, tm_x, args);
}

template <typename IO>
int dispatch_xchg(pgb_comm* comm, int bn, const XchgArgs& args, const void* x, const void* w, cudaStream_t s) {
  switch (bn) {
    case 32: return launch_xchg<IO, 32>(comm, args, x, w, s);
    case 64: return launch_xchg<IO, 64>(comm, args, x, w, s);
    case 128: return launch_xchg<IO, 128>(comm, args, x, w, s);
    case 256: return launch_xchg<IO, 256>(comm, args, x, w, s);
    default: return set_error(PGB_ERR_INVALID, "row exchange: no kernel for tile width %d", bn);
  }
}

}  // namespace

// Plan and launch the exchange kernel when it applies (several ranks, a
// decode-shaped GEMM, a 16-bit type, a payload the communicator buffers
// hold). Returns PGB_ERR_UNSUPPORTED, without launching, when it does not.
int row_xchg(pgb_comm* comm, const void* x_local, const void* w_local, const void* bias, void* residual,
             const void* norm_w, float eps, void* out, int T, int N, int K_local, int dtype, void* stream) {
  const int n = comm->world;
  if (n < 2 || T > 256 || (dtype != PGB_BF16 && dtype != PGB_F16))
    return PGB_ERR_UNSUPPORTED;
  const double S = 2.0 * T * N;
  const bool can_one = static_cast<double>(n) * S <= static_cast<double>(comm->slot_parity_bytes);
  // Two-shot slices: every rank owns 128 / n features of each 128-feature
  // tile, a whole number of 16-byte pieces (n = 2, 4, 8).
  const bool can_two = kTileP % n == 0 && (kTileP / n) % 8 == 0 && N % kTileP == 0 &&
                       S <= static_cast<double>(comm->slot_parity_bytes) &&
                       S <= static_cast<double>(comm->result_parity_bytes);
  // NVLS: partials of S bytes per rank in the multicast-bound region.
  const bool nvls = comm->exchange_mode == PGB_XCHG_NVLS && comm->nvls && N % 8 == 0 &&
                    S <= static_cast<double>(comm->nv_parity_bytes / 2);
  if (!can_one && !can_two && !nvls) return PGB_ERR_UNSUPPORTED;
  // One-shot sends (n - 1) S per rank in one hop; two-shot 2 (n - 1) / n S
  // in two hops (one more flag round trip, ~2 us measured on NVLink).
  constexpr double kBw = 700e9, kHop = 2e-6;
  const double t_one = (n - 1) * S / kBw, t_two = 2.0 * (n - 1) / n * S / kBw + kHop;
  bool one = can_one && (!can_two || t_one <= t_two);
  if (comm->exchange_mode == PGB_XCHG_ONESHOT && can_one) one = true;
  if (comm->exchange_mode == PGB_XCHG_TWOSHOT && can_two) one = false;

  const GemmPlan p = plan_gemm(T, N, K_local, comm->sm_count, kSplitScratchBytes);
  if (!p.swap) return PGB_ERR_UNSUPPORTED;
  if (p.counter_bytes > kTileCounterBytes)
    return set_error(PGB_ERR_UNSUPPORTED, "row_gemm: too many split tiles (%d)", p.tiles - p.split_first);
  XchgArgs args{};
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
  args.nvls = nvls ? 1 : 0;
  args.nv_uc = reinterpret_cast<uint8_t*>(comm->nv_uc);
  args.nv_mc = reinterpret_cast<uint8_t*>(comm->nv_mc);
  args.nv_parity_bytes = comm->nv_parity_bytes;
  args.oneshot = one ? 1 : 0;
  args.fslice = kTileP / n;
  args.out = out;
  args.residual = residual;
  args.norm_w = norm_w;
  args.bias = bias;
  args.eps = eps;
  args.do_norm = norm_w != nullptr ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PGB_BF16) return dispatch_xchg<__nv_bfloat16>(comm, p.bn, args, x_local, w_local, s);
  return dispatch_xchg<__half>(comm, p.bn, args, x_local, w_local, s);
}

}  // namespace pgb

#ifdef PGB_TRACE
// Work builds only: point this translation unit's trace buffer at `buf`.
extern "C" PGB_API int pgb_debug_set_trace_xchg(void* buf) {
  cudaError_t e = cudaMemcpyToSymbol(pgb::pgb_trace_buf, &buf, sizeof(buf));
  return e == cudaSuccess ? 0 : 2;
}
#endif
