// gemm_col.cu - column-parallel GEMM (qkv_proj, gate_up_proj).
//
// y[T, N] = x[T, K] . W[N, K]^T (+ bias), the computation of
// LinearTPImpl.forward (python/picosgl/layers/linear.py:23-27) for the
// column-parallel layers LinearColParallelMerged / LinearColParallelPartitioned
// (linear.py:45-73). No collective follows a column-parallel GEMM.
#include "gemm_plan.h"
#include "gemm_sm100.cuh"
#include "host_common.h"

namespace pgb {

template <typename IO, int BN, bool SWAP, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    col_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    GemmShape g, IO* __restrict__ y, const IO* __restrict__ bias) {
  extern __shared__ uint8_t smem_raw[];
  GemmCtl c = gemm_carve_smem<BN, STAGES>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    mbar_init(&c.acc_full[0], 1);
    mbar_init(&c.acc_full[1], 1);
    mbar_init(&c.acc_empty[0], kEpiThreads);
    mbar_init(&c.acc_empty[1], kEpiThreads);
    mbar_init(c.drain, 1);
    *c.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(c.tmem_base, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t hw = l2_policy_evict_first();
      const uint64_t hx = l2_policy_evict_last();
      gemm_producer<BN, STAGES>(g, c, &tm_a, &tm_b, SWAP ? hw : hx, SWAP ? hx : hw);
    }
  } else if (warp == 1) {
    if (lane == 0) gemm_mma<BN, STAGES>(g, c, umma_idesc_f16(kTileP, BN, std::is_same<IO, __nv_bfloat16>::value));
  } else {
    const uint32_t tmem = *c.tmem_base;
    const int row = epi_row();
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = blockIdx.x; unit < g.num_units; unit += gridDim.x) {
      const TileCoord tc = decode_unit(g, unit);
      if (!mbar_wait(&c.acc_full[acc], acc_phase, g.wait_ns, c.abort)) {
        record_error(g.status, kDevTimeoutPipeline);
        *reinterpret_cast<volatile int*>(c.abort) = 1;
        break;
      }
      tc_fence_after();
      bool owner = true;
      if (g.splits > 1) owner = splitk_publish<BN>(g, c, tc, tmem, acc);
      if (owner) {
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          epi_load_chunk<BN>(g, tc, tmem, acc, col, v);
          if constexpr (SWAP) {
            // Lane = output feature n, columns = tokens: transpose through
            // shared memory and store 16-byte pieces of token rows.
            const int n = tc.p * kTileP + row;
            if (bias != nullptr && n < g.N) {
              const float b = io_to_f32<IO>(bias[n]);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += b;
            }
            const int N = g.N;
            swap_epilogue_store<IO>(c.epi, v, tc.q * BN + col, g.T, tc.p * kTileP, N,
                                    [&](int t, int n0, uint4 piece) {
                                      *reinterpret_cast<uint4*>(y + static_cast<size_t>(t) * N + n0) = piece;
                                    });
          } else {
            // Lane = token t, columns = output features.
            const int t = tc.p * kTileP + row;
            const int n0 = tc.q * BN + col;
            if (t < g.T) {
              IO* dst = y + static_cast<size_t>(t) * g.N + n0;
              if (bias != nullptr) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (n0 + j < g.N) v[j] += io_to_f32<IO>(bias[n0 + j]);
              }
              if (n0 + 32 <= g.N) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  reinterpret_cast<uint4*>(dst)[j] = pack8<IO>(v + 8 * j);
              } else {
                for (int j = 0; j < 32 && n0 + j < g.N; ++j) dst[j] = f32_to_io<IO>(v[j]);
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
}

namespace {

template <typename IO, int BN, bool SWAP>
int launch_col(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w,
               const void* bias, void* y, int T, int N, int K, uint8_t* ws, cudaStream_t stream) {
  constexpr int STAGES = gemm_stages<BN>();
  using L = GemmSmem<BN, STAGES>;
  static_assert(L::kBytes <= 232448, "shared memory budget");
  auto kern = col_gemm_kernel<IO, BN, SWAP, STAGES>;
  if (L::kBytes > dev.max_smem_optin)
    return set_error(PGB_ERR_UNSUPPORTED, "kernel needs %d B shared memory, device allows %d",
                     L::kBytes, dev.max_smem_optin);
  PGB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));

  constexpr bool kBf16 = std::is_same<IO, __nv_bfloat16>::value;
  CUtensorMap tm_x, tm_w;
  int rc = make_tmap_2d_16bit(&tm_x, x, K, T, static_cast<uint64_t>(K) * 2, kBlockK,
                              SWAP ? BN : kTileP, kBf16);
  if (rc) return rc;
  rc = make_tmap_2d_16bit(&tm_w, w, K, N, static_cast<uint64_t>(K) * 2, kBlockK,
                          SWAP ? kTileP : BN, kBf16);
  if (rc) return rc;

  GemmShape g{};
  g.T = T;
  g.N = N;
  g.K = K;
  g.kblocks = p.kblocks;
  g.splits = p.splits;
  g.p_tiles = p.p_tiles;
  g.q_tiles = p.q_tiles;
  g.num_units = p.units;
  g.status = reinterpret_cast<int*>(ws);
  g.tile_counters = reinterpret_cast<uint32_t*>(ws + kWsHeaderBytes);
  g.ws = reinterpret_cast<float*>(ws + kWsHeaderBytes + p.counter_bytes);
  g.wait_ns = 2000000000ull;  // 2 s: far beyond any legitimate pipeline stall

  kern<<<p.grid, kGemmThreads, L::kBytes, stream>>>(SWAP ? tm_w : tm_x, SWAP ? tm_x : tm_w, g,
                                                    static_cast<IO*>(y),
                                                    static_cast<const IO*>(bias));
  PGB_CUDA_TRY(cudaGetLastError());
  return PGB_OK;
}

template <typename IO>
int dispatch_col(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w,
                 const void* bias, void* y, int T, int N, int K, uint8_t* ws,
                 cudaStream_t stream) {
  if (!p.swap) return launch_col<IO, 256, false>(p, dev, x, w, bias, y, T, N, K, ws, stream);
  switch (p.bn) {
    case 32: return launch_col<IO, 32, true>(p, dev, x, w, bias, y, T, N, K, ws, stream);
    case 64: return launch_col<IO, 64, true>(p, dev, x, w, bias, y, T, N, K, ws, stream);
    case 128: return launch_col<IO, 128, true>(p, dev, x, w, bias, y, T, N, K, ws, stream);
    case 256: return launch_col<IO, 256, true>(p, dev, x, w, bias, y, T, N, K, ws, stream);
    default: return set_error(PGB_ERR_INVALID, "no kernel for tile width %d", p.bn);
  }
}

int sm_count_or_default() {
  DeviceInfo d;
  if (current_device_info(&d) == PGB_OK) return d.sm_count;
  return 148;
}

}  // namespace

}  // namespace pgb

extern "C" size_t pgb_col_gemm_workspace_size(int T, int N, int K) {
  if (T <= 0 || N <= 0 || K <= 0) return pgb::kWsHeaderBytes;
  const pgb::GemmPlan p = pgb::plan_gemm(T, N, K, pgb::sm_count_or_default(), SIZE_MAX);
  return pgb::col_workspace_bytes(p);
}

extern "C" int pgb_col_gemm(const void* x, const void* w, const void* bias, void* y, int T, int N,
                            int K, int dtype, void* workspace, size_t workspace_bytes,
                            void* stream) {
  using namespace pgb;
  if (T < 0 || N <= 0 || K <= 0)
    return set_error(PGB_ERR_INVALID, "col_gemm: bad shape T=%d N=%d K=%d", T, N, K);
  if (T == 0) return PGB_OK;
  if (dtype != PGB_BF16 && dtype != PGB_F16)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: dtype %d not supported (bf16/f16 only)", dtype);
  if (K % 8 != 0 || N % 8 != 0)
    return set_error(PGB_ERR_INVALID, "col_gemm: K=%d and N=%d must be multiples of 8", K, N);
  if (x == nullptr || w == nullptr || y == nullptr || workspace == nullptr)
    return set_error(PGB_ERR_INVALID, "col_gemm: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(y) & 15u) != 0u)
    return set_error(PGB_ERR_INVALID, "col_gemm: output is not 16-byte aligned");
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const GemmPlan p = plan_gemm(T, N, K, dev.sm_count, SIZE_MAX);
  const size_t need = col_workspace_bytes(p);
  if (workspace_bytes < need)
    return set_error(PGB_ERR_INVALID, "col_gemm: workspace of %zu bytes, %zu needed", workspace_bytes,
                     need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (dtype == PGB_BF16) return dispatch_col<__nv_bfloat16>(p, dev, x, w, bias, y, T, N, K, ws, s);
  return dispatch_col<__half>(p, dev, x, w, bias, y, T, N, K, ws, s);
}
