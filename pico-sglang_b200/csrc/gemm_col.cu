// gemm_col.cu - column-parallel GEMM (qkv_proj, gate_up_proj).
//
// y[T, N] = x[T, K] . W[N, K]^T (+ bias), the computation of
// LinearTPImpl.forward (python/picosgl/layers/linear.py:23-27) for the
// column-parallel layers LinearColParallelMerged / LinearColParallelPartitioned
// (linear.py:45-73). No collective follows a column-parallel GEMM.
//
// Gated mode (GLU = true): the gate_up_proj GEMM with silu_and_mul in its
// epilogue, out[T, I] = silu(x . Wg^T) * (x . Wu^T) for the merged weight
// W = [Wg; Wu] of 2I rows, which is GatedMLP.forward's gate_up_proj.forward
// followed by act_fn (python/picosgl/layers/mlp.py:43-46). The [T, 2I]
// intermediate never leaves the SM.
#include "activation.h"
#include "gemm_f32.h"
#include "gemm_plan.h"
#include "gemm_sm100.cuh"
#include "host_common.h"

namespace pgb {

template <typename IO, int BN, bool SWAP, int STAGES, bool GLU>
__global__ void __launch_bounds__(kGemmThreads, gemm_ctas_per_sm(BN))
    col_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    GemmShape g, IO* __restrict__ y, const IO* __restrict__ bias) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_pre;  // stages armed with weight tiles before pdl_wait()
  GemmCtl c = gemm_carve_smem<BN, STAGES>(smem_raw);
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
        const int N = g.N;
        split_reduce_tile<IO, BN, GLU>(g, tc, c, tmem, acc, bias, [&](int t, int n0, uint4 piece) {
          *reinterpret_cast<uint4*>(y + static_cast<size_t>(t) * N + n0) = piece;
        });
      } else if constexpr (GLU && !SWAP) {
        // Lane = token t; columns [0, BN/2) are the gate and [BN/2, BN) the
        // up values of output features q * BN/2 ... Each is rounded to IO
        // (the reference materialises gate_up) before silu(gate) * up.
        const int t = tc.p * kTileP + row;
#pragma unroll 1
        for (int col = 0; col < BN / 2; col += 32) {
          float gv[32], uv[32];
          epi_load_chunk<BN>(tmem, acc, col, gv);
          epi_load_chunk<BN>(tmem, acc, BN / 2 + col, uv);
          const int f0 = tc.q * (BN / 2) + col;
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
      } else {
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          epi_load_chunk<BN>(tmem, acc, col, v);
          if constexpr (SWAP) {
            // Lane = output feature n, columns = tokens: transpose through
            // shared memory and store 16-byte pieces of token rows.
            const int n = swap_weight_row<GLU>(g, tc.p, row);
            if (bias != nullptr && n >= 0) {
              const float b = io_to_f32<IO>(bias[n]);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += b;
            }
            const int N = g.N;
            swap_epilogue_store<IO, GLU>(c.epi, v, tc.q * BN + col, 0, g.T, tc.p * (GLU ? kTileP / 2 : kTileP), N,
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
  if (threadIdx.x == 0) trace(1001);
}

namespace {

// N is the output width; the weight has N rows, or 2N ([gate; up]) when GLU.
template <typename IO, int BN, bool SWAP, bool GLU>
int launch_col(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w,
               const void* bias, void* y, int T, int N, int K, uint8_t* ws, size_t ws_bytes,
               cudaStream_t stream) {
  constexpr int STAGES = gemm_stages<BN>();
  using L = GemmSmem<BN, STAGES>;
  static_assert(L::kBytes <= 232448, "shared memory budget");
  auto kern = col_gemm_kernel<IO, BN, SWAP, STAGES, GLU>;
  if (L::kBytes > dev.max_smem_optin)
    return set_error(PGB_ERR_UNSUPPORTED, "kernel needs %d B shared memory, device allows %d",
                     L::kBytes, dev.max_smem_optin);
  PGB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  if (p.nsplit > 1 && split_recv_bytes(BN, p.nsplit) > static_cast<size_t>(STAGES) * L::kStageBytes)
    return set_error(PGB_ERR_STATE, "col_gemm: split of %d does not fit the pipeline ring", p.nsplit);
  if (col_workspace_bytes(p) > ws_bytes)
    return set_error(PGB_ERR_INVALID, "col_gemm: workspace of %zu bytes, %zu needed", ws_bytes,
                     col_workspace_bytes(p));
  if (p.counter_bytes > kWsCounterBytes)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: %d split tiles exceed the counter region",
                     p.tiles - p.split_first);

  constexpr bool kBf16 = std::is_same<IO, __nv_bfloat16>::value;
  CUtensorMap tm_x, tm_w;
  int rc = make_tmap_2d_16bit(&tm_x, x, K, T, static_cast<uint64_t>(K) * 2, kBlockK,
                              SWAP ? BN : kTileP, kBf16);
  if (rc) return rc;
  constexpr int kWRows = (SWAP ? kTileP : BN) / (GLU ? 2 : 1);  // weight box height
  rc = make_tmap_2d_16bit(&tm_w, w, K, GLU ? 2 * N : N, static_cast<uint64_t>(K) * 2, kBlockK, kWRows, kBf16);
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
  g.status = reinterpret_cast<int*>(ws);
  g.ctr = reinterpret_cast<uint32_t*>(ws + kWsHeaderBytes);
  g.xchg = reinterpret_cast<float*>(ws + kWsHeaderBytes + kWsCounterBytes);
  g.wait_ns = 2000000000ull;  // 2 s: far beyond any legitimate pipeline stall
  g.glu = GLU ? 1 : 0;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  const CUtensorMap& ta = SWAP ? tm_w : tm_x;
  const CUtensorMap& tb = SWAP ? tm_x : tm_w;
  // The CTAs of a split tile wait for each other: cooperative launch.
  return launch_ex(cfg, /*cooperative=*/p.split_ctas > 0, 1, kern, ta, tb, g, static_cast<IO*>(y),
                   static_cast<const IO*>(bias));
}

template <typename IO, bool GLU>
int dispatch_col(const GemmPlan& p, const DeviceInfo& dev, const void* x, const void* w,
                 const void* bias, void* y, int T, int N, int K, uint8_t* ws, size_t wsb,
                 cudaStream_t stream) {
  if (!p.swap) return launch_col<IO, 256, false, GLU>(p, dev, x, w, bias, y, T, N, K, ws, wsb, stream);
  switch (p.bn) {
    case 32: return launch_col<IO, 32, true, GLU>(p, dev, x, w, bias, y, T, N, K, ws, wsb, stream);
    case 64: return launch_col<IO, 64, true, GLU>(p, dev, x, w, bias, y, T, N, K, ws, wsb, stream);
    case 128: return launch_col<IO, 128, true, GLU>(p, dev, x, w, bias, y, T, N, K, ws, wsb, stream);
    case 256: return launch_col<IO, 256, true, GLU>(p, dev, x, w, bias, y, T, N, K, ws, wsb, stream);
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
  if (dtype == PGB_F32) {
    // f32 check mode: CUDA-core GEMM, no workspace.
    if (x == nullptr || w == nullptr || y == nullptr)
      return set_error(PGB_ERR_INVALID, "col_gemm: null pointer argument");
    return launch_gemm_f32(static_cast<const float*>(x), static_cast<const float*>(w),
                           static_cast<const float*>(bias), static_cast<float*>(y), T, N, K,
                           static_cast<cudaStream_t>(stream));
  }
  if (dtype != PGB_BF16 && dtype != PGB_F16)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: dtype %d not supported", dtype);
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
  if (dtype == PGB_BF16)
    return dispatch_col<__nv_bfloat16, false>(p, dev, x, w, bias, y, T, N, K, ws, workspace_bytes, s);
  return dispatch_col<__half, false>(p, dev, x, w, bias, y, T, N, K, ws, workspace_bytes, s);
}

// ---------------------------------------------------------------------------
// gate_up_proj GEMM with silu_and_mul in the epilogue.
//
// The work decomposition is that of the unfused [T, 2I] GEMM: a swap tile
// pairs 64 gate rows with their 64 up rows, a prefill tile 128 with 128, so
// plan_gemm(T, 2I, K) gives the same tile count, splits and scratch. The f32
// check mode runs the f32 GEMM into the workspace and the activation kernel
// after it.
// ---------------------------------------------------------------------------

namespace {
size_t f32_gate_up_bytes(int T, int I) { return static_cast<size_t>(T) * 2u * static_cast<size_t>(I) * 4u; }
}  // namespace

extern "C" size_t pgb_gate_up_silu_workspace_size(int T, int I, int K, int dtype) {
  using namespace pgb;
  if (T <= 0 || I <= 0 || K <= 0) return kWsHeaderBytes;
  if (dtype == PGB_F32) return kWsHeaderBytes + kWsCounterBytes + f32_gate_up_bytes(T, I);
  const GemmPlan p = plan_gemm(T, 2 * I, K, sm_count_or_default(), SIZE_MAX);
  return col_workspace_bytes(p);
}

extern "C" int pgb_gate_up_silu(const void* x, const void* w, const void* bias, void* out, int T, int I,
                                int K, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace pgb;
  if (T < 0 || I <= 0 || K <= 0 || I > (1 << 29))
    return set_error(PGB_ERR_INVALID, "gate_up_silu: bad shape T=%d I=%d K=%d", T, I, K);
  if (T == 0) return PGB_OK;
  if (x == nullptr || w == nullptr || out == nullptr || workspace == nullptr)
    return set_error(PGB_ERR_INVALID, "gate_up_silu: null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PGB_F32) {
    // f32 check mode: gate_up in the workspace's exchange area (the
    // counters before it stay untouched), then the activation.
    const size_t need = kWsHeaderBytes + kWsCounterBytes + f32_gate_up_bytes(T, I);
    if (workspace_bytes < need)
      return set_error(PGB_ERR_INVALID, "gate_up_silu: workspace of %zu bytes, %zu needed", workspace_bytes,
                       need);
    float* gu =
        reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsHeaderBytes + kWsCounterBytes);
    int rc = launch_gemm_f32(static_cast<const float*>(x), static_cast<const float*>(w),
                             static_cast<const float*>(bias), gu, T, 2 * I, K, s);
    if (rc) return rc;
    return launch_silu_and_mul(gu, out, T, I, PGB_F32, s);
  }
  if (dtype != PGB_BF16 && dtype != PGB_F16)
    return set_error(PGB_ERR_UNSUPPORTED, "gate_up_silu: dtype %d not supported", dtype);
  if (K % 8 != 0 || I % 8 != 0)
    return set_error(PGB_ERR_INVALID, "gate_up_silu: K=%d and I=%d must be multiples of 8", K, I);
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0u)
    return set_error(PGB_ERR_INVALID, "gate_up_silu: output is not 16-byte aligned");
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const GemmPlan p = plan_gemm(T, 2 * I, K, dev.sm_count, SIZE_MAX);
  const size_t need = col_workspace_bytes(p);
  if (workspace_bytes < need)
    return set_error(PGB_ERR_INVALID, "gate_up_silu: workspace of %zu bytes, %zu needed", workspace_bytes,
                     need);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (dtype == PGB_BF16)
    return dispatch_col<__nv_bfloat16, true>(p, dev, x, w, bias, out, T, I, K, ws, workspace_bytes, s);
  return dispatch_col<__half, true>(p, dev, x, w, bias, out, T, I, K, ws, workspace_bytes, s);
}

// ---------------------------------------------------------------------------
// Allocation-free column GEMM.
//
// Some callers cannot allocate device memory at the point where they run the
// GEMM. Examples are a serving runtime that has already handed nearly all of
// HBM to its KV-cache pool, an allocator hook that must not re-enter the
// allocator, and code on a latency path where cudaMalloc/cudaFree would
// synchronise the device. pgb_col_gemm_noalloc serves them: its split-K
// scratch (status word, split-tile counters, exchange area) is a fixed array inside this library's device image, so the call
// itself allocates nothing.
//
// Limits and rules:
//  - The scratch is PGB_NOALLOC_SCRATCH_BYTES per device. A shape whose plan
//    needs more is refused with PGB_ERR_INVALID.
//  - All calls on one device share that scratch. Two calls whose GPU work
//    overlaps (different streams, no ordering between them) race on it and
//    give wrong results. Order them on one stream, or use pgb_col_gemm with a
//    workspace per stream.
//  - The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current). Make that first call
//    before any stream capture.
// ---------------------------------------------------------------------------

static __device__ __align__(256) uint8_t pgb_noalloc_scratch[PGB_NOALLOC_SCRATCH_BYTES];

namespace pgb {
namespace {

constexpr int kNoAllocMaxDevices = 64;

// Device address of pgb_noalloc_scratch on the current device; looked up once
// per device and cached.
int noalloc_scratch(uint8_t** out) {
  static std::mutex mu;
  static void* addr[kNoAllocMaxDevices] = {};
  int dev = 0;
  PGB_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm_noalloc: device ordinal %d above %d", dev,
                     kNoAllocMaxDevices - 1);
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, pgb_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(pgb_noalloc_scratch)");
    if (p == nullptr) return set_error(PGB_ERR_CUDA, "col_gemm_noalloc: null scratch address");
    addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(addr[dev]);
  return PGB_OK;
}

}  // namespace
}  // namespace pgb

extern "C" int pgb_col_gemm_noalloc(const void* x, const void* w, const void* bias, void* y, int T,
                                    int N, int K, int dtype, void* stream) {
  using namespace pgb;
  if (T < 0 || N <= 0 || K <= 0)
    return set_error(PGB_ERR_INVALID, "col_gemm_noalloc: bad shape T=%d N=%d K=%d", T, N, K);
  if (T == 0) return PGB_OK;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const GemmPlan p = plan_gemm(T, N, K, dev.sm_count, SIZE_MAX);
  const size_t need = col_workspace_bytes(p);
  if (need > PGB_NOALLOC_SCRATCH_BYTES)
    return set_error(PGB_ERR_INVALID,
                     "col_gemm_noalloc: T=%d N=%d K=%d needs %zu bytes of scratch, above the fixed "
                     "%zu; call pgb_col_gemm with a workspace instead",
                     T, N, K, need, static_cast<size_t>(PGB_NOALLOC_SCRATCH_BYTES));
  uint8_t* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // The status word and the split-tile counters must start at zero; the
  // exchange area behind them is written before it is read.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PGB_CUDA_TRY(cudaMemsetAsync(scratch, 0, kWsHeaderBytes + kWsCounterBytes, s));
  return pgb_col_gemm(x, w, bias, y, T, N, K, dtype, scratch, PGB_NOALLOC_SCRATCH_BYTES, stream);
}

#ifdef PGB_TRACE
// Work-build only: point this translation unit's trace buffer at `buf`.
extern "C" PGB_API int pgb_debug_set_trace(void* buf) {
  cudaError_t e = cudaMemcpyToSymbol(pgb::pgb_trace_buf, &buf, sizeof(buf));
  return e == cudaSuccess ? 0 : 2;
}
#endif
