// gemm_col.cu - column-parallel GEMM (qkv_proj, gate_up_proj).
//
// y[T, N] = x[T, K] . W[N, K]^T (+ bias), the computation of
// LinearTPImpl.forward (python/picosgl/layers/linear.py:23-27) for the
// column-parallel layers LinearColParallelMerged / LinearColParallelPartitioned
// (linear.py:45-73). No collective follows a column-parallel GEMM.
//
// Gated mode (EpiGlu): the gate_up_proj GEMM with silu_and_mul in its
// epilogue, out[T, I] = silu(x . Wg^T) * (x . Wu^T) for the merged weight
// W = [Wg; Wu] of 2I rows, which is GatedMLP.forward's gate_up_proj.forward
// followed by act_fn (python/picosgl/layers/mlp.py:43-46). The [T, 2I]
// intermediate never leaves the SM.
#include "activation.h"
#include "col_kernel.cuh"
#include "gemm_f32.h"

namespace pgb {

namespace {

int sm_count_or_default() {
  DeviceInfo d;
  if (current_device_info(&d) == PGB_OK) return d.sm_count;
  return 148;
}

}  // namespace

int col_gemm_on_scratch(const void* x, const void* w, const void* bias, void* y, int T, int N, int K, int dtype,
                        const ColScratch& sc, void* stream) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const GemmPlan p = plan_gemm_col(T, N, K, dev.sm_count, sc.xchg_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PGB_BF16)
    return dispatch_col<__nv_bfloat16>(p, dev, x, w, T, N, K, sc, s,
                                       EpiPlain<__nv_bfloat16>{static_cast<__nv_bfloat16*>(y),
                                                               static_cast<const __nv_bfloat16*>(bias)});
  if (dtype == PGB_F16)
    return dispatch_col<__half>(p, dev, x, w, T, N, K, sc, s,
                                EpiPlain<__half>{static_cast<__half*>(y), static_cast<const __half*>(bias)});
  return set_error(PGB_ERR_UNSUPPORTED, "col_gemm: dtype %d not supported", dtype);
}

}  // namespace pgb

extern "C" size_t pgb_col_gemm_workspace_size(int T, int N, int K) {
  if (T <= 0 || N <= 0 || K <= 0) return pgb::kWsHeaderBytes;
  const pgb::GemmPlan p = pgb::plan_gemm_col(T, N, K, pgb::sm_count_or_default(), SIZE_MAX);
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
  const GemmPlan p = plan_gemm_col(T, N, K, dev.sm_count, SIZE_MAX);
  const size_t need = col_workspace_bytes(p);
  if (workspace_bytes < need)
    return set_error(PGB_ERR_INVALID, "col_gemm: workspace of %zu bytes, %zu needed", workspace_bytes,
                     need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const ColScratch sc = col_scratch(ws, workspace_bytes);
  if (dtype == PGB_BF16)
    return dispatch_col<__nv_bfloat16>(p, dev, x, w, T, N, K, sc, s,
                                       EpiPlain<__nv_bfloat16>{static_cast<__nv_bfloat16*>(y),
                                                               static_cast<const __nv_bfloat16*>(bias)});
  return dispatch_col<__half>(p, dev, x, w, T, N, K, sc, s,
                              EpiPlain<__half>{static_cast<__half*>(y), static_cast<const __half*>(bias)});
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
  const GemmPlan p = plan_gemm_col(T, 2 * I, K, sm_count_or_default(), SIZE_MAX);
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
  const GemmPlan p = plan_gemm_col(T, 2 * I, K, dev.sm_count, SIZE_MAX);
  const size_t need = col_workspace_bytes(p);
  if (workspace_bytes < need)
    return set_error(PGB_ERR_INVALID, "gate_up_silu: workspace of %zu bytes, %zu needed", workspace_bytes,
                     need);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const ColScratch sc = col_scratch(ws, workspace_bytes);
  if (dtype == PGB_BF16)
    return dispatch_col<__nv_bfloat16>(p, dev, x, w, T, I, K, sc, s,
                                       EpiGlu<__nv_bfloat16>{static_cast<__nv_bfloat16*>(out),
                                                             static_cast<const __nv_bfloat16*>(bias)});
  return dispatch_col<__half>(p, dev, x, w, T, I, K, sc, s,
                              EpiGlu<__half>{static_cast<__half*>(out), static_cast<const __half*>(bias)});
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
//    before any stream capture. The address is kept for the life of the
//    process, so the library must not be used across a cudaDeviceReset.
//  - The kernel's status word sits in the array too and is sticky: a
//    device-side wait that ran out leaves it set until
//    pgb_col_gemm_noalloc_status reads and resets it.
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
  // f32 check mode runs the CUDA-core GEMM, which uses no scratch at all.
  if (dtype == PGB_F32) return pgb_col_gemm(x, w, bias, y, T, N, K, dtype, nullptr, 0, stream);
  // Everything pgb_col_gemm would refuse is refused here first, so a refused
  // call never touches the shared scratch.
  if (dtype != PGB_BF16 && dtype != PGB_F16)
    return set_error(PGB_ERR_UNSUPPORTED, "col_gemm_noalloc: dtype %d not supported", dtype);
  if (K % 8 != 0 || N % 8 != 0)
    return set_error(PGB_ERR_INVALID, "col_gemm_noalloc: K=%d and N=%d must be multiples of 8", K, N);
  if (x == nullptr || w == nullptr || y == nullptr)
    return set_error(PGB_ERR_INVALID, "col_gemm_noalloc: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(y) & 15u) != 0u)
    return set_error(PGB_ERR_INVALID, "col_gemm_noalloc: output is not 16-byte aligned");
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const GemmPlan p = plan_gemm_col(T, N, K, dev.sm_count, SIZE_MAX);
  const size_t need = col_workspace_bytes(p);
  if (need > PGB_NOALLOC_SCRATCH_BYTES)
    return set_error(PGB_ERR_INVALID,
                     "col_gemm_noalloc: T=%d N=%d K=%d needs %zu bytes of scratch, above the fixed "
                     "%zu; call pgb_col_gemm with a workspace instead",
                     T, N, K, need, static_cast<size_t>(PGB_NOALLOC_SCRATCH_BYTES));
  uint8_t* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // The split-tile counters must start at zero; the exchange area behind
  // them is written before it is read. The status word in the header is left
  // alone: it stays set after a device-side wait ran out, until
  // pgb_col_gemm_noalloc_status resets it.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PGB_CUDA_TRY(cudaMemsetAsync(scratch + kWsHeaderBytes, 0, kWsCounterBytes, s));
  return pgb_col_gemm(x, w, bias, y, T, N, K, dtype, scratch, PGB_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int pgb_col_gemm_noalloc_status(int* out, int reset) {
  using namespace pgb;
  if (out == nullptr) return set_error(PGB_ERR_INVALID, "col_gemm_noalloc_status: null output");
  uint8_t* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  PGB_CUDA_TRY(cudaDeviceSynchronize());
  int v = 0;
  PGB_CUDA_TRY(cudaMemcpy(&v, scratch, sizeof(int), cudaMemcpyDeviceToHost));
  *out = v == kDevOk ? PGB_OK : (v == kDevBadArgs ? PGB_ERR_INVALID : PGB_ERR_TIMEOUT);
  if (reset) PGB_CUDA_TRY(cudaMemset(scratch, 0, sizeof(int)));
  return PGB_OK;
}

#ifdef PGB_TRACE
// Work-build only: point this translation unit's trace buffer at `buf`.
extern "C" PGB_API int pgb_debug_set_trace(void* buf) {
  cudaError_t e = cudaMemcpyToSymbol(pgb::pgb_trace_buf, &buf, sizeof(buf));
  return e == cudaSuccess ? 0 : 2;
}

namespace {
__global__ void trace_selftest_kernel() { pgb::trace(7); }
}  // namespace

// Work-build only: reads the pointer back and records slot 7 of CTA 0 from a
// one-thread kernel. Returns 0 when the pointer read back equals `expect`.
extern "C" PGB_API int pgb_debug_trace_selftest(void* expect) {
  void* got = nullptr;
  if (cudaMemcpyFromSymbol(&got, pgb::pgb_trace_buf, sizeof(got)) != cudaSuccess) return 2;
  trace_selftest_kernel<<<1, 1>>>();
  if (cudaDeviceSynchronize() != cudaSuccess) return 3;
  return got == expect ? 0 : 1;
}
#endif
