// norm.cu - standalone RMSNorm kernels for the norms that are not fused
// into a row-parallel GEMM: the first layer's input_layernorm (residual is
// None, python/picosgl/layers/norm.py:71-72) and any fused_add_rmsnorm whose
// producer is not a row-parallel layer (norm.py:73-75).
//
// One CTA per row, 8-element vectors, f32 statistics; the semantics of
// FlashInfer's RMSNormKernel / FusedAddRMSNormKernel (norm.cuh:387-470):
// the f32 sum x + residual is normalised and stored into residual rounded.
#include "host_common.h"
#include "reduce_phases.cuh"

namespace pgb {

constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 8;     // width <= 256 * 64 = 16384
constexpr int kAddNormMaxVec = 4;  // fused_add_rmsnorm_kernel: width <= 256 * 32 = 8192 (wider rows: the rows kernel)

template <typename IO>
__global__ void __launch_bounds__(kNormThreads) fused_add_rmsnorm_kernel(IO* x, IO* residual,
                                                                         const IO* w, float eps,
                                                                         int width) {
  __shared__ float red[32];
  // The next kernel (a GEMM) may become resident now and prefetch its
  // weights; it reads this kernel's outputs only after its own wait.
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const int nvec = width >> 3;
  float s[kAddNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kAddNormMaxVec; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nvec) {
      float a[8], r[8];
      load8<IO>(x + static_cast<size_t>(t) * width + v * 8, a);
      load8<IO>(residual + static_cast<size_t>(t) * width + v * 8, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[i][j] = a[j] + r[j];
        ss += s[i][j] * s[i][j];
      }
    }
  }
  // The norm weights' loads are issued before the reduction, off its
  // critical path; the residual is stored while the reduction runs.
  float wv[kAddNormMaxVec][8];
#pragma unroll
  for (int i = 0; i < kAddNormMaxVec; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nvec) {
      load8<IO>(w + v * 8, wv[i]);
      store8<IO>(residual + static_cast<size_t>(t) * width + v * 8, s[i]);
    }
  }
  const float rcp = rsqrtf(block_sum(ss, red) / static_cast<float>(width) + eps);
#pragma unroll
  for (int i = 0; i < kAddNormMaxVec; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nvec) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = s[i][j] * rcp * wv[i][j];
      store8<IO>(x + static_cast<size_t>(t) * width + v * 8, o);
    }
  }
}

// Long batches (prefill): one warp per row, 8 rows per CTA, rows strided over
// a grid of at most 8 CTAs per SM. Pass 1 forms s = x + residual in f32 and
// its sum of squares with many 16-byte loads in flight per lane; pass 2 reads
// x and residual again (from L2, just fetched), forms the same s, stores the
// rounded residual and s * rcp * w. The same arithmetic as
// fused_add_rmsnorm_kernel except the order of the squares' sum.
template <typename IO>
__global__ void __launch_bounds__(kNormThreads) fused_add_rmsnorm_rows_kernel(IO* x, IO* residual, const IO* w,
                                                                              float eps, int T, int width) {
  if (threadIdx.x == 0) pdl_launch_dependents();  // as in fused_add_rmsnorm_kernel
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = width >> 3;
  for (int t = blockIdx.x * (kNormThreads / 32) + warp; t < T; t += gridDim.x * (kNormThreads / 32)) {
    IO* xr = x + static_cast<size_t>(t) * width;
    IO* rr = residual + static_cast<size_t>(t) * width;
    float ss = 0.f;
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      float a[8], r[8];
      load8<IO>(xr + v * 8, a);
      load8<IO>(rr + v * 8, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sj = a[j] + r[j];
        ss += sj * sj;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rcp = rsqrtf(ss / static_cast<float>(width) + eps);
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      float a[8], r[8], wv[8], o[8];
      load8<IO>(xr + v * 8, a);
      load8<IO>(rr + v * 8, r);
      load8<IO>(w + v * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a[j] += r[j];
        o[j] = a[j] * rcp * wv[j];
      }
      store8<IO>(rr + v * 8, a);
      store8<IO>(xr + v * 8, o);
    }
  }
}

// Batches from this size up use fused_add_rmsnorm_rows_kernel.
constexpr int kNormRowsKernelMinT = 1024;

template <typename IO>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const IO* x, const IO* w, float eps,
                                                               IO* out, int width) {
  __shared__ float red[32];
  if (threadIdx.x == 0) pdl_launch_dependents();  // as in fused_add_rmsnorm_kernel
  pdl_wait();
  const int t = blockIdx.x;
  const int nvec = width >> 3;
  float s[kNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nvec) {
      load8<IO>(x + static_cast<size_t>(t) * width + v * 8, s[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += s[i][j] * s[i][j];
    }
  }
  const float rcp = rsqrtf(block_sum(ss, red) / static_cast<float>(width) + eps);
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nvec) {
      float wv[8], o[8];
      load8<IO>(w + v * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = s[i][j] * rcp * wv[j];
      store8<IO>(out + static_cast<size_t>(t) * width + v * 8, o);
    }
  }
}

namespace {
template <typename K, typename... Args>
int launch_norm(cudaStream_t s, int T, K kern, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(T);
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = s;
  return launch_ex(cfg, /*cooperative=*/false, 1, kern, args...);
}

int check_norm_args(const char* what, int T, int H, int dtype, const void* a, const void* b,
                    const void* c) {
  if (T < 0 || H <= 0) return set_error(PGB_ERR_INVALID, "%s: bad shape T=%d H=%d", what, T, H);
  if (H % 8 != 0) return set_error(PGB_ERR_INVALID, "%s: hidden size %d not a multiple of 8", what, H);
  if (H > kNormThreads * 8 * kNormMaxVec)
    return set_error(PGB_ERR_UNSUPPORTED, "%s: hidden size %d above %d", what, H,
                     kNormThreads * 8 * kNormMaxVec);
  if (dtype != PGB_BF16 && dtype != PGB_F16 && dtype != PGB_F32)
    return set_error(PGB_ERR_INVALID, "%s: unknown dtype %d", what, dtype);
  const uintptr_t m = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                      reinterpret_cast<uintptr_t>(c);
  if (a == nullptr || b == nullptr || c == nullptr)
    return set_error(PGB_ERR_INVALID, "%s: null pointer argument", what);
  if ((m & 15u) != 0u) return set_error(PGB_ERR_INVALID, "%s: pointers must be 16-byte aligned", what);
  return PGB_OK;
}
}  // namespace

}  // namespace pgb

extern "C" int pgb_fused_add_rmsnorm(void* x, void* residual, const void* w, float eps, int T,
                                     int H, int dtype, void* stream) {
  using namespace pgb;
  int rc = check_norm_args("fused_add_rmsnorm", T, H, dtype, x, residual, w);
  if (rc || T == 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T >= kNormRowsKernelMinT || H > kNormThreads * 8 * kAddNormMaxVec) {
    DeviceInfo dev;
    rc = current_device_info(&dev);
    if (rc) return rc;
    const int grid = std::min((T + kNormThreads / 32 - 1) / (kNormThreads / 32), 8 * dev.sm_count);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kNormThreads);
    cfg.stream = s;
    switch (dtype) {
      case PGB_BF16:
        return launch_ex(cfg, false, 1, fused_add_rmsnorm_rows_kernel<__nv_bfloat16>,
                         static_cast<__nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(residual),
                         static_cast<const __nv_bfloat16*>(w), eps, T, H);
      case PGB_F16:
        return launch_ex(cfg, false, 1, fused_add_rmsnorm_rows_kernel<__half>, static_cast<__half*>(x),
                         static_cast<__half*>(residual), static_cast<const __half*>(w), eps, T, H);
      default:
        return launch_ex(cfg, false, 1, fused_add_rmsnorm_rows_kernel<float>, static_cast<float*>(x),
                         static_cast<float*>(residual), static_cast<const float*>(w), eps, T, H);
    }
  }
  switch (dtype) {
    case PGB_BF16:
      rc = launch_norm(s, T, fused_add_rmsnorm_kernel<__nv_bfloat16>, 
          static_cast<__nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(residual),
          static_cast<const __nv_bfloat16*>(w), eps, H);
      break;
    case PGB_F16:
      rc = launch_norm(s, T, fused_add_rmsnorm_kernel<__half>, 
          static_cast<__half*>(x), static_cast<__half*>(residual), static_cast<const __half*>(w), eps, H);
      break;
    default:
      rc = launch_norm(s, T, fused_add_rmsnorm_kernel<float>, 
          static_cast<float*>(x), static_cast<float*>(residual), static_cast<const float*>(w), eps, H);
  }
  return rc;
}

extern "C" int pgb_rmsnorm(const void* x, const void* w, float eps, void* out, int T, int H,
                           int dtype, void* stream) {
  using namespace pgb;
  int rc = check_norm_args("rmsnorm", T, H, dtype, x, w, out);
  if (rc || T == 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PGB_BF16:
      rc = launch_norm(s, T, rmsnorm_kernel<__nv_bfloat16>, 
          static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), eps,
          static_cast<__nv_bfloat16*>(out), H);
      break;
    case PGB_F16:
      rc = launch_norm(s, T, rmsnorm_kernel<__half>, static_cast<const __half*>(x),
                                                       static_cast<const __half*>(w), eps,
                                                       static_cast<__half*>(out), H);
      break;
    default:
      rc = launch_norm(s, T, rmsnorm_kernel<float>, static_cast<const float*>(x),
                                                      static_cast<const float*>(w), eps,
                                                      static_cast<float*>(out), H);
  }
  return rc;
}
