// gemm_f32.cu - f32 check mode of the linear path.
//
// y[T, N] = x[T, K] . W[N, K]^T (+ bias) in IEEE f32 on the CUDA cores:
// fused multiply-adds within each 16-deep k slice, slice sums added in
// increasing k order. This is the precision a float32 model gets from the
// reference's F.linear (python/picosgl/layers/linear.py:23-27) with TF32
// disabled, and what the f32 check mode compares the fused bf16 path with.
// It is not a hot path: 128 x 128 output tiles, 16-deep k slices staged in
// shared memory, 8 x 8 outputs per thread.
#include "gemm_f32.h"
#include "host_common.h"
#include "sm100.cuh"

namespace pgb {

namespace {
constexpr int kTile = 128;
constexpr int kSlice = 16;
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) gemm_f32_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            int T, int N, int K) {
  __shared__ float xs[kSlice][kTile + 4];  // [k][token]
  __shared__ float ws[kSlice][kTile + 4];  // [k][feature]
  pdl_wait();
  const int t0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;  // outputs (t0 + ty + 16 i, n0 + tx + 16 j)
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += kSlice) {
#pragma unroll
    for (int i = 0; i < kTile * kSlice / kThreads; ++i) {
      const int e = tid + i * kThreads;
      const int r = e / kSlice, kk = e % kSlice;
      const int k = k0 + kk;
      xs[kk][r] = (t0 + r < T && k < K) ? x[static_cast<size_t>(t0 + r) * K + k] : 0.f;
      ws[kk][r] = (n0 + r < N && k < K) ? w[static_cast<size_t>(n0 + r) * K + k] : 0.f;
    }
    __syncthreads();
    // Two-level sum: the 16 products of a slice are accumulated from zero,
    // then the slice sum is added to the running total (pairwise-style
    // error growth instead of the sequential sum's).
    float part[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) part[i][j] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kSlice; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = xs[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = ws[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) part[i][j] = fmaf(a[i], b[j], part[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] += part[i][j];
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = t0 + ty + 16 * i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n < N) y[static_cast<size_t>(t) * N + n] = acc[i][j] + (bias != nullptr ? bias[n] : 0.f);
    }
  }
}
}  // namespace

int launch_gemm_f32(const float* x, const float* w, const float* bias, float* y, int T, int N, int K,
                    cudaStream_t stream) {
  if (T == 0) return PGB_OK;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((N + kTile - 1) / kTile, (T + kTile - 1) / kTile);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  return launch_ex(cfg, /*cooperative=*/false, 1, gemm_f32_kernel, x, w, bias, y, T, N, K);
}

}  // namespace pgb
