// gemm_f32.h - f32 check-mode GEMM (CUDA cores, IEEE f32 accumulation).
#pragma once

#include <cuda_runtime.h>

namespace pgb {

// y[T, N] = x[T, K] . w[N, K]^T (+ bias[N]), all f32, row-major, enqueued
// on `stream`. Returns PGB_OK or an error code (message via pgb_last_error).
int launch_gemm_f32(const float* x, const float* w, const float* bias, float* y, int T, int N, int K,
                    cudaStream_t stream);

}  // namespace pgb
