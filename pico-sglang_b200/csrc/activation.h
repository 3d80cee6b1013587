// activation.h - SiLU-and-multiply on a materialised gate_up tensor.
#pragma once

#include <cuda_runtime.h>

namespace pgb {

// out[T, I] = silu(in[t, 0:I]) * in[t, I:2I] for in [T, 2I] row-major, element
// type dtype (PGB_BF16, PGB_F16 or PGB_F32), enqueued on `stream`. Returns
// PGB_OK or an error code (message via pgb_last_error).
int launch_silu_and_mul(const void* in, void* out, int T, int I, int dtype, cudaStream_t stream);

}  // namespace pgb
