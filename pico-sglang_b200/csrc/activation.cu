// activation.cu - silu_and_mul on a materialised [T, 2I] gate_up tensor.
//
// The reference's GatedMLP.forward (python/picosgl/layers/mlp.py:43-48)
// materialises gate_up_proj's output and calls silu_and_mul
// (python/picosgl/layers/activation.py:9-12), which runs flashinfer's
// act_and_mul kernel: per element silu(gate) * up in f32, rounded once to
// the tensor's type. The hot path fuses this into the gate_up GEMM's
// epilogue (pgb_gate_up_silu); this standalone kernel serves callers that
// hold a gate_up tensor already and the f32 check mode.
//
// HBM-bound: every element of the input is read once and every output
// written once, 16 bytes per thread access where the row width allows.
#include "activation.h"
#include "gemm_sm100.cuh"
#include "host_common.h"

namespace pgb {

namespace {
constexpr int kActThreads = 256;

template <typename E, int VEC>
__device__ __forceinline__ void act_piece(const E* g, const E* u, E* o) {
  if constexpr (VEC == 8) {
    *reinterpret_cast<uint4*>(o) =
        silu_mul8<E, false>(__ldg(reinterpret_cast<const uint4*>(g)), __ldg(reinterpret_cast<const uint4*>(u)));
  } else if constexpr (VEC == 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(g));
    const float4 b = __ldg(reinterpret_cast<const float4*>(u));
    *reinterpret_cast<float4*>(o) =
        make_float4(silu_f32(a.x) * b.x, silu_f32(a.y) * b.y, silu_f32(a.z) * b.z, silu_f32(a.w) * b.w);
  } else if constexpr (std::is_same<E, float>::value) {
    *o = silu_f32(*g) * *u;
  } else {
    *o = f32_to_io<E>(silu_f32(io_to_f32<E>(*g)) * io_to_f32<E>(*u));
  }
}

// Grid-stride over the T * I / VEC output pieces of the row-major output.
template <typename E, int VEC>
__global__ void __launch_bounds__(kActThreads) silu_and_mul_kernel(const E* __restrict__ in, E* __restrict__ out,
                                                                   int T, int I) {
  // The next kernel may become resident and prefetch its weights; it reads
  // this kernel's output only after its own wait.
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  const long long per_row = I / VEC;
  const long long total = static_cast<long long>(T) * per_row;
  for (long long i = static_cast<long long>(blockIdx.x) * kActThreads + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * kActThreads) {
    const long long t = i / per_row, v = i - t * per_row;
    const E* g = in + t * 2 * I + v * VEC;
    act_piece<E, VEC>(g, g + I, out + t * I + v * VEC);
  }
}

template <typename E, int VEC>
int launch_act(const void* in, void* out, int T, int I, cudaStream_t stream) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const long long pieces = static_cast<long long>(T) * (I / VEC);
  const long long want = (pieces + kActThreads - 1) / kActThreads;
  const long long cap = static_cast<long long>(dev.sm_count) * 8;  // 8 resident CTAs per SM
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(want < cap ? want : cap));
  cfg.blockDim = dim3(kActThreads);
  cfg.stream = stream;
  return launch_ex(cfg, /*cooperative=*/false, 1, silu_and_mul_kernel<E, VEC>, static_cast<const E*>(in),
                   static_cast<E*>(out), T, I);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u; }
}  // namespace

int launch_silu_and_mul(const void* in, void* out, int T, int I, int dtype, cudaStream_t stream) {
  if (T < 0 || I <= 0) return set_error(PGB_ERR_INVALID, "silu_and_mul: bad shape T=%d I=%d", T, I);
  if (T == 0) return PGB_OK;
  if (in == nullptr || out == nullptr) return set_error(PGB_ERR_INVALID, "silu_and_mul: null pointer argument");
  const bool vec = aligned16(in) && aligned16(out);
  switch (dtype) {
    case PGB_BF16:
      return vec && I % 8 == 0 ? launch_act<__nv_bfloat16, 8>(in, out, T, I, stream)
                               : launch_act<__nv_bfloat16, 1>(in, out, T, I, stream);
    case PGB_F16:
      return vec && I % 8 == 0 ? launch_act<__half, 8>(in, out, T, I, stream)
                               : launch_act<__half, 1>(in, out, T, I, stream);
    case PGB_F32:
      return vec && I % 4 == 0 ? launch_act<float, 4>(in, out, T, I, stream)
                               : launch_act<float, 1>(in, out, T, I, stream);
    default:
      return set_error(PGB_ERR_UNSUPPORTED, "silu_and_mul: dtype %d not supported", dtype);
  }
}

}  // namespace pgb

extern "C" int pgb_silu_and_mul(const void* x, void* out, int T, int I, int dtype, void* stream) {
  return pgb::launch_silu_and_mul(x, out, T, I, dtype, static_cast<cudaStream_t>(stream));
}
