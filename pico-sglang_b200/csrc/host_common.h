// host_common.h - host-side helpers shared by the C-ABI translation units:
// thread-local last-error string, CUDA error mapping, TMA descriptor
// encoding through the driver entry point, and device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/pgb.h"

namespace pgb {

// Record a formatted message as this thread's last error and return code.
int set_error(int code, const char* fmt, ...);
// Map a CUDA runtime error to PGB_ERR_CUDA with a message naming the call site.
int cuda_error(cudaError_t e, const char* what);

#define PGB_CUDA_TRY(expr)                                  \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return ::pgb::cuda_error(_e, #expr); \
  } while (0)

struct DeviceInfo {
  int device;
  int sm_count;
  int max_smem_optin;
  int cc_major, cc_minor;
};
// Cached per-device properties of the current device.
int current_device_info(DeviceInfo* out);

// Encode a 2-D tiled tensor map for a row-major [outer, inner] matrix of
// 16-bit elements with 128-byte swizzle and zero fill out of bounds.
int make_tmap_2d_16bit(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                       bool is_bf16);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Whether launches request programmatic stream serialization (PDL). Cleared
// for the process if the driver refuses a launch with it.
bool& pdl_enabled();

// Launch with cudaLaunchKernelEx: optional cooperative attribute, cluster
// dimension (cluster > 1) and PDL. If the PDL combination is refused,
// retries once without it and keeps it off for the rest of the process.
template <typename Kern, typename... Args>
int launch_ex(cudaLaunchConfig_t cfg, bool cooperative, int cluster, Kern kern, Args... args) {
  cudaLaunchAttribute attr[3];
  int n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (cooperative) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  const bool pdl = pdl_enabled();
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess && pdl) {
    (void)cudaGetLastError();
    pdl_enabled() = false;
    cfg.numAttrs = n - 1;
    e = cudaLaunchKernelEx(&cfg, kern, args...);
  }
  if (e != cudaSuccess) return cuda_error(e, "cudaLaunchKernelEx");
  return PGB_OK;
}

}  // namespace pgb
