// host_common.cu - last-error handling, device properties, TMA descriptors.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "host_common.h"

namespace pgb {

namespace {
thread_local std::string g_last_error;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
bool g_dev_valid[kMaxDevices] = {};
std::mutex g_dev_mu;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(PGB_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(e),
                   cudaGetErrorString(e));
}

const char* last_error_cstr() { return g_last_error.c_str(); }

bool& pdl_enabled() {
  static bool on = [] {
    const char* v = getenv("PGB_DISABLE_PDL");
    return !(v != nullptr && v[0] == '1');
  }();
  return on;
}

int current_device_info(DeviceInfo* out) {
  int dev = 0;
  PGB_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(PGB_ERR_INVALID, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_dev_valid[dev]) {
    DeviceInfo d{};
    d.device = dev;
    PGB_CUDA_TRY(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
    PGB_CUDA_TRY(
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    PGB_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
    PGB_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
    g_dev[dev] = d;
    g_dev_valid[dev] = true;
  }
  *out = g_dev[dev];
  if (out->cc_major != 10 || out->cc_minor != 0)
    return set_error(PGB_ERR_UNSUPPORTED,
                     "device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev,
                     out->cc_major, out->cc_minor);
  return PGB_OK;
}

int make_tmap_2d_16bit(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                       bool is_bf16) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    g_encode_status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_encode_status == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr)
    return set_error(PGB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0u)
    return set_error(PGB_ERR_INVALID, "tensor base %p is not 16-byte aligned", base);
  if (row_stride_bytes % 16u != 0u)
    return set_error(PGB_ERR_INVALID, "row stride %llu bytes is not a multiple of 16",
                     static_cast<unsigned long long>(row_stride_bytes));
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(PGB_ERR_CUDA,
                     "cuTensorMapEncodeTiled failed (%d) for [%llu x %llu], stride %llu, box %u x %u",
                     static_cast<int>(r), static_cast<unsigned long long>(outer),
                     static_cast<unsigned long long>(inner),
                     static_cast<unsigned long long>(row_stride_bytes), box_outer, box_inner);
  return PGB_OK;
}

}  // namespace pgb
