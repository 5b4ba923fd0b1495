// cabi.cu — library-wide C entry points (version, status text) and the
// per-device property cache.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace gdn {

int device_info(DeviceInfo* out) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool filled[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GDN_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (!filled[dev]) {
    DeviceInfo d;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return GDN_ERR_DEVICE;
    cache[dev] = d;
    filled[dev] = true;
  }
  *out = cache[dev];
  // The kernels are built for sm_100a only.
  if (out->cc_major != 10 || out->cc_minor != 0) return GDN_ERR_DEVICE;
  return GDN_OK;
}

}  // namespace gdn

extern "C" int gdn_abi_version(void) { return GDN_B200_ABI_VERSION; }

extern "C" const char* gdn_status_string(int code) {
  switch (code) {
    case GDN_OK: return "ok";
    case GDN_ERR_NULL: return "a required pointer is NULL";
    case GDN_ERR_SHAPE: return "unsupported or inconsistent sizes";
    case GDN_ERR_ALIGN: return "pointer or stride is not 16-byte aligned";
    case GDN_ERR_DTYPE: return "unsupported dtype or gate kind";
    case GDN_ERR_LAUNCH: return "CUDA kernel launch failed";
    case GDN_ERR_DEVICE: return "no CUDA device, or the device is not sm_100";
    case GDN_ERR_WORKSPACE: return "workspace missing or too small";
    case GDN_ERR_DEVICE_WAIT: return "a device-side wait timed out";
    default: return "unknown gdn status code";
  }
}
