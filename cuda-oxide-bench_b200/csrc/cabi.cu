// cabi.cu — library-wide C entry points (version, status text) and the
// per-device property cache.
#include <cuda_runtime.h>

#include <cstring>
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

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  const void* base;
  uint64_t rows, cols;
  uint32_t box_rows, box_cols;
  int dev;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
           box_cols == o.box_cols && dev == o.dev;
  }
};

}  // namespace

int fp32_tensor_map_2d(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols,
                       uint32_t box_rows, uint32_t box_cols) {
  static std::mutex mu;
  static MapKey keys[32];
  static CUtensorMap maps[32];
  static int used = 0, next = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_DEVICE;
  const MapKey key{base, rows, cols, box_rows, box_cols, dev};
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (keys[i] == key) {
      *out = maps[i];
      return GDN_OK;
    }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return GDN_ERR_DEVICE;
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 4};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return GDN_ERR_SHAPE;
  const int slot = used < 32 ? used++ : (next++ & 31);
  keys[slot] = key;
  maps[slot] = m;
  *out = m;
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
