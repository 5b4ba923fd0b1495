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
        cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) !=
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
  int dev, dtype, rank, swizzle;
  uint64_t dims[5], strides[4];
  uint32_t box[5];
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};

}  // namespace

int tensor_map(CUtensorMap* out, CUtensorMapDataType dtype, uint32_t rank, const void* base,
               const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
               CUtensorMapSwizzle swizzle) {
  static std::mutex mu;
  static MapKey keys[64];
  static CUtensorMap maps[64];
  static int used = 0, next = 0;
  if (rank < 1 || rank > 5) return GDN_ERR_SHAPE;
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  if (cudaGetDevice(&key.dev) != cudaSuccess) return GDN_ERR_DEVICE;
  key.base = base;
  key.dtype = static_cast<int>(dtype);
  key.rank = static_cast<int>(rank);
  key.swizzle = static_cast<int>(swizzle);
  for (uint32_t i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) key.strides[i] = strides[i];
  }
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
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  if (fn(&m, dtype, rank, const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
         swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return GDN_ERR_SHAPE;
  const int slot = used < 64 ? used++ : (next++ & 63);
  keys[slot] = key;
  maps[slot] = m;
  *out = m;
  return GDN_OK;
}

int fp32_tensor_map_2d(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols,
                       uint32_t box_rows, uint32_t box_cols) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {cols * 4};
  const uint32_t box[2] = {box_cols, box_rows};
  return tensor_map(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
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
