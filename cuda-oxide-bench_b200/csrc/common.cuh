// common.cuh — host-side helpers shared by the launchers (device properties,
// validation, alignment checks).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/gdn_b200.h"

namespace gdn {

struct DeviceInfo {
  int sm_count = 0;
  int smem_optin = 0;  // max dynamic shared memory per block (opt-in)
  int smem_per_sm = 0; // shared memory per SM
  int cc_major = 0, cc_minor = 0;
};

// Cached per device (filled on first use; the values never change).
int device_info(DeviceInfo* out);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool stride_ok(int64_t elems, int esize) { return ((elems * esize) & 15) == 0; }
inline int host_dtype_size(int dt) { return dt == GDN_DT_F32 ? 4 : 2; }
inline bool dtype_valid(int dt) { return dt == GDN_DT_F32 || dt == GDN_DT_BF16 || dt == GDN_DT_F16; }

// Encodes (or returns a cached) 2-D fp32 tensor map over a row-major matrix
// of `rows` x `cols` with a box of `box_rows` x `box_cols`.  Returns GDN_OK or
// an error code.  The cache is keyed by every argument and guarded by a mutex.
int fp32_tensor_map_2d(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols,
                       uint32_t box_rows, uint32_t box_cols);

// General tiled tensor map (cached likewise); strides are in bytes for
// dimensions 1..rank-1, dims/box innermost first.  No interleave, zero OOB fill.
int tensor_map(CUtensorMap* out, CUtensorMapDataType dtype, uint32_t rank, const void* base,
               const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
               CUtensorMapSwizzle swizzle);

// Raises the kernel's dynamic shared-memory limit once per device.
template <typename Kernel>
int ensure_smem_attr(Kernel k, int bytes, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_DEVICE;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load(std::memory_order_acquire) & bit) return GDN_OK;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return GDN_OK;
}

}  // namespace gdn
