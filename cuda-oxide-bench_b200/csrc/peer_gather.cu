// peer_gather.cu — all-gather of per-rank decode outputs over NVLink with the
// copy engines (no SMs), for value-head-sharded decode with one process per
// GPU.
//
// Each rank owns a gather buffer G[N][slice] and a flag array F[N] in its own
// HBM and exports both through CUDA IPC.  After its decode step, rank r pushes
// its output slice into every peer's G[r] with cudaMemcpyAsync (a DMA over
// NVLink; the persistent decode kernel keeps every SM) and then writes the
// step number into the peer's F[r] with a stream memory operation, which the
// stream orders after the copy.  A consumer makes its stream wait (on the GPU
// front end, no kernel, no spin on the SMs) until F[p] >= step for every peer.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
typedef CUresult (*WriteValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
typedef CUresult (*WaitValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

struct MemOps {
  WriteValue32Fn write = nullptr;
  WaitValue32Fn wait = nullptr;
  AddressRangeFn range = nullptr;
};

const MemOps& memops() {
  static MemOps m;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      m.write = reinterpret_cast<WriteValue32Fn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuStreamWaitValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      m.wait = reinterpret_cast<WaitValue32Fn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      m.range = reinterpret_cast<AddressRangeFn>(p);
  });
  return m;
}

}  // namespace

// An IPC handle names the whole allocation that contains dev_ptr (a caching
// allocator hands out pieces of larger allocations), and opening it yields
// that allocation's base.  The offset of dev_ptr inside its allocation is
// therefore exported with the handle and added back by gdn_ipc_open.
extern "C" int gdn_ipc_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return GDN_ERR_NULL;
  const MemOps& m = memops();
  if (!m.range) return GDN_ERR_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (m.range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return GDN_ERR_DEVICE;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return GDN_ERR_DEVICE;
  static_assert(sizeof(h) == GDN_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return GDN_OK;
}

extern "C" int gdn_ipc_open(const void* handle, uint64_t offset, void** dev_ptr_out,
                            void** base_out) {
  if (!handle || !dev_ptr_out || !base_out) return GDN_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return GDN_ERR_DEVICE;
  *base_out = base;
  *dev_ptr_out = static_cast<char*>(base) + offset;
  return GDN_OK;
}

extern "C" int gdn_ipc_close(void* base) {
  if (!base) return GDN_ERR_NULL;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? GDN_OK : GDN_ERR_DEVICE;
}

extern "C" int gdn_gather_push(const void* src, size_t bytes, void* const* peer_dst,
                               uint32_t* const* peer_flag, int32_t n_peers, uint32_t value,
                               gdn_stream_t stream) {
  if (!src || !peer_dst || !peer_flag || n_peers < 0) return GDN_ERR_NULL;
  const MemOps& m = memops();
  if (!m.write) return GDN_ERR_DEVICE;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  for (int i = 0; i < n_peers; ++i) {
    if (!peer_dst[i] || !peer_flag[i]) return GDN_ERR_NULL;
    if (cudaMemcpyAsync(peer_dst[i], src, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return GDN_ERR_LAUNCH;
  }
  // the flags follow every copy on this stream, so a peer that sees the new
  // value also sees the data
  for (int i = 0; i < n_peers; ++i)
    if (m.write(reinterpret_cast<CUstream>(s), reinterpret_cast<CUdeviceptr>(peer_flag[i]), value,
                CU_STREAM_WRITE_VALUE_DEFAULT) != CUDA_SUCCESS)
      return GDN_ERR_LAUNCH;
  return GDN_OK;
}

extern "C" int gdn_gather_wait(const uint32_t* flags, int32_t n, uint32_t value,
                               gdn_stream_t stream) {
  if (!flags || n < 0) return GDN_ERR_NULL;
  const MemOps& m = memops();
  if (!m.wait) return GDN_ERR_DEVICE;
  for (int i = 0; i < n; ++i)
    if (m.wait(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flags + i), value,
               CU_STREAM_WAIT_VALUE_GEQ) != CUDA_SUCCESS)
      return GDN_ERR_LAUNCH;
  return GDN_OK;
}

// ------------------------------------------------------------------------
// Consumer side of the fused output all-gather of the decode kernel
// (gdn_peer_out_t): one thread waits, bounded, until an arrival counter that
// peer GPUs increment reaches `target`.  Stream-ordered after this rank's own
// decode, so later work on the stream sees every rank's outputs.
#include "ptx.cuh"

namespace {

__global__ void counter_wait_kernel(const uint32_t* counter, uint32_t target, uint32_t* status) {
  const uint64_t t0 = gdn::global_timer_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
    if (static_cast<int32_t>(v - target) >= 0) return;  // v >= target, modulo 2^32
    if (gdn::global_timer_ns() - t0 > gdn::kWaitLimitNs) {
      gdn::report(status, GDN_DEVERR_PEER_TIMEOUT);
      return;
    }
  }
}

}  // namespace

extern "C" int gdn_gather_wait_counter(const uint32_t* counter, uint32_t target, uint32_t* status,
                                       gdn_stream_t stream) {
  if (!counter) return GDN_ERR_NULL;
  counter_wait_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(counter, target, status);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
