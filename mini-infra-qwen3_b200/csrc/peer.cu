// Peer memory of a KV-head partition: CUDA IPC handles of device buffers, so that every rank's
// kernels can store into the other ranks' buffers over NVLink (mi_paged_decode_exchange).
//
// A handle names the whole cudaMalloc allocation that holds the pointer (a caching allocator hands
// out pieces of larger allocations), so it travels with the pointer's offset into that
// allocation; opening it maps the allocation and adds the offset back.  Peer access is enabled
// lazily by the driver.  No device memory is allocated here.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 3020, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

}  // namespace

extern "C" {

int mi_peer_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) == MI_PEER_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle_out || !offset_out) return fail(MI_ERR_INVALID, "mi_peer_handle: null pointer argument");
  auto range = address_range_fn();
  if (!range) return fail(MI_ERR_CUDA, "mi_peer_handle: cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(MI_ERR_INVALID, "mi_peer_handle: not a device allocation (CUresult %d)", (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "mi_peer_handle: cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return MI_OK;
}

int mi_peer_open(const void* handle, int64_t offset, void** ptr_out) {
  if (!handle || !ptr_out || offset < 0) return fail(MI_ERR_INVALID, "mi_peer_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "mi_peer_open: cudaIpcOpenMemHandle");
  *ptr_out = static_cast<char*>(base) + offset;
  return MI_OK;
}

int mi_peer_close(void* ptr, int64_t offset) {
  if (!ptr || offset < 0) return fail(MI_ERR_INVALID, "mi_peer_close: bad argument");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_peer_close: cudaIpcCloseMemHandle");
}

}  // extern "C"
