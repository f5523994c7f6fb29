// peer.cu -- CUDA IPC for the pooled-row scatter of the slot-sharded multi-GPU
// path: each rank exports its receive buffers, the other ranks of the node map
// them, and rb_rep_gather_pool_scatter stores pooled rows into them over NVLink.
// Plain loads and stores only: no multicast object is created.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace rb {
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(f);
  });
  return fn;
}
}  // namespace rb

using namespace rb;

static_assert(sizeof(cudaIpcMemHandle_t) == RB_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int rb_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(RB_ERR_VALUE, "rb_ipc_export: null argument");
  AddressRangeFn range = address_range_fn();
  if (range == nullptr) return fail(RB_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(RB_ERR_VALUE, "rb_ipc_export: %p is not device memory (%d)", ptr, (int)r);
  cudaIpcMemHandle_t h;
  const int rc = check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (rc) return rc;
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return RB_OK;
}

extern "C" int rb_ipc_import(const void* handle, int64_t offset, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr || offset < 0) return fail(RB_ERR_VALUE, "rb_ipc_import: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const int rc = check_cuda(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  if (rc) return rc;
  *ptr_out = static_cast<char*>(base) + offset;
  return RB_OK;
}

extern "C" int rb_ipc_close(void* ptr, int64_t offset) {
  if (ptr == nullptr) return fail(RB_ERR_VALUE, "rb_ipc_close: null pointer");
  return check_cuda(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset), "cudaIpcCloseMemHandle");
}
