// Peer mappings for the multi-GPU gather of B's slices.
//
// One process drives one GPU.  A rank exports the device allocation that
// holds its column-blocked slice buffer as a CUDA IPC handle; every peer maps
// it once and then pulls the blocks it needs with copy-engine copies over
// NVLink (cudaMemcpyAsync device to device), so the transfer needs no SMs and
// overlaps the GEMMs of the blocks already present.  There is no counterpart
// in the reference, which has no multi-GPU path.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "oz_common.cuh"

namespace oz {
namespace {

typedef CUresult (*GetRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);

GetRangeFn get_range_fn() {
  static GetRangeFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(ptr);
  }
  return fn;
}

}  // namespace
}  // namespace oz

extern "C" int oz_ipc_export(const void *ptr, void *handle, int64_t *offset) {
  using namespace oz;
  if (!ptr || !handle || !offset) return set_error(OZ_ERR_INVALID, "null argument");
  GetRangeFn range = get_range_fn();
  if (!range) return set_error(OZ_ERR_CUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = range(&base, &size, (CUdeviceptr)(uintptr_t)ptr);
  if (r != CUDA_SUCCESS)
    return set_error(OZ_ERR_INVALID, "pointer is not a device allocation (%d)", (int)r);
  cudaIpcMemHandle_t h;
  if (int rc = check_cuda(cudaIpcGetMemHandle(&h, (void *)(uintptr_t)base), "cudaIpcGetMemHandle"))
    return rc;
  static_assert(sizeof(h) == OZ_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)((uintptr_t)ptr - (uintptr_t)base);
  return OZ_OK;
}

extern "C" int oz_ipc_import(const void *handle, int64_t offset, void **ptr) {
  using namespace oz;
  if (!handle || !ptr || offset < 0) return set_error(OZ_ERR_INVALID, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  if (int rc = check_cuda(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess),
                          "cudaIpcOpenMemHandle"))
    return rc;
  *ptr = static_cast<unsigned char *>(base) + offset;
  return OZ_OK;
}

extern "C" int oz_ipc_close(void *ptr, int64_t offset) {
  using namespace oz;
  if (!ptr || offset < 0) return set_error(OZ_ERR_INVALID, "bad argument");
  return check_cuda(cudaIpcCloseMemHandle(static_cast<unsigned char *>(ptr) - offset),
                    "cudaIpcCloseMemHandle");
}

extern "C" int oz_copy_async(void *dst, const void *src, int64_t bytes, void *stream) {
  using namespace oz;
  if (bytes < 0 || (bytes > 0 && (!dst || !src))) return set_error(OZ_ERR_INVALID, "bad argument");
  if (bytes == 0) return OZ_OK;
  return check_cuda(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault,
                                    reinterpret_cast<cudaStream_t>(stream)),
                    "cudaMemcpyAsync");
}
