// Peer mappings and copy-engine copies for the seed-sharded step's field exchange.
//
// In the sharded schedule each rank generates the Gaussian fields of its own pairs over
// every parameter, and every rank needs every pair's field on its own share of the
// parameters for the step's last pass. These entry points let ranks (one process per
// GPU) map each other's field stores and push the slices with cudaMemcpyAsync, which
// runs on the copy engines over NVLink and leaves the SMs to the noise passes.
// Nothing here allocates device memory: the buffers are the caller's (torch's), only
// mapped into this process.
#include <cuda.h>
#include <cstring>

#include "zt_common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) <= ZT_IPC_HANDLE_BYTES, "IPC handle size");

namespace {

// cuMemGetAddressRange through the runtime's driver entry point, so the library keeps
// linking the runtime only.
using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

int address_range(const void* ptr, uintptr_t* base) {
  static GetRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (int rc = zt::check_cuda(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q),
                                "zt_ipc_export: cudaGetDriverEntryPoint"))
      return rc;
    if (q != cudaDriverEntryPointSuccess || !p)
      return zt::set_error(ZT_ERR_CUDA, "zt_ipc_export: cuMemGetAddressRange not found");
    fn = reinterpret_cast<GetRangeFn>(p);
  }
  CUdeviceptr b = 0;
  size_t size = 0;
  if (fn(&b, &size, (CUdeviceptr)(uintptr_t)ptr) != CUDA_SUCCESS)
    return zt::set_error(ZT_ERR_INVALID, "zt_ipc_export: pointer is not in a device allocation");
  *base = (uintptr_t)b;
  return ZT_OK;
}

}  // namespace

extern "C" {

int zt_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  zt::clear_error();
  if (!ptr || !handle_out || !offset_out) return zt::set_error(ZT_ERR_INVALID, "zt_ipc_export: null pointer");
  uintptr_t base = 0;
  if (int rc = address_range(ptr, &base)) return rc;
  cudaIpcMemHandle_t h;
  if (int rc = zt::check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "zt_ipc_export: cudaIpcGetMemHandle"))
    return rc;
  std::memset(handle_out, 0, ZT_IPC_HANDLE_BYTES);
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)((uintptr_t)ptr - base);
  return ZT_OK;
}

int zt_ipc_open(const void* handle, void** base_out) {
  zt::clear_error();
  if (!handle || !base_out) return zt::set_error(ZT_ERR_INVALID, "zt_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (int rc = zt::check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                              "zt_ipc_open: cudaIpcOpenMemHandle"))
    return rc;
  *base_out = p;
  return ZT_OK;
}

int zt_ipc_close(void* base) {
  zt::clear_error();
  if (!base) return zt::set_error(ZT_ERR_INVALID, "zt_ipc_close: null pointer");
  return zt::check_cuda(cudaIpcCloseMemHandle(base), "zt_ipc_close: cudaIpcCloseMemHandle");
}

int zt_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  zt::clear_error();
  if (bytes == 0) return ZT_OK;
  if (!dst || !src) return zt::set_error(ZT_ERR_INVALID, "zt_copy_async: null pointer");
  return zt::check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, zt::as_stream(stream)),
                        "zt_copy_async: cudaMemcpyAsync");
}

}  // extern "C"
