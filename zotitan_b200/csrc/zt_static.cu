// zt_pass_static: the fused pass for callers that cannot allocate device memory.
//
// zt_pass needs a caller-allocated workspace for the tensor descriptor table and
// the work-unit prefix. Some callers cannot provide one: processes whose device
// memory is owned by another allocator that has reserved it up front (a serving or
// training runtime that holds nearly all of HBM in its own pool), and host code that
// must not call cudaMalloc/cudaFree while a step is in flight, because those calls
// synchronise the device and fragment the owner's pool. This entry point keeps that
// table in a fixed-size array compiled into the library instead, and allocates
// nothing.
#include <mutex>

#include "zt_common.cuh"

namespace {

constexpr size_t kStaticBytes =
    ((sizeof(zt_tensor) * ZT_STATIC_MAX_TENSORS + 255) & ~(size_t)255) + sizeof(int64_t) * (ZT_STATIC_MAX_TENSORS + 1);

// Descriptor table + unit prefix of the most recent call on each device. Every GPU that
// loads the library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_static_workspace[kStaticBytes];

// Device address of g_static_workspace per device. In host code the symbol's name is
// a host-side stand-in, not a device address, so it is resolved with
// cudaGetSymbolAddress once per device, with that device current.
std::mutex g_mu;
void* g_addr[64] = {nullptr};

int static_workspace(void** out) {
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "zt_pass_static: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return zt::set_error(ZT_ERR_LIMIT, "zt_pass_static: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    if (int rc = zt::check_cuda(cudaGetSymbolAddress(&p, g_static_workspace), "zt_pass_static: cudaGetSymbolAddress"))
      return rc;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return ZT_OK;
}

}  // namespace

extern "C" {

int zt_pass_static(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, const zt_pass_cfg* cfg,
                   const zt_stream* streams, int32_t n_streams, void* stream) {
  zt::clear_error();
  if (n_tensors < 0) return zt::set_error(ZT_ERR_INVALID, "zt_pass_static: n_tensors < 0");
  if (n_tensors > ZT_STATIC_MAX_TENSORS)
    return zt::set_error(ZT_ERR_LIMIT, "zt_pass_static: " + std::to_string(n_tensors) + " tensors > ZT_STATIC_MAX_TENSORS (" +
                                           std::to_string(ZT_STATIC_MAX_TENSORS) + "); use zt_plan_init + zt_pass");
  void* ws = nullptr;
  if (int rc = static_workspace(&ws)) return rc;
  zt_plan plan;
  // The table is rewritten in full on every call (descriptors and prefix), so nothing
  // in the array has to start at zero; the copy is ordered before the pass on `stream`.
  if (int rc = zt::plan_build(host_tensors, n_tensors, n_params, ws, kStaticBytes, &plan, stream, false)) return rc;
  return zt::pass_launch(&plan, cfg, streams, n_streams, stream);
}

}  // extern "C"
