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
#include <cstring>
#include <mutex>

#include "zt_common.cuh"

namespace {

constexpr size_t kStaticBytes = zt::plan_prefix_offset(ZT_STATIC_MAX_TENSORS) + sizeof(int64_t) * (ZT_STATIC_MAX_TENSORS + 1);

// Descriptor table + unit prefix of the most recent call on each device. Every GPU that
// loads the library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_static_workspace[kStaticBytes];

// Host image of the array, one per host thread: a call assembles its table and prefix
// here and copies them with one cudaMemcpyAsync. This is ordinary pageable memory, which
// the CUDA runtime copies into its own staging buffer before cudaMemcpyAsync returns, so
// neither this image nor the caller's table (pinned or not) is read after the call.
alignas(256) thread_local unsigned char t_stage[kStaticBytes];

// Device address of g_static_workspace per device. In host code the symbol's name is
// a host-side stand-in, not a device address, so it is resolved with
// cudaGetSymbolAddress once per device, with that device current. The address belongs
// to the device's primary context: after cudaDeviceReset it is stale, and this entry
// point must not be called again in that process.
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
  if (n_tensors > 0 && !host_tensors) return zt::set_error(ZT_ERR_INVALID, "zt_pass_static: null tensor table");
  cudaStream_t s = zt::as_stream(stream);
  // A captured copy would replay from this thread's host image, which later calls
  // overwrite, so the call refuses a capturing stream.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (int rc = zt::check_cuda(cudaStreamIsCapturing(s, &cap), "zt_pass_static: cudaStreamIsCapturing")) return rc;
  if (cap != cudaStreamCaptureStatusNone)
    return zt::set_error(ZT_ERR_INVALID, "zt_pass_static: the stream is capturing; use zt_plan_init + zt_pass in graphs");
  void* ws = nullptr;
  if (int rc = static_workspace(&ws)) return rc;
  // Every check of the table and the pass runs before the shared array is written, so a
  // rejected call leaves the previous call's table in place.
  const size_t off = zt::plan_prefix_offset(n_tensors);
  int64_t* prefix = reinterpret_cast<int64_t*>(t_stage + off);
  zt_plan plan;
  if (int rc = zt::plan_scan(host_tensors, n_tensors, n_params, ws, prefix, &plan)) return rc;
  if (int rc = zt::pass_check(&plan, cfg, streams, n_streams)) return rc;
  // The table is rewritten in full on every call (descriptors and prefix), so nothing
  // in the array has to start at zero; the copy is ordered before the pass on `stream`.
  if (n_tensors > 0) std::memcpy(t_stage, host_tensors, sizeof(zt_tensor) * (size_t)n_tensors);
  const size_t bytes = off + sizeof(int64_t) * ((size_t)n_tensors + 1);
  if (int rc = zt::check_cuda(cudaMemcpyAsync(ws, t_stage, bytes, cudaMemcpyHostToDevice, s), "zt_pass_static: copy table"))
    return rc;
  return zt::pass_launch(&plan, cfg, streams, n_streams, stream);
}

}  // extern "C"
