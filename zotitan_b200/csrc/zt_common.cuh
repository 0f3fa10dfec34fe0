// Internal helpers shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "../../include/zotitan_b200.h"

namespace zt {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
void clear_error();
// Checks a CUDA runtime status; on failure records it with `what` and returns ZT_ERR_CUDA.
int check_cuda(cudaError_t st, const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// SM count of the current device (cached per device).
int sm_count();

// Workspace layout of a plan of n tensors: the descriptor table at offset 0, the
// work-unit prefix (n + 1 int64) at this 256-byte aligned offset.
constexpr size_t plan_prefix_offset(int32_t n_tensors) {
  return (sizeof(zt_tensor) * (size_t)n_tensors + 255) & ~(size_t)255;
}

// Validate a host tensor table and compute its work-unit prefix (n_tensors + 1 entries)
// and the plan's fields, with the table and prefix pointers placed in `workspace`;
// copies nothing.
int plan_scan(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, void* workspace, int64_t* prefix,
              zt_plan* plan);

// plan_scan, then copy the table and prefix into `workspace` and wait for the copies;
// the body of zt_plan_init.
int plan_build(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, void* workspace,
               size_t workspace_bytes, zt_plan* plan, void* stream);

// Every argument check of a pass (plan, configuration, streams, device), without a launch.
int pass_check(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams);

// Validate a pass and launch it; the body of zt_pass.
int pass_launch(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams,
                void* stream);

// pass_check (launch = false) or pass_launch (launch = true).
int pass_run(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams, void* stream,
             bool launch);

// --- parameter-dtype rounding ----------------------------------------------------
template <int DT> struct Dt;
// round2 rounds two values with one paired conversion (the conversion of a single value
// runs on the quarter-rate XU pipe; the paired one handles two at once) and unpacks them
// with integer shifts: the same values as two round() calls.
template <> struct Dt<ZT_F32> {
  __device__ static __forceinline__ float round(float x) { return x; }
  __device__ static __forceinline__ void round2(float&, float&) {}
};
template <> struct Dt<ZT_BF16> {
  __device__ static __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  __device__ static __forceinline__ void round2(float& a, float& b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(&h);
    a = __uint_as_float(w << 16);
    b = __uint_as_float(w & 0xffff0000u);
  }
};
template <> struct Dt<ZT_F16> {
  __device__ static __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
  __device__ static __forceinline__ void round2(float& a, float& b) {
    const float2 f = __half22float2(__floats2half2_rn(a, b));
    a = f.x;
    b = f.y;
  }
};

}  // namespace zt
