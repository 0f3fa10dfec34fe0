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

// Validate a tensor table and copy it (with its work-unit prefix) into `workspace`;
// the body of zt_plan_init. sync_copies: wait for the copies before returning.
int plan_build(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, void* workspace,
               size_t workspace_bytes, zt_plan* plan, void* stream, bool sync_copies);

// Validate a pass and launch it; the body of zt_pass.
int pass_launch(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams,
                void* stream);

// --- parameter-dtype rounding ----------------------------------------------------
template <int DT> struct Dt;
template <> struct Dt<ZT_F32> {
  __device__ static __forceinline__ float round(float x) { return x; }
};
template <> struct Dt<ZT_BF16> {
  __device__ static __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};
template <> struct Dt<ZT_F16> {
  __device__ static __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};

}  // namespace zt
