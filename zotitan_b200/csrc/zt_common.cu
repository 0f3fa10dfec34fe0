// Error reporting, version and small host utilities of the C ABI.
#include <mutex>

#include "zt_common.cuh"
#include "zt_philox.cuh"

namespace zt {

static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

void clear_error() { g_last_error.clear(); }

int check_cuda(cudaError_t st, const char* what) {
  if (st == cudaSuccess) return ZT_OK;
  return set_error(ZT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(st) + " (" +
                                    cudaGetErrorString(st) + ")");
}

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace zt

extern "C" {

const char* zt_last_error(void) { return zt::g_last_error.c_str(); }

int zt_abi_version(void) { return ZT_ABI_VERSION; }

uint32_t zt_param_key(uint64_t seed, uint32_t n_params, uint32_t index) {
  return zt::param_key(seed, n_params, index);
}

}  // extern "C"

// The ctypes mirror (zotitan_b200/_lib.py) and its layout test assume these sizes.
static_assert(sizeof(zt_pass_cfg) == 240 && offsetof(zt_pass_cfg, zcache) == 128 && offsetof(zt_pass_cfg, zfield_stride) == 144 &&
                  offsetof(zt_pass_cfg, zpush) == 152 && offsetof(zt_pass_cfg, zpush_stride) == 232,
              "zt_pass_cfg layout");
static_assert(sizeof(zt_stream) == 40 && sizeof(zt_tensor) == 64, "zt_stream / zt_tensor layout");
static_assert(sizeof(zt_lowrank_desc) == 1104 && offsetof(zt_lowrank_desc, p) == 1056 &&
                  offsetof(zt_lowrank_desc, factors_given) == 1096 &&
                  sizeof(zt_lowrank_apply_args) == 576 && offsetof(zt_lowrank_apply_args, coef) == 44 &&
                  offsetof(zt_lowrank_apply_args, test_wait_cycles) == 568,
              "zt_lowrank_desc / zt_lowrank_apply_args layout");
