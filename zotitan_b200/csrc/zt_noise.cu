// Raw noise entry points (test and debugging surface of the noise contract).
#include "zt_common.cuh"
#include "zt_philox.cuh"

namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) words_kernel(uint32_t key, const uint32_t* __restrict__ offs,
                                                         int64_t n, uint4* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    uint32_t w[4];
    zt::philox_w4(offs[i], key, w);
    out[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void __launch_bounds__(kThreads) randn_kernel(uint32_t key, int64_t off0, int64_t n,
                                                         float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    out[i] = zt::gauss((uint32_t)(off0 + i), key);
  }
}

__global__ void __launch_bounds__(kThreads) randn_at_kernel(uint32_t key, const uint32_t* __restrict__ offs,
                                                            int64_t n, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    out[i] = zt::gauss(offs[i], key);
  }
}

constexpr int kMaxKeys = 1024;
struct KeysParams {
  uint32_t keys[kMaxKeys];
};

// out[j * n + t] = N(0,1) at offset t for key keys[j]: one launch for many tensors.
__global__ void __launch_bounds__(kThreads) randn_keys_kernel(const __grid_constant__ KeysParams K, int32_t n_keys,
                                                              int64_t n, float* __restrict__ out) {
  const int64_t total = (int64_t)n_keys * n;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < total; i += (int64_t)gridDim.x * kThreads) {
    const int64_t j = i / n;
    out[i] = zt::gauss((uint32_t)(i - j * n), K.keys[j]);
  }
}

int grid_for(int64_t n) {
  const int64_t want = (n + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)zt::sm_count() * 16;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace

extern "C" {

int zt_philox_words(uint32_t key, const uint32_t* offsets, int64_t n, uint32_t* out4, void* stream) {
  zt::clear_error();
  if (n < 0) return zt::set_error(ZT_ERR_INVALID, "zt_philox_words: n < 0");
  if (n == 0) return ZT_OK;
  if (!offsets || !out4) return zt::set_error(ZT_ERR_INVALID, "zt_philox_words: null pointer");
  if (((uintptr_t)out4 & 15) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_philox_words: out4 not 16-byte aligned");
  words_kernel<<<grid_for(n), kThreads, 0, zt::as_stream(stream)>>>(key, offsets, n, reinterpret_cast<uint4*>(out4));
  return zt::check_cuda(cudaGetLastError(), "zt_philox_words launch");
}

int zt_randn(uint32_t key, int64_t off0, int64_t n, float* out, void* stream) {
  zt::clear_error();
  if (n < 0 || off0 < 0) return zt::set_error(ZT_ERR_INVALID, "zt_randn: negative offset or size");
  if (off0 + n > (int64_t)ZT_MAX_NUMEL + 1)
    return zt::set_error(ZT_ERR_LIMIT, "zt_randn: offsets beyond 2^31 (int32 element offsets)");
  if (n == 0) return ZT_OK;
  if (!out) return zt::set_error(ZT_ERR_INVALID, "zt_randn: null output");
  randn_kernel<<<grid_for(n), kThreads, 0, zt::as_stream(stream)>>>(key, off0, n, out);
  return zt::check_cuda(cudaGetLastError(), "zt_randn launch");
}

int zt_randn_keys(const uint32_t* keys, int32_t n_keys, int64_t n, float* out, void* stream) {
  zt::clear_error();
  if (n_keys < 0 || n < 0) return zt::set_error(ZT_ERR_INVALID, "zt_randn_keys: negative size");
  if (n_keys > kMaxKeys) return zt::set_error(ZT_ERR_LIMIT, "zt_randn_keys: more than 1024 keys");
  if (n > (int64_t)ZT_MAX_NUMEL + 1) return zt::set_error(ZT_ERR_LIMIT, "zt_randn_keys: n beyond 2^31");
  if (n_keys == 0 || n == 0) return ZT_OK;
  if (!keys || !out) return zt::set_error(ZT_ERR_INVALID, "zt_randn_keys: null pointer");
  KeysParams K;
  for (int j = 0; j < n_keys; ++j) K.keys[j] = keys[j];
  for (int j = n_keys; j < kMaxKeys; ++j) K.keys[j] = 0;
  randn_keys_kernel<<<grid_for((int64_t)n_keys * n), kThreads, 0, zt::as_stream(stream)>>>(K, n_keys, n, out);
  return zt::check_cuda(cudaGetLastError(), "zt_randn_keys launch");
}

int zt_randn_at(uint32_t key, const uint32_t* offsets, int64_t n, float* out, void* stream) {
  zt::clear_error();
  if (n < 0) return zt::set_error(ZT_ERR_INVALID, "zt_randn_at: n < 0");
  if (n == 0) return ZT_OK;
  if (!offsets || !out) return zt::set_error(ZT_ERR_INVALID, "zt_randn_at: null pointer");
  randn_at_kernel<<<grid_for(n), kThreads, 0, zt::as_stream(stream)>>>(key, offsets, n, out);
  return zt::check_cuda(cudaGetLastError(), "zt_randn_at launch");
}

}  // extern "C"
