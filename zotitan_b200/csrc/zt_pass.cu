// The fused zeroth-order pass: perturb / restore / gradient estimate / optimizer
// update over every trainable tensor in one launch, noise regenerated in registers.
//
// Work decomposition: each tensor is cut into units of ZT_UNIT_ELEMS = 256 threads x
// 8 elements; a persistent grid walks the units, finds the owning tensor by binary
// search over the per-tensor unit prefix, and each thread handles 8 consecutive
// elements with one 16-byte access per buffer (bf16/fp16) or two (fp32).
//
// Arithmetic follows the reference's eager op sequence (zotitan/train_zo.py) with
// the fp32 opmath scalars torch's CUDA kernels use, one rounding to the parameter
// dtype per torch op. Products, quotients and sums whose rounding matters are
// written with __f*_rn intrinsics so the compiler cannot contract them.
#include <vector>

#include "zt_common.cuh"
#include "zt_philox.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kEpt = 8;  // elements per thread per unit
static_assert(kThreads * kEpt == ZT_UNIT_ELEMS, "unit size");

struct KStream {
  uint64_t seed;
  float chain[ZT_MAX_CHAIN];
  float ge_coef;
  float mom_coef;
  uint8_t n_chain;
  uint8_t flags;
  uint8_t pad[2];
};
static_assert(sizeof(KStream) == 32, "KStream layout");

struct PassParams {
  const zt_tensor* tensors;
  const int64_t* unit_prefix;
  int64_t n_units;
  int32_t n_tensors;
  uint32_t n_params;
  zt_pass_cfg cfg;
  int32_t n_streams;
  KStream streams[ZT_MAX_STREAMS];
};

// ---- 8-element loads and stores ------------------------------------------------

template <int DT> struct Io;

template <> struct Io<ZT_F32> {
  __device__ static __forceinline__ void load(const void* base, int64_t e0, int nvalid, bool vec, float v[kEpt]) {
    const float* p = static_cast<const float*>(base) + e0;
    if (vec) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p));
      const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) v[e] = e < nvalid ? p[e] : 0.0f;
    }
  }
  __device__ static __forceinline__ void store(void* base, int64_t e0, int nvalid, bool vec, const float v[kEpt]) {
    float* p = static_cast<float*>(base) + e0;
    if (vec) {
      reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e)
        if (e < nvalid) p[e] = v[e];
    }
  }
};

template <> struct Io<ZT_BF16> {
  __device__ static __forceinline__ void load(const void* base, int64_t e0, int nvalid, bool vec, float v[kEpt]) {
    const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(base) + e0;
    if (vec) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
      }
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) v[e] = e < nvalid ? __bfloat162float(p[e]) : 0.0f;
    }
  }
  __device__ static __forceinline__ void store(void* base, int64_t e0, int nvalid, bool vec, const float v[kEpt]) {
    __nv_bfloat16* p = static_cast<__nv_bfloat16*>(base) + e0;
    if (vec) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e)
        if (e < nvalid) p[e] = __float2bfloat16_rn(v[e]);
    }
  }
};

template <> struct Io<ZT_F16> {
  __device__ static __forceinline__ void load(const void* base, int64_t e0, int nvalid, bool vec, float v[kEpt]) {
    const __half* p = static_cast<const __half*>(base) + e0;
    if (vec) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
        const float2 f = __half22float2(h);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) v[e] = e < nvalid ? __half2float(p[e]) : 0.0f;
    }
  }
  __device__ static __forceinline__ void store(void* base, int64_t e0, int nvalid, bool vec, const float v[kEpt]) {
    __half* p = static_cast<__half*>(base) + e0;
    if (vec) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e)
        if (e < nvalid) p[e] = __float2half_rn(v[e]);
    }
  }
};

// ---- one thread's 8-element group ---------------------------------------------------

template <int DT>
__device__ __forceinline__ void run_group(const PassParams& P, const zt_tensor& t, int64_t e0, int nvalid, bool vec) {
  using R = zt::Dt<DT>;
  using IO = Io<DT>;
  const zt_pass_cfg& c = P.cfg;

  float th[kEpt], ge[kEpt], mom[kEpt];
  IO::load(c.src == ZT_BUF_LIVE ? t.live : t.data, e0, nvalid, vec, th);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) { ge[e] = 0.0f; mom[e] = 0.0f; }

  const uint32_t ctr0 = (uint32_t)e0;
  for (int s = 0; s < P.n_streams; ++s) {
    const KStream& S = P.streams[s];
    const uint32_t key = zt::param_key(S.seed, P.n_params, (uint32_t)t.index);
    float z[kEpt];
#pragma unroll
    for (int e = 0; e < kEpt; ++e) z[e] = zt::gauss(ctr0 + (uint32_t)e, key);
    // _apply_z: theta <- round(theta + a*z), one rounding per call (train_zo.py:350-351)
    for (int k = 0; k < S.n_chain; ++k) {
      const float a = S.chain[k];
#pragma unroll
      for (int e = 0; e < kEpt; ++e) th[e] = R::round(__fmaf_rn(z[e], a, th[e]));
    }
    if (S.flags & ZT_STREAM_GE) {
      const float a = S.ge_coef;
      if (c.ge_mode == ZT_GE_PRODUCT) {
#pragma unroll
        for (int e = 0; e < kEpt; ++e) ge[e] = __fmul_rn(z[e], a);  // fp32 (train_zo.py:552)
      } else {
#pragma unroll
        for (int e = 0; e < kEpt; ++e) ge[e] = R::round(__fmaf_rn(z[e], a, ge[e]));  // (:556, :577)
      }
    }
    if (S.flags & ZT_STREAM_MOM) {
      const float a = S.mom_coef;
#pragma unroll
      for (int e = 0; e < kEpt; ++e) mom[e] = R::round(__fmaf_rn(z[e], a, mom[e]));  // (:345)
    }
  }

  if (c.ge_scale_on) {  // norm clipping rescales grad_est (train_zo.py:457)
    if (c.ge_mode == ZT_GE_PRODUCT) {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) ge[e] = __fmul_rn(ge[e], c.ge_scale);
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) ge[e] = R::round(__fmul_rn(ge[e], c.ge_scale));
    }
  }

  if (c.update) {
    float g[kEpt];
    if (c.momentum == ZT_MOM_STORED_EMA) {  // (:418-419, :330-331)
      float m[kEpt];
      IO::load(t.m, e0, nvalid, vec, m);
#pragma unroll
      for (int e = 0; e < kEpt; ++e) {
        m[e] = R::round(__fmul_rn(m[e], c.beta1));
        m[e] = R::round(__fmaf_rn(ge[e], c.one_minus_beta1, m[e]));
        g[e] = R::round(__fmul_rn(m[e], c.m_scale));
      }
      IO::store(t.m, e0, nvalid, vec, m);
    } else if (c.momentum == ZT_MOM_SEED_WINDOW) {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) g[e] = mom[e];
    } else {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) g[e] = ge[e];
    }
    if (c.second_moment) {  // (:423-425, :392-397)
      float v[kEpt];
      IO::load(t.v, e0, nvalid, vec, v);
      const float nlr = -c.lr;
#pragma unroll
      for (int e = 0; e < kEpt; ++e) {
        v[e] = R::round(__fmul_rn(v[e], c.beta2));
        v[e] = R::round(__fmaf_rn(__fmul_rn(c.one_minus_beta2, ge[e]), ge[e], v[e]));
        float vh = R::round(__fdiv_rn(v[e], c.bc2));
        vh = R::round(__fsqrt_rn(vh));
        vh = R::round(__fadd_rn(vh, c.denom_eps));
        th[e] = R::round(__fadd_rn(th[e], __fdiv_rn(__fmul_rn(nlr, g[e]), vh)));
      }
      IO::store(t.v, e0, nvalid, vec, v);
    } else {
      const float nlr = -c.lr;
#pragma unroll
      for (int e = 0; e < kEpt; ++e) th[e] = R::round(__fmaf_rn(g[e], nlr, th[e]));  // (:399)
    }
    if (c.wd == ZT_WD_STANDARD) {  // (:401-402)
#pragma unroll
      for (int e = 0; e < kEpt; ++e) th[e] = R::round(__fmul_rn(th[e], c.wd_factor));
    } else if (c.wd == ZT_WD_ANCHORED_L2 || c.wd == ZT_WD_ANCHORED_L1) {  // (:403-407)
      float a0[kEpt];
      IO::load(t.anchor, e0, nvalid, vec, a0);
      const float nlam = -c.wd_lam;
      const bool l1 = c.wd == ZT_WD_ANCHORED_L1;
#pragma unroll
      for (int e = 0; e < kEpt; ++e) {
        const float d = R::round(__fsub_rn(th[e], a0[e]));
        const float x = l1 ? (float)((d > 0.0f) - (d < 0.0f)) : d;
        th[e] = R::round(__fmaf_rn(x, nlam, th[e]));
      }
    }
  }

  if (c.dst & ZT_BUF_DATA) IO::store(t.data, e0, nvalid, vec, th);
  if (c.dst & ZT_BUF_LIVE) IO::store(t.live, e0, nvalid, vec, th);
}

__device__ __forceinline__ int find_tensor(const int64_t* __restrict__ prefix, int n, int64_t u) {
  int lo = 0, hi = n;  // prefix[lo] <= u < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(prefix + mid) <= u) lo = mid; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

__global__ void __launch_bounds__(kThreads) pass_kernel(const __grid_constant__ PassParams P) {
  for (int64_t u = blockIdx.x; u < P.n_units; u += gridDim.x) {
    const int ti = find_tensor(P.unit_prefix, P.n_tensors, u);
    const zt_tensor t = P.tensors[ti];
    const int64_t e0 = (u - __ldg(P.unit_prefix + ti)) * ZT_UNIT_ELEMS + (int64_t)threadIdx.x * kEpt;
    if (e0 >= t.numel) continue;
    const int64_t rem = t.numel - e0;
    const int nvalid = rem < kEpt ? (int)rem : kEpt;
    bool vec = nvalid == kEpt && aligned16(t.data);
    const zt_pass_cfg& c = P.cfg;
    if (c.src == ZT_BUF_LIVE || (c.dst & ZT_BUF_LIVE)) vec = vec && aligned16(t.live);
    if (c.update && c.momentum == ZT_MOM_STORED_EMA) vec = vec && aligned16(t.m);
    if (c.update && c.second_moment) vec = vec && aligned16(t.v);
    if (c.update && (c.wd == ZT_WD_ANCHORED_L1 || c.wd == ZT_WD_ANCHORED_L2)) vec = vec && aligned16(t.anchor);
    if (t.dtype == ZT_BF16) run_group<ZT_BF16>(P, t, e0, nvalid, vec);
    else if (t.dtype == ZT_F32) run_group<ZT_F32>(P, t, e0, nvalid, vec);
    else run_group<ZT_F16>(P, t, e0, nvalid, vec);
  }
}

int pass_grid(int64_t n_units) {
  static int occ = 0;
  if (occ == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, pass_kernel, kThreads, 0) != cudaSuccess || n <= 0) n = 1;
    occ = n;
  }
  const int64_t cap = (int64_t)zt::sm_count() * occ;
  return (int)(n_units < cap ? n_units : cap);
}

}  // namespace

extern "C" {

size_t zt_plan_workspace_bytes(int32_t n_tensors) {
  if (n_tensors < 0) return 0;
  const size_t t = sizeof(zt_tensor) * (size_t)n_tensors;
  const size_t tp = (t + 255) & ~(size_t)255;
  return tp + sizeof(int64_t) * ((size_t)n_tensors + 1);
}

int zt_plan_init(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, void* workspace,
                 size_t workspace_bytes, zt_plan* plan, void* stream) {
  zt::clear_error();
  if (!plan || (n_tensors > 0 && (!host_tensors || !workspace)))
    return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: null pointer");
  if (n_tensors < 0) return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: n_tensors < 0");
  if (workspace_bytes < zt_plan_workspace_bytes(n_tensors))
    return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: workspace too small");
  if (((uintptr_t)workspace & 15) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: workspace not 16-byte aligned");
  std::vector<int64_t> prefix((size_t)n_tensors + 1, 0);
  int64_t total = 0;
  int32_t buffers = ZT_HAS_LIVE | ZT_HAS_M | ZT_HAS_V | ZT_HAS_ANCHOR;
  for (int32_t i = 0; i < n_tensors; ++i) {
    const zt_tensor& t = host_tensors[i];
    if (t.numel < 0 || t.numel > (int64_t)ZT_MAX_NUMEL)
      return zt::set_error(ZT_ERR_LIMIT, "zt_plan_init: tensor " + std::to_string(i) +
                                             " numel outside [0, 2^31-1] (int32 element offsets)");
    if (t.numel > 0 && !t.data) return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: tensor " + std::to_string(i) + " has no data");
    if (t.dtype != ZT_F32 && t.dtype != ZT_BF16 && t.dtype != ZT_F16)
      return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: tensor " + std::to_string(i) + " has an unsupported dtype");
    if (t.index < 0 || (uint32_t)t.index >= n_params)
      return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: tensor " + std::to_string(i) + " index outside [0, n_params)");
    if (t.numel > 0) {
      if (!t.live) buffers &= ~ZT_HAS_LIVE;
      if (!t.m) buffers &= ~ZT_HAS_M;
      if (!t.v) buffers &= ~ZT_HAS_V;
      if (!t.anchor) buffers &= ~ZT_HAS_ANCHOR;
    }
    prefix[i + 1] = prefix[i] + (t.numel + ZT_UNIT_ELEMS - 1) / ZT_UNIT_ELEMS;
    total += t.numel;
  }
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "zt_plan_init: cudaGetDevice")) return rc;
  char* ws = static_cast<char*>(workspace);
  const size_t tbytes = sizeof(zt_tensor) * (size_t)n_tensors;
  const size_t off = (tbytes + 255) & ~(size_t)255;
  cudaStream_t s = zt::as_stream(stream);
  if (n_tensors > 0) {
    if (int rc = zt::check_cuda(cudaMemcpyAsync(ws, host_tensors, tbytes, cudaMemcpyHostToDevice, s), "zt_plan_init: copy tensors")) return rc;
  }
  if (int rc = zt::check_cuda(cudaMemcpyAsync(ws + off, prefix.data(), sizeof(int64_t) * prefix.size(),
                                              cudaMemcpyHostToDevice, s), "zt_plan_init: copy prefix")) return rc;
  // The host staging buffers are released when this function returns; make the
  // copies complete first so the caller's arrays and `prefix` may be freed.
  if (int rc = zt::check_cuda(cudaStreamSynchronize(s), "zt_plan_init: synchronize")) return rc;
  plan->tensors = reinterpret_cast<const zt_tensor*>(ws);
  plan->unit_prefix = reinterpret_cast<const int64_t*>(ws + off);
  plan->n_units = prefix[n_tensors];
  plan->numel_total = total;
  plan->n_tensors = n_tensors;
  plan->n_params = n_params;
  plan->device = dev;
  plan->buffers = buffers;
  return ZT_OK;
}

int zt_pass(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams, void* stream) {
  zt::clear_error();
  if (!plan || !cfg) return zt::set_error(ZT_ERR_INVALID, "zt_pass: null plan or cfg");
  if (n_streams < 0 || (n_streams > 0 && !streams)) return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad stream list");
  if (n_streams > ZT_MAX_STREAMS)
    return zt::set_error(ZT_ERR_LIMIT, "zt_pass: more than ZT_MAX_STREAMS (" + std::to_string(ZT_MAX_STREAMS) + ") noise streams");
  if (cfg->src != ZT_BUF_DATA && cfg->src != ZT_BUF_LIVE) return zt::set_error(ZT_ERR_INVALID, "zt_pass: src must be DATA or LIVE");
  if ((cfg->dst & ~(ZT_BUF_DATA | ZT_BUF_LIVE)) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad dst mask");
  if (cfg->ge_mode < ZT_GE_NONE || cfg->ge_mode > ZT_GE_ACCUM) return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad ge_mode");
  if (cfg->momentum < ZT_MOM_NONE || cfg->momentum > ZT_MOM_SEED_WINDOW) return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad momentum");
  if (cfg->wd < ZT_WD_NONE || cfg->wd > ZT_WD_ANCHORED_L1) return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad wd");
  if (!cfg->update && (cfg->momentum != ZT_MOM_NONE || cfg->second_moment || cfg->wd != ZT_WD_NONE))
    return zt::set_error(ZT_ERR_INVALID, "zt_pass: optimizer state and weight decay require update");
  {
    const bool live = cfg->src == ZT_BUF_LIVE || (cfg->dst & ZT_BUF_LIVE);
    const bool anchored = cfg->wd == ZT_WD_ANCHORED_L1 || cfg->wd == ZT_WD_ANCHORED_L2;
    if (live && !(plan->buffers & ZT_HAS_LIVE)) return zt::set_error(ZT_ERR_INVALID, "zt_pass: cfg uses live buffers the plan lacks");
    if (cfg->update && cfg->momentum == ZT_MOM_STORED_EMA && !(plan->buffers & ZT_HAS_M))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: stored-EMA momentum needs m buffers");
    if (cfg->update && cfg->second_moment && !(plan->buffers & ZT_HAS_V))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: second moment needs v buffers");
    if (cfg->update && anchored && !(plan->buffers & ZT_HAS_ANCHOR))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: anchored weight decay needs anchor buffers");
  }
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "zt_pass: cudaGetDevice")) return rc;
  if (dev != plan->device) return zt::set_error(ZT_ERR_INVALID, "zt_pass: plan belongs to another device");
  if (plan->n_units == 0) return ZT_OK;

  PassParams P;
  P.tensors = plan->tensors;
  P.unit_prefix = plan->unit_prefix;
  P.n_units = plan->n_units;
  P.n_tensors = plan->n_tensors;
  P.n_params = plan->n_params;
  P.cfg = *cfg;
  P.n_streams = n_streams;
  for (int s = 0; s < n_streams; ++s) {
    const zt_stream& S = streams[s];
    if (S.n_chain < 0 || S.n_chain > ZT_MAX_CHAIN) return zt::set_error(ZT_ERR_INVALID, "zt_pass: n_chain outside [0, 3]");
    if ((S.flags & ~(ZT_STREAM_GE | ZT_STREAM_MOM)) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad stream flags");
    if ((S.flags & ZT_STREAM_GE) && cfg->ge_mode == ZT_GE_NONE)
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: GE stream with ge_mode NONE");
    if ((S.flags & ZT_STREAM_MOM) && cfg->momentum != ZT_MOM_SEED_WINDOW)
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: MOM stream without seed-window momentum");
    KStream& K = P.streams[s];
    K.seed = S.seed;
    for (int k = 0; k < ZT_MAX_CHAIN; ++k) K.chain[k] = S.chain[k];
    K.ge_coef = S.ge_coef;
    K.mom_coef = S.mom_coef;
    K.n_chain = (uint8_t)S.n_chain;
    K.flags = (uint8_t)S.flags;
    K.pad[0] = K.pad[1] = 0;
  }
  for (int s = n_streams; s < ZT_MAX_STREAMS; ++s) P.streams[s] = KStream{};
  pass_kernel<<<pass_grid(plan->n_units), kThreads, 0, zt::as_stream(stream)>>>(P);
  return zt::check_cuda(cudaGetLastError(), "zt_pass launch");
}

}  // extern "C"
