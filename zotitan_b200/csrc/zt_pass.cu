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
#include <atomic>
#include <vector>

#include "zt_common.cuh"
#include "zt_philox.cuh"

namespace {

#ifndef ZT_CHAIN_EPT
#define ZT_CHAIN_EPT 8  // elements per thread, perturb/restore passes
#endif
#ifndef ZT_CHAIN_MINB
#define ZT_CHAIN_MINB 3  // resident blocks per SM the chain kernel is compiled for
#endif
#ifndef ZT_FULL_EPT
#define ZT_FULL_EPT 8  // elements per thread, passes with gradient / optimizer stages
#endif
#ifndef ZT_FULL_MINB
#define ZT_FULL_MINB 2
#endif
constexpr int kChainEpt = ZT_CHAIN_EPT;
constexpr int kFullEpt = ZT_FULL_EPT;
static_assert(ZT_UNIT_ELEMS % (kChainEpt * 32) == 0 && ZT_UNIT_ELEMS % (kFullEpt * 32) == 0, "unit size");

struct KStream {
  uint64_t seed;
  float chain[ZT_MAX_CHAIN];
  float ge_coef;
  float mom_coef;
  uint8_t n_chain;
  uint8_t flags;
  uint16_t zslot;  // ZT_STREAM_Z_FIELD: slot in cfg.zfield
};
static_assert(sizeof(KStream) == 32, "KStream layout");

struct PassParams {
  const zt_tensor* tensors;
  const int64_t* unit_prefix;
  int64_t unit_begin;  // first unit of this launch
  int64_t n_units;     // one past the last unit of this launch
  int32_t n_tensors;
  uint32_t n_params;
  zt_pass_cfg cfg;
  int32_t n_streams;
  KStream streams[ZT_MAX_STREAMS];
};

// ---- per-thread element group loads and stores ------------------------------------
// A thread owns kEpt consecutive elements; the vector path moves them with one or two
// 8/16-byte accesses per buffer (tensor bases 16-byte aligned, offsets multiples of kEpt).

template <int DT> struct Elem;
template <> struct Elem<ZT_F32> { static constexpr int kBytes = 4; };
template <> struct Elem<ZT_BF16> { static constexpr int kBytes = 2; };
template <> struct Elem<ZT_F16> { static constexpr int kBytes = 2; };

template <int NW>
__device__ __forceinline__ void ld_words(const void* p, uint32_t (&w)[NW]) {
  if constexpr (NW % 4 == 0) {
#pragma unroll
    for (int i = 0; i < NW / 4; ++i) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + i);
      w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
  } else {
    static_assert(NW == 2, "vector width");
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  }
}

template <int NW>
__device__ __forceinline__ void st_words(void* p, const uint32_t (&w)[NW]) {
  if constexpr (NW % 4 == 0) {
#pragma unroll
    for (int i = 0; i < NW / 4; ++i)
      reinterpret_cast<uint4*>(p)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  } else {
    reinterpret_cast<uint2*>(p)[0] = make_uint2(w[0], w[1]);
  }
}

// Noise cache: a thread's EPT consecutive fp32 z values, 16-byte accesses. The cache
// covers whole units, so ragged tails read and write full groups too. z is re-read only
// by a later pass (after a forward in training), so both directions stream past L2.
template <int EPT>
__device__ __forceinline__ void ld_z(const float* p, float (&z)[EPT]) {
  static_assert(EPT % 4 == 0, "16-byte groups");
#pragma unroll
  for (int i = 0; i < EPT / 4; ++i) {
    const float4 v = __ldcs(reinterpret_cast<const float4*>(p) + i);
    z[4 * i] = v.x; z[4 * i + 1] = v.y; z[4 * i + 2] = v.z; z[4 * i + 3] = v.w;
  }
}

template <int EPT>
__device__ __forceinline__ void st_z(float* p, const float (&z)[EPT]) {
  static_assert(EPT % 4 == 0, "16-byte groups");
#pragma unroll
  for (int i = 0; i < EPT / 4; ++i)
    __stcs(reinterpret_cast<float4*>(p) + i, make_float4(z[4 * i], z[4 * i + 1], z[4 * i + 2], z[4 * i + 3]));
}

template <int DT, int EPT> struct Io {
  static constexpr int kNW = EPT * Elem<DT>::kBytes / 4;
  __device__ static __forceinline__ float scalar_ld(const void* base, int64_t i) {
    if constexpr (DT == ZT_F32) return static_cast<const float*>(base)[i];
    else if constexpr (DT == ZT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
    else return __half2float(static_cast<const __half*>(base)[i]);
  }
  __device__ static __forceinline__ void scalar_st(void* base, int64_t i, float v) {
    if constexpr (DT == ZT_F32) static_cast<float*>(base)[i] = v;
    else if constexpr (DT == ZT_BF16) static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
    else static_cast<__half*>(base)[i] = __float2half_rn(v);
  }
  __device__ static __forceinline__ void load(const void* base, int64_t e0, int nvalid, bool vec, float (&v)[EPT]) {
    if (vec) {
      uint32_t w[kNW];
      ld_words<kNW>(static_cast<const char*>(base) + e0 * Elem<DT>::kBytes, w);
#pragma unroll
      for (int k = 0; k < kNW; ++k) {
        if constexpr (DT == ZT_F32) {
          v[k] = __uint_as_float(w[k]);
        } else if constexpr (DT == ZT_BF16) {
          v[2 * k] = __uint_as_float(w[k] << 16);
          v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
          v[2 * k] = f.x;
          v[2 * k + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < EPT; ++e) v[e] = e < nvalid ? scalar_ld(base, e0 + e) : 0.0f;
    }
  }
  __device__ static __forceinline__ void store(void* base, int64_t e0, int nvalid, bool vec, const float (&v)[EPT]) {
    if (vec) {
      uint32_t w[kNW];
#pragma unroll
      for (int k = 0; k < kNW; ++k) {
        if constexpr (DT == ZT_F32) {
          w[k] = __float_as_uint(v[k]);
        } else if constexpr (DT == ZT_BF16) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
          w[k] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
          const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
          w[k] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      st_words<kNW>(static_cast<char*>(base) + e0 * Elem<DT>::kBytes, w);
    } else {
#pragma unroll
      for (int e = 0; e < EPT; ++e)
        if (e < nvalid) scalar_st(base, e0 + e, v[e]);
    }
  }
};

// ---- one thread's element group -------------------------------------------------

// out[e] = round(f(e)) for e < EPT, two elements per paired conversion (Dt::round2).
template <int DT, int EPT, class F>
__device__ __forceinline__ void round_each(float (&out)[EPT], F f) {
  static_assert(EPT % 2 == 0, "pairs");
#pragma unroll
  for (int e = 0; e < EPT; e += 2) {
    float a = f(e), b = f(e + 1);
    zt::Dt<DT>::round2(a, b);
    out[e] = a;
    out[e + 1] = b;
  }
}

// Perturb / restore passes: theta <- round(theta + a*z) for each chained coefficient of
// each stream (train_zo.py:350-351), nothing else.
// Field-store slot of stream S for this thread's group: zf_off = (u - unit_begin) *
// ZT_UNIT_ELEMS + the group's offset inside the unit.
__device__ __forceinline__ const float* zfield_at(const PassParams& P, const KStream& S, int64_t zf_off) {
  return P.cfg.zfield + (int64_t)S.zslot * P.cfg.zfield_stride + zf_off;
}

template <int DT, int EPT>
__device__ __forceinline__ void run_chain(const PassParams& P, const zt_tensor& t, int64_t e0, int nvalid, bool vec,
                                          float* zc, int64_t zf_off) {
  using R = zt::Dt<DT>;
  using IO = Io<DT, EPT>;
  const zt_pass_cfg& c = P.cfg;
  float th[EPT];
  IO::load(c.src == ZT_BUF_LIVE ? t.live : t.data, e0, nvalid, vec, th);
  const uint32_t ctr0 = (uint32_t)e0;
  for (int s = 0; s < P.n_streams; ++s) {
    const KStream& S = P.streams[s];
    if (S.flags & (ZT_STREAM_Z_LOAD | ZT_STREAM_Z_STORE | ZT_STREAM_Z_FIELD)) {  // z held as an array
      float z[EPT];
      if (S.flags & ZT_STREAM_Z_LOAD) {
        ld_z<EPT>(zc, z);
      } else if (S.flags & ZT_STREAM_Z_FIELD) {
        ld_z<EPT>(zfield_at(P, S, zf_off), z);
      } else {
        const zt::RoundKeys rk = zt::round_keys(zt::param_key(S.seed, P.n_params, (uint32_t)t.index));
#pragma unroll
        for (int e = 0; e < EPT; ++e) z[e] = zt::gauss_rk(ctr0 + (uint32_t)e, rk);
        st_z<EPT>(zc, z);
      }
      for (int k = 0; k < S.n_chain; ++k) {
        const float a = S.chain[k];
        round_each<DT>(th, [&](int e) { return __fmaf_rn(z[e], a, th[e]); });
      }
      continue;
    }
    const zt::RoundKeys rk = zt::round_keys(zt::param_key(S.seed, P.n_params, (uint32_t)t.index));
    const float a0 = S.chain[0], a1 = S.chain[1], a2 = S.chain[2];
    if (S.n_chain > 0) {  // the chain length is uniform: branch once, not per element
      float z[EPT];
#pragma unroll
      for (int e = 0; e < EPT; ++e) z[e] = zt::gauss_rk(ctr0 + (uint32_t)e, rk);
      round_each<DT>(th, [&](int e) { return __fmaf_rn(z[e], a0, th[e]); });
      if (S.n_chain > 1) round_each<DT>(th, [&](int e) { return __fmaf_rn(z[e], a1, th[e]); });
      if (S.n_chain > 2) round_each<DT>(th, [&](int e) { return __fmaf_rn(z[e], a2, th[e]); });
    }
  }
  if (c.dst & ZT_BUF_DATA) IO::store(t.data, e0, nvalid, vec, th);
  if (c.dst & ZT_BUF_LIVE) IO::store(t.live, e0, nvalid, vec, th);
}

template <int DT, int EPT>
__device__ __forceinline__ void run_full(const PassParams& P, const zt_tensor& t, int64_t e0, int nvalid, bool vec,
                                         float dev_coef, float* zc, int64_t zf_off) {
  using R = zt::Dt<DT>;
  using IO = Io<DT, EPT>;
  const zt_pass_cfg& c = P.cfg;

  float th[EPT], ge[EPT], mom[EPT];
  IO::load(c.src == ZT_BUF_LIVE ? t.live : t.data, e0, nvalid, vec, th);
  if (c.ge_load) {
    IO::load(t.ge, e0, nvalid, vec, ge);
  } else {
#pragma unroll
    for (int e = 0; e < EPT; ++e) ge[e] = 0.0f;
  }
#pragma unroll
  for (int e = 0; e < EPT; ++e) mom[e] = 0.0f;

  const uint32_t ctr0 = (uint32_t)e0;
  for (int s = 0; s < P.n_streams; ++s) {
    const KStream& S = P.streams[s];
    float z[EPT];
    if (S.flags & ZT_STREAM_Z_LOAD) {
      ld_z<EPT>(zc, z);
    } else if (S.flags & ZT_STREAM_Z_FIELD) {
      ld_z<EPT>(zfield_at(P, S, zf_off), z);
    } else {
      const zt::RoundKeys rk = zt::round_keys(zt::param_key(S.seed, P.n_params, (uint32_t)t.index));
#pragma unroll
      for (int e = 0; e < EPT; ++e) z[e] = zt::gauss_rk(ctr0 + (uint32_t)e, rk);
      if (S.flags & ZT_STREAM_Z_STORE) st_z<EPT>(zc, z);
    }
    // _apply_z: theta <- round(theta + a*z), one rounding per call (train_zo.py:350-351)
    for (int k = 0; k < S.n_chain; ++k) {
      const float a = S.chain[k];
      round_each<DT>(th, [&](int e) { return __fmaf_rn(z[e], a, th[e]); });
    }
    if (S.flags & ZT_STREAM_GE) {
      const float a = (S.flags & ZT_STREAM_GE_DEV) ? dev_coef : S.ge_coef;
      if (c.ge_mode == ZT_GE_PRODUCT) {
#pragma unroll
        for (int e = 0; e < EPT; ++e) ge[e] = __fmul_rn(z[e], a);  // fp32 (train_zo.py:552)
      } else {
        round_each<DT>(ge, [&](int e) { return __fmaf_rn(z[e], a, ge[e]); });  // (:556, :577)
      }
    }
    if (S.flags & ZT_STREAM_MOM) {
      const float a = S.mom_coef;
      round_each<DT>(mom, [&](int e) { return __fmaf_rn(z[e], a, mom[e]); });  // (:345)
    }
  }

  if (c.ge_scale_on) {  // norm clipping rescales grad_est (train_zo.py:457)
    if (c.ge_mode == ZT_GE_PRODUCT) {
#pragma unroll
      for (int e = 0; e < EPT; ++e) ge[e] = __fmul_rn(ge[e], c.ge_scale);
    } else {
#pragma unroll
      for (int e = 0; e < EPT; ++e) ge[e] = R::round(__fmul_rn(ge[e], c.ge_scale));
    }
  }

  if (c.ge_store) IO::store(t.ge, e0, nvalid, vec, ge);

  if (c.update) {
    float g[EPT];
    if (c.momentum == ZT_MOM_STORED_EMA) {  // (:418-419, :330-331)
      float m[EPT];
      IO::load(t.m, e0, nvalid, vec, m);
#pragma unroll
      for (int e = 0; e < EPT; ++e) {
        m[e] = R::round(__fmul_rn(m[e], c.beta1));
        m[e] = R::round(__fmaf_rn(ge[e], c.one_minus_beta1, m[e]));
        g[e] = R::round(__fmul_rn(m[e], c.m_scale));
      }
      IO::store(t.m, e0, nvalid, vec, m);
    } else if (c.momentum == ZT_MOM_SEED_WINDOW) {
#pragma unroll
      for (int e = 0; e < EPT; ++e) g[e] = mom[e];
    } else {
#pragma unroll
      for (int e = 0; e < EPT; ++e) g[e] = ge[e];
    }
    if (c.second_moment) {  // (:423-425, :392-397)
      float v[EPT];
      IO::load(t.v, e0, nvalid, vec, v);
      const float nlr = -c.lr;
#pragma unroll
      for (int e = 0; e < EPT; ++e) {
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
      for (int e = 0; e < EPT; ++e) th[e] = R::round(__fmaf_rn(g[e], nlr, th[e]));  // (:399)
    }
    if (c.wd == ZT_WD_STANDARD) {  // (:401-402)
#pragma unroll
      for (int e = 0; e < EPT; ++e) th[e] = R::round(__fmul_rn(th[e], c.wd_factor));
    } else if (c.wd == ZT_WD_ANCHORED_L2 || c.wd == ZT_WD_ANCHORED_L1) {  // (:403-407)
      float a0[EPT];
      IO::load(t.anchor, e0, nvalid, vec, a0);
      const float nlam = -c.wd_lam;
      const bool l1 = c.wd == ZT_WD_ANCHORED_L1;
#pragma unroll
      for (int e = 0; e < EPT; ++e) {
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

// Persistent grid over work units. The owning tensor is looked up only when a unit
// leaves the current tensor's unit range (grid-stride steps rarely do).
template <bool kFull, int EPT>
__device__ __forceinline__ void walk_units(const PassParams& P) {
  constexpr int kThreadsT = ZT_UNIT_ELEMS / EPT;
  const zt_pass_cfg& c = P.cfg;
  int64_t lo = 0, hi = -1;  // unit range of the cached tensor
  zt_tensor t{};
  bool base_vec = false;
  // Coefficient of a ZT_STREAM_GE_DEV stream: the reference's (v+ - v-)/(2 eps), clamp
  // and /z_batch in fp32 (train_zo.py:544-556), from the two device values. A NaN value
  // propagates through the comparisons unchanged, as torch.clamp does.
  float dev_coef = 0.0f;
  if (kFull && c.dev_vals) {
    const float d = __fsub_rn(__ldg(c.dev_vals), __ldg(c.dev_vals + 1));
    float pg = __fmul_rn(d, c.dev_inv2eps);
    pg = pg < -c.dev_tau ? -c.dev_tau : (pg > c.dev_tau ? c.dev_tau : pg);
    dev_coef = __fmul_rn(pg, c.dev_invz);
  }
  for (int64_t u = P.unit_begin + blockIdx.x; u < P.n_units; u += gridDim.x) {
    if (u < lo || u >= hi) {
      const int ti = find_tensor(P.unit_prefix, P.n_tensors, u);
      lo = __ldg(P.unit_prefix + ti);
      hi = __ldg(P.unit_prefix + ti + 1);
      t = P.tensors[ti];
      base_vec = aligned16(t.data);
      if (c.src == ZT_BUF_LIVE || (c.dst & ZT_BUF_LIVE)) base_vec = base_vec && aligned16(t.live);
      if (kFull && c.update && c.momentum == ZT_MOM_STORED_EMA) base_vec = base_vec && aligned16(t.m);
      if (kFull && c.update && c.second_moment) base_vec = base_vec && aligned16(t.v);
      if (kFull && c.update && (c.wd == ZT_WD_ANCHORED_L1 || c.wd == ZT_WD_ANCHORED_L2))
        base_vec = base_vec && aligned16(t.anchor);
      if (kFull && (c.ge_load || c.ge_store)) base_vec = base_vec && aligned16(t.ge);
    }
    const int64_t e0 = (u - lo) * ZT_UNIT_ELEMS + (int64_t)(threadIdx.x % kThreadsT) * EPT;
    if (e0 >= t.numel) continue;
    const int64_t rem = t.numel - e0;
    const int nvalid = rem < EPT ? (int)rem : EPT;
    const bool vec = base_vec && nvalid == EPT;
    // this thread's slot of the noise cache (unit u, same offset inside the unit as e0)
    float* zc = c.zcache ? c.zcache + u * ZT_UNIT_ELEMS + (int64_t)(threadIdx.x % kThreadsT) * EPT : nullptr;
    // and of the field store (units counted from the pass's first unit)
    const int64_t zf = (u - P.unit_begin) * ZT_UNIT_ELEMS + (int64_t)(threadIdx.x % kThreadsT) * EPT;
    if (kFull) {
      if (t.dtype == ZT_BF16) run_full<ZT_BF16, EPT>(P, t, e0, nvalid, vec, dev_coef, zc, zf);
      else if (t.dtype == ZT_F32) run_full<ZT_F32, EPT>(P, t, e0, nvalid, vec, dev_coef, zc, zf);
      else run_full<ZT_F16, EPT>(P, t, e0, nvalid, vec, dev_coef, zc, zf);
    } else {
      if (t.dtype == ZT_BF16) run_chain<ZT_BF16, EPT>(P, t, e0, nvalid, vec, zc, zf);
      else if (t.dtype == ZT_F32) run_chain<ZT_F32, EPT>(P, t, e0, nvalid, vec, zc, zf);
      else run_chain<ZT_F16, EPT>(P, t, e0, nvalid, vec, zc, zf);
    }
  }
}

__global__ void __launch_bounds__(ZT_UNIT_ELEMS / kChainEpt, ZT_CHAIN_MINB)
chain_kernel(const __grid_constant__ PassParams P) {
  walk_units<false, kChainEpt>(P);
}

__global__ void __launch_bounds__(ZT_UNIT_ELEMS / kFullEpt, ZT_FULL_MINB)
full_kernel(const __grid_constant__ PassParams P) {
  walk_units<true, kFullEpt>(P);
}

// ---- kernels specialised for the pass shapes that dominate a step -------------------
// For plans whose tensors share one dtype and whose 8-element groups are all whole and
// 16-byte aligned (ZT_PLAN_VEC8), these shapes run without the per-unit dtype dispatch,
// the scalar fallback and the stream loop of the generic kernels. That keeps the
// register footprint low enough for more resident warps. Arithmetic and its order are
// those of run_chain / run_full, so the results are identical.
enum FastShape : int {
  kFastChain1 = 0,  // one stream, one coefficient, no roles (the +eps and -2eps passes)
  kFastChain2 = 1,  // two such streams (restore one pair, perturb the next)
  kFastAccum = 2,   // stream 0: +a z and its grad_est term (ACCUM, stored); stream 1: +a z
  kFastReplay = 3,  // any number of streams, each its chain and grad_est term (ACCUM, host
                    // coefficient, in registers; grad_est starting from the ge buffers with
                    // ge_load), then the SGD update (+ standard decay): the last pass of a
                    // step, and the sharded replay of every pair
  kFastShapes = 4,
};

// Noise-cache variants of the specialised shapes (ZT_STREAM_Z_LOAD / _STORE): stream 0
// reads its field from the cache, and/or the last stream writes its field to it.
enum FastZ : int {
  kZNone = 0,
  kZLoad = 1,       // stream 0 loads
  kZStore = 2,      // the last stream (stream 0 of kFastChain1, stream 1 otherwise) stores
  kZLoadStore = 3,  // stream 0 loads, stream 1 stores (in place: load first)
  kZPush = 4,       // with kZStore (kFastChain1): the stored field also goes to the owners' stores
};

constexpr int32_t kZFlags = ZT_STREAM_Z_LOAD | ZT_STREAM_Z_STORE;
constexpr int32_t kZSrc = ZT_STREAM_Z_LOAD | ZT_STREAM_Z_FIELD;  // where a stream's z may come from

#ifndef ZT_EARLY_GEN
#define ZT_EARLY_GEN 1  // generate the next pair's field before applying the cached one
#endif
#ifndef ZT_EARLY_GEN0
#define ZT_EARLY_GEN0 1  // generate a regenerated stream-0 field before unpacking theta
#endif
#ifndef ZT_FAST_CHAIN_MINB
#define ZT_FAST_CHAIN_MINB 5
#endif
#ifndef ZT_FAST_ACCUM_MINB
#define ZT_FAST_ACCUM_MINB 4
#endif
#ifndef ZT_FAST_REPLAY_MINB
#define ZT_FAST_REPLAY_MINB 4
#endif

// 8 elements as 32-bit storage words: two per word for 16-bit formats, one for fp32.
template <int DT> struct Words {
  static constexpr int kBytes = Elem<DT>::kBytes;
  static constexpr int kPer = 4 / kBytes;
  static constexpr int kNW = 8 / kPer;
  __device__ static __forceinline__ void unpack(uint32_t w, float (&v)[kPer]) {
    if constexpr (DT == ZT_F32) {
      v[0] = __uint_as_float(w);
    } else if constexpr (DT == ZT_BF16) {
      v[0] = __uint_as_float(w << 16);
      v[1] = __uint_as_float(w & 0xffff0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
      v[0] = f.x;
      v[1] = f.y;
    }
  }
  __device__ static __forceinline__ uint32_t pack(const float (&v)[kPer]) {
    if constexpr (DT == ZT_F32) {
      return __float_as_uint(v[0]);
    } else if constexpr (DT == ZT_BF16) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[0], v[1]);
      return *reinterpret_cast<const uint32_t*>(&h);
    } else {
      const __half2 h = __floats2half2_rn(v[0], v[1]);
      return *reinterpret_cast<const uint32_t*>(&h);
    }
  }
};

// Per-tensor state of the unit being processed. It is block-uniform and kept in shared
// memory, so it holds no registers across the noise loop. Unit and element indices are
// 32-bit: the host takes this path only when the plan has fewer than 2^31 units, and a
// tensor has fewer than 2^31 elements.
struct FastTensor {
  const char* src;
  char* data;
  char* live;
  char* ge;
  uint32_t numel;
  int32_t lo, hi;
  uint32_t key0, key1;
  uint32_t index;
};

__device__ __forceinline__ void st_global16(char* p, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  __stwb(reinterpret_cast<uint4*>(p), make_uint4(x, y, z, w));
}

template <int NW>
__device__ __forceinline__ void st_words_global(char* p, const uint32_t (&w)[NW]) {
  static_assert(NW % 4 == 0, "16-byte groups");
#pragma unroll
  for (int i = 0; i < NW / 4; ++i) st_global16(p + 16 * i, w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

template <int DT, int SHAPE, int ZM>
__device__ __forceinline__ void fast_walk(const PassParams& P) {
  static_assert(ZM == kZNone || SHAPE != kFastReplay, "the replay shape handles its cache loads per stream");
  static_assert(ZM != kZLoadStore || SHAPE != kFastChain1, "one stream cannot both load and store");
  using W = Words<DT>;
  const zt_pass_cfg& c = P.cfg;
  const KStream& S0 = P.streams[0];
  const KStream& S1 = P.streams[1];
  const float a0 = S0.chain[0];
  const float a1 = S1.chain[0];
  float gcoef = 0.0f;
  if (SHAPE == kFastAccum) {
    gcoef = S0.ge_coef;
    if (S0.flags & ZT_STREAM_GE_DEV) {  // as walk_units: (v+ - v-) / (2 eps), clamp, / z_batch
      const float d = __fsub_rn(__ldg(c.dev_vals), __ldg(c.dev_vals + 1));
      float pg = __fmul_rn(d, c.dev_inv2eps);
      pg = pg < -c.dev_tau ? -c.dev_tau : (pg > c.dev_tau ? c.dev_tau : pg);
      gcoef = __fmul_rn(pg, c.dev_invz);
    }
  }
  __shared__ FastTensor st;
  const int32_t n_units = (int32_t)P.n_units;
  int32_t lo = 0, hi = -1;
  for (int32_t u = (int32_t)P.unit_begin + (int32_t)blockIdx.x; u < n_units; u += (int32_t)gridDim.x) {
    if (u < lo || u >= hi) {  // u, lo and hi are block-uniform
      __syncthreads();  // every thread is done with the previous tensor's state
      if (threadIdx.x == 0) {
        const int ti = find_tensor(P.unit_prefix, P.n_tensors, u);
        const zt_tensor& t = P.tensors[ti];
        st.lo = (int32_t)__ldg(P.unit_prefix + ti);
        st.hi = (int32_t)__ldg(P.unit_prefix + ti + 1);
        st.numel = (uint32_t)t.numel;
        st.src = static_cast<const char*>(c.src == ZT_BUF_LIVE ? t.live : t.data);
        st.data = static_cast<char*>(t.data);
        st.live = static_cast<char*>(t.live);
        st.ge = static_cast<char*>(t.ge);
        st.key0 = zt::param_key(S0.seed, P.n_params, (uint32_t)t.index);
        st.key1 = SHAPE != kFastChain1 ? zt::param_key(S1.seed, P.n_params, (uint32_t)t.index) : 0u;
        st.index = (uint32_t)t.index;
      }
      __syncthreads();
      lo = st.lo;
      hi = st.hi;
    }
    const uint32_t e0 = (uint32_t)(u - lo) * ZT_UNIT_ELEMS + threadIdx.x * 8u;
    if (e0 >= st.numel) continue;
    const size_t off = (size_t)e0 * W::kBytes;
    if constexpr (SHAPE == kFastReplay) {
      using R = zt::Dt<DT>;
      uint32_t w[W::kNW];
      ld_words<W::kNW>(st.src + off, w);
      float th[8], ge[8];
#pragma unroll
      for (int k = 0; k < W::kNW; ++k) {
        float t[W::kPer];
        W::unpack(w[k], t);
#pragma unroll
        for (int i = 0; i < W::kPer; ++i) th[k * W::kPer + i] = t[i];
      }
      if (c.ge_load) {  // grad_est accumulated by earlier passes (the on-the-fly schedule)
        uint32_t gw[W::kNW];
        ld_words<W::kNW>(st.ge + off, gw);
#pragma unroll
        for (int k = 0; k < W::kNW; ++k) {
          float t[W::kPer];
          W::unpack(gw[k], t);
#pragma unroll
          for (int i = 0; i < W::kPer; ++i) ge[k * W::kPer + i] = t[i];
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) ge[e] = 0.0f;
      }
      // Fields read from memory are requested one stream ahead, so a load is in flight
      // while the previous stream's chain (or its noise regeneration) runs.
      float zn[8];
      auto prefetch = [&](int s2) {
        if (s2 < P.n_streams && (P.streams[s2].flags & kZSrc)) {
          const KStream& T = P.streams[s2];
          const float* zp = (T.flags & ZT_STREAM_Z_LOAD)
                                ? c.zcache + (size_t)u * ZT_UNIT_ELEMS + threadIdx.x * 8u
                                : c.zfield + (size_t)T.zslot * (size_t)c.zfield_stride +
                                      (size_t)(u - (int32_t)P.unit_begin) * ZT_UNIT_ELEMS + threadIdx.x * 8u;
          ld_z<8>(zp, zn);
        }
      };
      prefetch(0);
      for (int s = 0; s < P.n_streams; ++s) {
        const KStream& S = P.streams[s];
        const float c0 = S.chain[0], c1 = S.chain[1], c2 = S.chain[2], gc = S.ge_coef;
        const int nc = S.n_chain;  // uniform: the branches below are taken by every thread
        // elements e and e+1 together: each rounding is one paired conversion (round2)
        auto apply2 = [&](int e, float za, float zb) {
          float xa = th[e], xb = th[e + 1];
          if (nc > 0) { xa = __fmaf_rn(za, c0, xa); xb = __fmaf_rn(zb, c0, xb); R::round2(xa, xb); }
          if (nc > 1) { xa = __fmaf_rn(za, c1, xa); xb = __fmaf_rn(zb, c1, xb); R::round2(xa, xb); }
          if (nc > 2) { xa = __fmaf_rn(za, c2, xa); xb = __fmaf_rn(zb, c2, xb); R::round2(xa, xb); }
          th[e] = xa;
          th[e + 1] = xb;
          float ga = __fmaf_rn(za, gc, ge[e]), gb = __fmaf_rn(zb, gc, ge[e + 1]);  // (train_zo.py:556)
          R::round2(ga, gb);
          ge[e] = ga;
          ge[e + 1] = gb;
        };
        if (S.flags & kZSrc) {
          // a field this rank cached (its last own pair) or one pushed into its field store,
          // loaded while the previous stream ran; the next such field is requested now
          float zl[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) zl[e] = zn[e];
          prefetch(s + 1);
#pragma unroll
          for (int e = 0; e < 8; e += 2) apply2(e, zl[e], zl[e + 1]);
        } else {
          prefetch(s + 1);
          const zt::RoundKeys rk = zt::round_keys(zt::param_key(S.seed, P.n_params, st.index));
#pragma unroll
          for (int e = 0; e < 8; e += 2)
            apply2(e, zt::gauss_rk(e0 + (uint32_t)e, rk), zt::gauss_rk(e0 + (uint32_t)e + 1u, rk));
        }
      }
      const float nlr = -c.lr;
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float xa = __fmaf_rn(ge[e], nlr, th[e]), xb = __fmaf_rn(ge[e + 1], nlr, th[e + 1]);  // (:399)
        R::round2(xa, xb);
        if (c.wd == ZT_WD_STANDARD) {  // (:401-402)
          xa = __fmul_rn(xa, c.wd_factor);
          xb = __fmul_rn(xb, c.wd_factor);
          R::round2(xa, xb);
        }
        th[e] = xa;
        th[e + 1] = xb;
      }
#pragma unroll
      for (int k = 0; k < W::kNW; ++k) {
        float t[W::kPer];
#pragma unroll
        for (int i = 0; i < W::kPer; ++i) t[i] = th[k * W::kPer + i];
        w[k] = W::pack(t);
      }
      if (c.dst & ZT_BUF_DATA) st_words_global<W::kNW>(st.data + off, w);
      if (c.dst & ZT_BUF_LIVE) st_words_global<W::kNW>(st.live + off, w);
      continue;
    }
    // Values stay packed in their storage format between noise streams: packing with
    // round-to-nearest is the rounding to the parameter dtype after each step.
    uint32_t w[W::kNW], gw[W::kNW];
    ld_words<W::kNW>(st.src + off, w);
    // noise-cache slot of this thread: unit u, the same 8-element group as e0
    float* zc = ZM != kZNone ? c.zcache + (size_t)u * ZT_UNIT_ELEMS + threadIdx.x * 8u : nullptr;
    float zl[8], zs[8];
    if constexpr ((ZM & kZLoad) != 0) ld_z<8>(zc, zl);
    if (SHAPE == kFastAccum) {
      if (c.ge_load) {
        ld_words<W::kNW>(st.ge + off, gw);
      } else {
#pragma unroll
        for (int k = 0; k < W::kNW; ++k) gw[k] = 0u;  // +0.0 in every format
      }
    }
    // When stream 0 reads its field from the cache, stream 1's field is generated first:
    // it needs none of the loaded values, so the loads land while the noise is computed
    // (applying the streams stays in their order).
    constexpr bool kEarly = ZT_EARLY_GEN && (ZM & kZLoad) != 0 && SHAPE != kFastChain1;
    float z1[8];
    if constexpr (kEarly) {
      const zt::RoundKeys rk = zt::round_keys(st.key1);
#pragma unroll
      for (int e = 0; e < 8; ++e) z1[e] = zt::gauss_rk(e0 + (uint32_t)e, rk);
    }
    // A stream-0 field that is regenerated is computed before theta is unpacked, so the
    // loads land while the noise is computed.
    constexpr bool kEarly0 = ZT_EARLY_GEN0 && (ZM & kZLoad) == 0;
    float z0[8];
    if constexpr (kEarly0) {
      const zt::RoundKeys rk = zt::round_keys(st.key0);
#pragma unroll
      for (int e = 0; e < 8; ++e) z0[e] = zt::gauss_rk(e0 + (uint32_t)e, rk);
    }
    {
      const zt::RoundKeys rk = zt::round_keys(kEarly0 ? 0u : st.key0);
#pragma unroll
      for (int k = 0; k < W::kNW; ++k) {
        float t[W::kPer], gg[W::kPer];
        W::unpack(w[k], t);
        if (SHAPE == kFastAccum) W::unpack(gw[k], gg);
#pragma unroll
        for (int i = 0; i < W::kPer; ++i) {
          const int e = k * W::kPer + i;
          const float z = (ZM & kZLoad) ? zl[e] : (kEarly0 ? z0[e] : zt::gauss_rk(e0 + (uint32_t)e, rk));
          if (SHAPE == kFastChain1 && (ZM & kZStore)) zs[e] = z;
          t[i] = __fmaf_rn(z, a0, t[i]);
          if (SHAPE == kFastAccum) gg[i] = __fmaf_rn(z, gcoef, gg[i]);
        }
        w[k] = W::pack(t);
        if (SHAPE == kFastAccum) gw[k] = W::pack(gg);
      }
    }
    if (SHAPE != kFastChain1) {
      const zt::RoundKeys rk = zt::round_keys(kEarly ? 0u : st.key1);
#pragma unroll
      for (int k = 0; k < W::kNW; ++k) {
        float t[W::kPer];
        W::unpack(w[k], t);
#pragma unroll
        for (int i = 0; i < W::kPer; ++i) {
          const int e = k * W::kPer + i;
          const float z = kEarly ? z1[e] : zt::gauss_rk(e0 + (uint32_t)e, rk);
          if (ZM & kZStore) zs[e] = z;
          t[i] = __fmaf_rn(z, a1, t[i]);
        }
        w[k] = W::pack(t);
      }
    }
    if constexpr ((ZM & kZStore) != 0) st_z<8>(zc, zs);
    if constexpr ((ZM & kZPush) != 0) {
      // the owner of unit u in the flat layout of zpush_ranks ranks, and the unit's place in
      // its store (u and the geometry are block-uniform)
      // (32-bit: this kernel runs on plans of fewer than 2^31 units)
      const uint32_t cu = (uint32_t)c.zpush_chunk_units;
      const uint32_t per_chunk = (uint32_t)c.zpush_ranks * cu;
      const uint32_t kc = (uint32_t)u / per_chunk;
      const uint32_t within = (uint32_t)u - kc * per_chunk;
      const uint32_t p = within / cu;
      const uint32_t o = within - p * cu;
      float* dst = c.zpush[p] + (size_t)c.zpush_slot * (size_t)c.zpush_stride +
                   ((size_t)kc * cu + o) * ZT_UNIT_ELEMS + threadIdx.x * 8u;
      reinterpret_cast<float4*>(dst)[0] = make_float4(zs[0], zs[1], zs[2], zs[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(zs[4], zs[5], zs[6], zs[7]);
    }
    if (SHAPE == kFastAccum) st_words_global<W::kNW>(st.ge + off, gw);
    if (c.dst & ZT_BUF_DATA) st_words_global<W::kNW>(st.data + off, w);
    if (c.dst & ZT_BUF_LIVE) st_words_global<W::kNW>(st.live + off, w);
  }
}

template <int DT, int SHAPE, int ZM>
__global__ void __launch_bounds__(ZT_UNIT_ELEMS / 8, SHAPE == kFastAccum    ? ZT_FAST_ACCUM_MINB
                                                      : SHAPE == kFastReplay ? ZT_FAST_REPLAY_MINB
                                                                             : ZT_FAST_CHAIN_MINB)
fast_kernel(const __grid_constant__ PassParams P) {
  fast_walk<DT, SHAPE, ZM>(P);
  // pushed fields: this thread's stores to the other GPUs' stores are ordered before
  // anything the host orders after the kernel (the collective that ends the pair loop)
  if constexpr ((ZM & kZPush) != 0) __threadfence_system();
}


// Noise-cache variant of a specialised shape: stream 0 may load, the last stream may
// store; anything else (-1) goes to the generic kernels, which take any placement.
int fast_zmode(int shape, const zt_stream* s, int32_t n) {
  if (shape == kFastReplay) {  // reads cached fields stream by stream; stores none
    for (int32_t i = 0; i < n; ++i)
      if (s[i].flags & ZT_STREAM_Z_STORE) return -1;
    return kZNone;
  }
  int zm = 0;
  for (int32_t i = 0; i < n; ++i) {
    if ((s[i].flags & ZT_STREAM_Z_LOAD) && i != 0) return -1;
    if ((s[i].flags & ZT_STREAM_Z_STORE) && i != n - 1) return -1;
  }
  if (n > 0 && (s[0].flags & ZT_STREAM_Z_LOAD)) zm |= kZLoad;
  if (n > 0 && (s[n - 1].flags & ZT_STREAM_Z_STORE)) zm |= kZStore;
  return zm;
}

// The push variant applies to the +eps pass that stores its field (kFastChain1, kZStore).
int fast_zmode_push(int shape, int zm, const zt_pass_cfg* cfg) {
  if (cfg->zpush_ranks <= 0) return zm;
  return (shape == kFastChain1 && zm == kZStore) ? (zm | kZPush) : -1;
}

// The specialised shape a pass matches, ignoring the noise-cache flags, or -1.
int fast_shape_base(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* s, int32_t n) {
  if (!(plan->props & ZT_PLAN_VEC8) || plan->n_units > (int64_t)INT32_MAX - (1 << 24) || cfg->ge_scale_on) return -1;
  if (cfg->update) {
    if (cfg->momentum != ZT_MOM_NONE || cfg->second_moment || (cfg->wd != ZT_WD_NONE && cfg->wd != ZT_WD_STANDARD) ||
        cfg->ge_mode != ZT_GE_ACCUM || cfg->ge_store || n < 1)
      return -1;
    for (int32_t i = 0; i < n; ++i)  // a host coefficient, no momentum role (z may come from memory)
      if ((s[i].flags & ~kZSrc) != ZT_STREAM_GE) return -1;
    return kFastReplay;
  }
  auto plain = [](const zt_stream& x) { return x.n_chain == 1 && (x.flags & ~kZFlags) == 0; };
  if (!cfg->ge_load && !cfg->ge_store) {
    if (n == 1 && plain(s[0])) return kFastChain1;
    if (n == 2 && plain(s[0]) && plain(s[1])) return kFastChain2;
    return -1;
  }
  if (cfg->ge_mode == ZT_GE_ACCUM && cfg->ge_store && n == 2 && s[0].n_chain == 1 &&
      (s[0].flags & ~(ZT_STREAM_GE_DEV | kZFlags)) == ZT_STREAM_GE && plain(s[1]))
    return kFastAccum;
  return -1;
}

// The specialised kernel a pass takes (shape + 16 * noise-cache mode), or -1 for the
// generic kernels.
int fast_shape(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* s, int32_t n) {
  const int shape = fast_shape_base(plan, cfg, s, n);
  if (shape < 0) return -1;
  int zm = fast_zmode(shape, s, n);
  if (zm >= 0) zm = fast_zmode_push(shape, zm, cfg);
  return zm < 0 ? -1 : shape + 16 * zm;
}

// Grid = SMs x resident blocks per SM (occupancy queried once per kernel).
template <typename K>
int grid_for(K kernel, int threads, int64_t n_units, std::atomic<int>& occ_cache) {
  int occ = occ_cache.load(std::memory_order_relaxed);
  if (occ <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, 0) != cudaSuccess || occ <= 0) occ = 1;
    occ_cache.store(occ, std::memory_order_relaxed);
  }
  const int64_t cap = (int64_t)zt::sm_count() * occ;
  return (int)(n_units < cap ? n_units : cap);
}

std::atomic<int> g_occ_chain{0}, g_occ_full{0};
std::atomic<int> g_occ_fast[3][kFastShapes][8];

template <int DT, int SHAPE, int ZM>
void launch_fast_one(const PassParams& P, int64_t units, cudaStream_t s) {
  constexpr int th = ZT_UNIT_ELEMS / 8;
  fast_kernel<DT, SHAPE, ZM><<<grid_for(fast_kernel<DT, SHAPE, ZM>, th, units, g_occ_fast[DT][SHAPE][ZM]), th, 0, s>>>(P);
}

// Returns false for a (shape, noise-cache mode) pair without a specialised kernel.
template <int DT>
bool launch_fast(int code, const PassParams& P, int64_t units, cudaStream_t s) {
  switch (code) {
    case kFastChain1: launch_fast_one<DT, kFastChain1, kZNone>(P, units, s); return true;
    case kFastChain1 + 16 * kZLoad: launch_fast_one<DT, kFastChain1, kZLoad>(P, units, s); return true;
    case kFastChain1 + 16 * kZStore: launch_fast_one<DT, kFastChain1, kZStore>(P, units, s); return true;
    case kFastChain1 + 16 * (kZStore | kZPush): launch_fast_one<DT, kFastChain1, kZStore | kZPush>(P, units, s); return true;
    case kFastChain2: launch_fast_one<DT, kFastChain2, kZNone>(P, units, s); return true;
    case kFastChain2 + 16 * kZLoadStore: launch_fast_one<DT, kFastChain2, kZLoadStore>(P, units, s); return true;
    case kFastAccum: launch_fast_one<DT, kFastAccum, kZNone>(P, units, s); return true;
    case kFastAccum + 16 * kZLoadStore: launch_fast_one<DT, kFastAccum, kZLoadStore>(P, units, s); return true;
    case kFastReplay: launch_fast_one<DT, kFastReplay, kZNone>(P, units, s); return true;
    default: return false;
  }
}

}  // namespace

extern "C" {

size_t zt_plan_workspace_bytes(int32_t n_tensors) {
  if (n_tensors < 0) return 0;
  return zt::plan_prefix_offset(n_tensors) + sizeof(int64_t) * ((size_t)n_tensors + 1);
}

int zt_plan_init(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, void* workspace,
                 size_t workspace_bytes, zt_plan* plan, void* stream) {
  zt::clear_error();
  return zt::plan_build(host_tensors, n_tensors, n_params, workspace, workspace_bytes, plan, stream);
}

int zt_pass(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams, void* stream) {
  zt::clear_error();
  return zt::pass_launch(plan, cfg, streams, n_streams, stream);
}

}  // extern "C"

namespace zt {

int plan_scan(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, void* workspace, int64_t* prefix,
              zt_plan* plan) {
  if (!plan || !prefix || (n_tensors > 0 && (!host_tensors || !workspace)))
    return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: null pointer");
  if (n_tensors < 0) return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: n_tensors < 0");
  if (((uintptr_t)workspace & 15) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: workspace not 16-byte aligned");
  prefix[0] = 0;
  int64_t total = 0;
  int32_t buffers = ZT_HAS_LIVE | ZT_HAS_M | ZT_HAS_V | ZT_HAS_ANCHOR | ZT_HAS_GE;
  int32_t props = ZT_PLAN_VEC8 | ZT_PLAN_ALL_F32 | ZT_PLAN_ALL_BF16 | ZT_PLAN_ALL_F16;
  auto a16 = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };  // null counts as aligned
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
      if (!t.ge) buffers &= ~ZT_HAS_GE;
      if (t.numel % 8 != 0 || !a16(t.data) || !a16(t.live) || !a16(t.m) || !a16(t.v) || !a16(t.anchor) || !a16(t.ge))
        props &= ~ZT_PLAN_VEC8;
      if (t.dtype != ZT_F32) props &= ~ZT_PLAN_ALL_F32;
      if (t.dtype != ZT_BF16) props &= ~ZT_PLAN_ALL_BF16;
      if (t.dtype != ZT_F16) props &= ~ZT_PLAN_ALL_F16;
    }
    prefix[i + 1] = prefix[i] + (t.numel + ZT_UNIT_ELEMS - 1) / ZT_UNIT_ELEMS;
    total += t.numel;
  }
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "zt_plan_init: cudaGetDevice")) return rc;
  char* ws = static_cast<char*>(workspace);
  plan->tensors = reinterpret_cast<const zt_tensor*>(ws);
  plan->unit_prefix = reinterpret_cast<const int64_t*>(ws + plan_prefix_offset(n_tensors));
  plan->n_units = prefix[n_tensors];
  plan->numel_total = total;
  plan->n_tensors = n_tensors;
  plan->n_params = n_params;
  plan->device = dev;
  plan->buffers = buffers;
  plan->props = props;
  plan->reserved = 0;
  return ZT_OK;
}

int plan_build(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params, void* workspace,
               size_t workspace_bytes, zt_plan* plan, void* stream) {
  if (n_tensors < 0) return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: n_tensors < 0");
  if (workspace_bytes < zt_plan_workspace_bytes(n_tensors))
    return zt::set_error(ZT_ERR_INVALID, "zt_plan_init: workspace too small");
  std::vector<int64_t> prefix((size_t)n_tensors + 1, 0);
  if (int rc = plan_scan(host_tensors, n_tensors, n_params, workspace, prefix.data(), plan)) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t s = zt::as_stream(stream);
  if (n_tensors > 0) {
    if (int rc = zt::check_cuda(cudaMemcpyAsync(ws, host_tensors, sizeof(zt_tensor) * (size_t)n_tensors,
                                                cudaMemcpyHostToDevice, s), "zt_plan_init: copy tensors")) return rc;
  }
  if (int rc = zt::check_cuda(cudaMemcpyAsync(ws + plan_prefix_offset(n_tensors), prefix.data(),
                                              sizeof(int64_t) * prefix.size(), cudaMemcpyHostToDevice, s),
                              "zt_plan_init: copy prefix")) return rc;
  // The caller's table may be pinned (then the copy reads it when the stream gets there)
  // and the prefix vector dies on return, so the plan is complete on the device, and
  // both host arrays are free, only once the copies have run.
  return zt::check_cuda(cudaStreamSynchronize(s), "zt_plan_init: synchronize");
}

int pass_check(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams) {
  return pass_run(plan, cfg, streams, n_streams, nullptr, false);
}

int pass_launch(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams,
                void* stream) {
  return pass_run(plan, cfg, streams, n_streams, stream, true);
}

int pass_run(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams, void* stream,
             bool launch) {
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
    if ((cfg->ge_load || cfg->ge_store) && !(plan->buffers & ZT_HAS_GE))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: ge_load/ge_store need ge buffers");
    if ((cfg->ge_load || cfg->ge_store) && cfg->ge_mode != ZT_GE_ACCUM)
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: ge_load/ge_store need ge_mode ACCUM");
  }
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "zt_pass: cudaGetDevice")) return rc;
  if (dev != plan->device) return zt::set_error(ZT_ERR_INVALID, "zt_pass: plan belongs to another device");
  if (plan->n_units == 0) return ZT_OK;

  int64_t ub = cfg->unit_begin, ue = cfg->unit_end;
  if (ue <= 0 || ue > plan->n_units) ue = plan->n_units;
  if (ub < 0) return zt::set_error(ZT_ERR_INVALID, "zt_pass: unit_begin < 0");
  if (ub >= ue) return ZT_OK;
  PassParams P;
  P.tensors = plan->tensors;
  P.unit_prefix = plan->unit_prefix;
  P.unit_begin = ub;
  P.n_units = ue;
  P.n_tensors = plan->n_tensors;
  P.n_params = plan->n_params;
  P.cfg = *cfg;
  P.n_streams = n_streams;
  for (int s = 0; s < n_streams; ++s) {
    const zt_stream& S = streams[s];
    if (S.n_chain < 0 || S.n_chain > ZT_MAX_CHAIN) return zt::set_error(ZT_ERR_INVALID, "zt_pass: n_chain outside [0, 3]");
    if ((S.flags & ~(ZT_STREAM_GE | ZT_STREAM_MOM | ZT_STREAM_GE_DEV | kZFlags | ZT_STREAM_Z_FIELD)) != 0)
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad stream flags");
    if ((S.flags & kZFlags) == kZFlags)
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: a stream cannot both load and store the noise cache");
    if ((S.flags & ZT_STREAM_Z_FIELD) && (S.flags & kZFlags))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: a field-store stream cannot also use the noise cache");
    if ((S.flags & ZT_STREAM_Z_FIELD) && (S.zslot < 0 || S.zslot > 65535))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: zslot outside [0, 65535]");
    if ((S.flags & ZT_STREAM_GE_DEV) && (!(S.flags & ZT_STREAM_GE) || !cfg->dev_vals || cfg->ge_mode != ZT_GE_ACCUM))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: GE_DEV stream needs GE, dev_vals and ge_mode ACCUM");
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
    K.zslot = (S.flags & ZT_STREAM_Z_FIELD) ? (uint16_t)S.zslot : (uint16_t)0;
  }
  for (int s = n_streams; s < ZT_MAX_STREAMS; ++s) P.streams[s] = KStream{};
  {
    int n_load = 0, n_store = 0, first_store = n_streams, last_load = -1;
    for (int s = 0; s < n_streams; ++s) {
      if (streams[s].flags & ZT_STREAM_Z_LOAD) { ++n_load; last_load = s; }
      if (streams[s].flags & ZT_STREAM_Z_STORE) { ++n_store; if (s < first_store) first_store = s; }
    }
    if (n_load > 1 || n_store > 1)
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: at most one stream may load and one may store the noise cache");
    if (last_load > first_store)
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: the noise-cache load must come before the store");
    if ((n_load || n_store) && (!cfg->zcache || ((uintptr_t)cfg->zcache & 15u) != 0))
      return zt::set_error(ZT_ERR_INVALID, "zt_pass: noise-cache streams need a 16-byte aligned cfg->zcache");
    if (!n_load && !n_store) P.cfg.zcache = nullptr;
    bool field = false;
    for (int s = 0; s < n_streams; ++s) field = field || (streams[s].flags & ZT_STREAM_Z_FIELD);
    if (field) {
      if (!cfg->zfield || ((uintptr_t)cfg->zfield & 15u) != 0)
        return zt::set_error(ZT_ERR_INVALID, "zt_pass: field-store streams need a 16-byte aligned cfg->zfield");
      if (cfg->zfield_stride % 4 != 0 || cfg->zfield_stride < (ue - ub) * (int64_t)ZT_UNIT_ELEMS)
        return zt::set_error(ZT_ERR_INVALID,
                             "zt_pass: zfield_stride must be a multiple of 4 and cover the pass's unit range");
    } else {
      P.cfg.zfield = nullptr;
      P.cfg.zfield_stride = 0;
    }
    if (cfg->zpush_ranks != 0) {
      if (cfg->zpush_ranks < 0 || cfg->zpush_ranks > ZT_MAX_PUSH_RANKS)
        return zt::set_error(ZT_ERR_INVALID, "zt_pass: zpush_ranks outside [0, ZT_MAX_PUSH_RANKS]");
      for (int p = 0; p < cfg->zpush_ranks; ++p)
        if (!cfg->zpush[p] || ((uintptr_t)cfg->zpush[p] & 15u) != 0)
          return zt::set_error(ZT_ERR_INVALID, "zt_pass: every zpush store must be a 16-byte aligned pointer");
      if (cfg->zpush_chunk_units <= 0 || cfg->zpush_chunk_units * cfg->zpush_ranks > (int64_t)INT32_MAX ||
          cfg->zpush_slot < 0 || cfg->zpush_stride < 0 || cfg->zpush_stride % 4 != 0)
        return zt::set_error(ZT_ERR_INVALID, "zt_pass: bad zpush geometry (chunk units, slot, stride)");
      const int32_t uni = plan->props & (ZT_PLAN_ALL_F32 | ZT_PLAN_ALL_BF16 | ZT_PLAN_ALL_F16);
      if (!uni || fast_shape(plan, cfg, streams, n_streams) != kFastChain1 + 16 * (kZStore | kZPush))
        return zt::set_error(ZT_ERR_INVALID,
                             "zt_pass: zpush needs the specialised +eps pass (one storing stream, one chain "
                             "coefficient, a plan of one dtype with ZT_PLAN_VEC8)");
    } else {
      for (int p = 0; p < ZT_MAX_PUSH_RANKS; ++p) P.cfg.zpush[p] = nullptr;
    }
  }
  if (!launch) return ZT_OK;
  const int shape = fast_shape(plan, cfg, streams, n_streams);
  const int32_t all_dt = plan->props & (ZT_PLAN_ALL_F32 | ZT_PLAN_ALL_BF16 | ZT_PLAN_ALL_F16);
  bool full = cfg->update || cfg->ge_scale_on || cfg->ge_load || cfg->ge_store;
  for (int s = 0; s < n_streams; ++s) full = full || (streams[s].flags & ~kZFlags) != 0;
  cudaStream_t cs = zt::as_stream(stream);
  bool done = false;
  if (shape >= 0 && all_dt == ZT_PLAN_ALL_BF16) done = launch_fast<ZT_BF16>(shape, P, ue - ub, cs);
  else if (shape >= 0 && all_dt == ZT_PLAN_ALL_F32) done = launch_fast<ZT_F32>(shape, P, ue - ub, cs);
  else if (shape >= 0 && all_dt == ZT_PLAN_ALL_F16) done = launch_fast<ZT_F16>(shape, P, ue - ub, cs);
  if (!done && full) {  // the generic kernels take every plan and stream combination
    constexpr int th = ZT_UNIT_ELEMS / kFullEpt;
    full_kernel<<<grid_for(full_kernel, th, ue - ub, g_occ_full), th, 0, cs>>>(P);
  } else if (!done) {
    constexpr int th = ZT_UNIT_ELEMS / kChainEpt;
    chain_kernel<<<grid_for(chain_kernel, th, ue - ub, g_occ_chain), th, 0, cs>>>(P);
  }
  return zt::check_cuda(cudaGetLastError(), "zt_pass launch");
}

}  // namespace zt
