// Next-token cross-entropy statistics of bf16 logits in one read of each row.
//
// One CTA per row: each thread streams 16-byte chunks of the row and keeps an online
// (max, sum of exp(x - max)) pair and the first argmax; the pairs are merged across the
// block in a fixed order. The row is read once from HBM (the torch path reads it as
// bf16, writes and re-reads an fp32 copy and a log-softmax of the same size).
#include <math.h>

#include "zt_common.cuh"

namespace {

constexpr int kXentThreads = 256;

struct Stat {
  float m;    // running max
  float s;    // sum of exp(x - m)
  float bv;   // argmax value
  int32_t bi; // argmax index (first occurrence)
};

__device__ __forceinline__ Stat merge(const Stat& a, const Stat& b) {
  Stat r;
  r.m = fmaxf(a.m, b.m);
  if (r.m == -INFINITY) {
    r.s = 0.f;
  } else {
    r.s = a.s * expf(a.m - r.m) + b.s * expf(b.m - r.m);
  }
  if (b.bv > a.bv || (b.bv == a.bv && b.bi < a.bi)) {
    r.bv = b.bv;
    r.bi = b.bi;
  } else {
    r.bv = a.bv;
    r.bi = a.bi;
  }
  return r;
}

__device__ __forceinline__ Stat shfl_stat(const Stat& v, int o) {
  Stat r;
  r.m = __shfl_xor_sync(0xffffffffu, v.m, o);
  r.s = __shfl_xor_sync(0xffffffffu, v.s, o);
  r.bv = __shfl_xor_sync(0xffffffffu, v.bv, o);
  r.bi = __shfl_xor_sync(0xffffffffu, v.bi, o);
  return r;
}

__device__ __forceinline__ void absorb(Stat& st, float x, int32_t idx) {
  if (x > st.m) {
    st.s = st.s * expf(st.m - x);
    st.m = x;
  }
  st.s += expf(x - st.m);
  if (x > st.bv) {  // indices arrive in increasing order within a thread
    st.bv = x;
    st.bi = idx;
  }
}

__global__ void __launch_bounds__(kXentThreads) xent_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                                            int32_t vocab, const int64_t* __restrict__ targets,
                                                            float* __restrict__ loss, float* __restrict__ lse,
                                                            int32_t* __restrict__ correct) {
  const int64_t row = blockIdx.x;
  const int64_t t = targets[row];
  if (t < 0) {
    if (threadIdx.x == 0) {
      loss[row] = 0.f;
      if (lse) lse[row] = 0.f;
      if (correct) correct[row] = 0;
    }
    return;
  }
  const __nv_bfloat16* x = logits + row * ld;
  Stat st{-INFINITY, 0.f, -INFINITY, 0x7fffffff};
  const int v8 = vocab / 8;
  const uint4* x8 = reinterpret_cast<const uint4*>(x);
  for (int c = threadIdx.x; c < v8; c += kXentThreads) {
    const uint4 u = __ldcs(x8 + c);  // streamed once: evict-first
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
    float cm = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) cm = fmaxf(cm, f[e]);
    if (cm > st.m) {
      st.s = st.s * expf(st.m - cm);
      st.m = cm;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) st.s += expf(f[e] - st.m);
    if (cm > st.bv) {
      int first = 0;
#pragma unroll
      for (int e = 7; e >= 0; --e)
        if (f[e] == cm) first = e;
      st.bv = cm;
      st.bi = 8 * c + first;
    }
  }
  for (int v = 8 * v8 + threadIdx.x; v < vocab; v += kXentThreads) absorb(st, __bfloat162float(x[v]), v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) st = merge(st, shfl_stat(st, o));
  __shared__ Stat red[kXentThreads / 32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = st;
  __syncthreads();
  if (threadIdx.x == 0) {
    Stat r = red[0];
    for (int w = 1; w < kXentThreads / 32; ++w) r = merge(r, red[w]);
    const float logs = logf(r.s);
    if (t >= vocab) {
      loss[row] = NAN;
      if (lse) lse[row] = NAN;
      if (correct) correct[row] = 0;
      return;
    }
    const float xt = __bfloat162float(x[t]);
    loss[row] = -((xt - r.m) - logs);
    if (lse) lse[row] = logs + r.m;
    if (correct) correct[row] = (r.bi == (int32_t)t) ? 1 : 0;
  }
}

}  // namespace

extern "C" {

int zt_xent_rows(const void* logits, int64_t ld, int64_t rows, int64_t vocab, const int64_t* targets, float* loss,
                 float* lse, int32_t* correct, void* stream) {
  zt::clear_error();
  if (rows < 0 || vocab <= 0 || ld < vocab) return zt::set_error(ZT_ERR_INVALID, "zt_xent_rows: bad shape");
  if (vocab > (int64_t)INT32_MAX - 8) return zt::set_error(ZT_ERR_LIMIT, "zt_xent_rows: vocab above 2^31");
  if (rows > (int64_t)INT32_MAX) return zt::set_error(ZT_ERR_LIMIT, "zt_xent_rows: more than 2^31-1 rows");
  if (rows == 0) return ZT_OK;
  if (!logits || !targets || !loss) return zt::set_error(ZT_ERR_INVALID, "zt_xent_rows: null pointer");
  if (((uintptr_t)logits & 15) != 0 || (ld % 8) != 0)
    return zt::set_error(ZT_ERR_INVALID, "zt_xent_rows: rows must start on 16-byte boundaries (ld % 8 == 0)");
  xent_kernel<<<(unsigned)rows, kXentThreads, 0, zt::as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(logits), ld, (int32_t)vocab, targets, loss, lse, correct);
  return zt::check_cuda(cudaGetLastError(), "zt_xent_rows launch");
}

}  // extern "C"
