// Element-wise companions of the EGGROLL population linear: the per-member rank-4
// factors, the per-member RMSNorm, rotary position embedding and SwiGLU of a Llama
// population forward. Each is one or two bandwidth-bound launches over rows that the
// population GEMM reads or writes; together they replace ~20 torch launches per layer.
#include <string>

#include "zt_common.cuh"
#include "zt_philox.cuh"

namespace {

constexpr int kMaxPairs = ZT_EGGROLL_MAX_PAIRS;
constexpr int kFacThreads = 256;
constexpr int kFacBlocks = ZT_EGGROLL_FACTOR_BLOCKS;
constexpr int kGram = 10;  // upper triangle of a symmetric 4 x 4 Gram matrix

// Per-pair Philox keys: by value (ka, kb), or, when seeds is set, derived on the device
// as zt_param_key(seeds[j], n_params, ia / ib) from pair seeds in device memory.
struct PairKeys {
  uint32_t ka[kMaxPairs];
  uint32_t kb[kMaxPairs];
  const uint64_t* seeds;
  uint32_t n_params, ia, ib;
};

__device__ __forceinline__ uint32_t pair_key_a(const PairKeys& K, int j) {
  return K.seeds ? zt::param_key(K.seeds[j], K.n_params, K.ia) : K.ka[j];
}
__device__ __forceinline__ uint32_t pair_key_b(const PairKeys& K, int j) {
  return K.seeds ? zt::param_key(K.seeds[j], K.n_params, K.ib) : K.kb[j];
}

// Host side: the keys of `pairs` pairs from host arrays, or the device seed form.
PairKeys make_pair_keys(const uint32_t* keys_a, const uint32_t* keys_b, int pairs, const uint64_t* seeds,
                        uint32_t n_params, uint32_t ia, uint32_t ib) {
  PairKeys K;
  for (int j = 0; j < kMaxPairs; ++j) {
    K.ka[j] = (!seeds && keys_a && j < pairs) ? keys_a[j] : 0u;
    K.kb[j] = (!seeds && keys_b && j < pairs) ? keys_b[j] : 0u;
  }
  K.seeds = seeds;
  K.n_params = n_params;
  K.ia = ia;
  K.ib = ib;
  return K;
}

__device__ __forceinline__ void gram_add(float g[kGram], const float v[4]) {
  g[0] = fmaf(v[0], v[0], g[0]); g[1] = fmaf(v[0], v[1], g[1]); g[2] = fmaf(v[0], v[2], g[2]);
  g[3] = fmaf(v[0], v[3], g[3]); g[4] = fmaf(v[1], v[1], g[4]); g[5] = fmaf(v[1], v[2], g[5]);
  g[6] = fmaf(v[1], v[3], g[6]); g[7] = fmaf(v[2], v[2], g[7]); g[8] = fmaf(v[2], v[3], g[8]);
  g[9] = fmaf(v[3], v[3], g[9]);
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}

// Pair j (blockIdx.y) draws P (n x 4, stream order o*4 + r under key ka[j]) and Psi
// (4 x k, stream order r*k + t under key kb[j]), rounds both to the parameter dtype and
// writes A = P and B = Psi^T for both members 2j and 2j+1. Items 0..n-1 are rows of P,
// items n..n+k-1 columns of Psi. Each block also writes its partial Gram matrices P^T P
// and Psi Psi^T (fixed-order block reduction) for the normalisation. With a_ext, A is also
// written in bf16 as the GEMM's rank-4 K-slab operand (exact: P is bf16-valued).
template <int DT>
__global__ void __launch_bounds__(kFacThreads) factor_kernel(const __grid_constant__ PairKeys K, int32_t n, int32_t k,
                                                              float4* __restrict__ a, float4* __restrict__ b,
                                                              float* __restrict__ part, uint4* __restrict__ a_ext,
                                                              int32_t ext_slot, __nv_bfloat16* __restrict__ b_ext,
                                                              int32_t b_ext_row) {
  const int j = blockIdx.y;
  const uint32_t ka = pair_key_a(K, j), kb = pair_key_b(K, j);
  const zt::RoundKeys rka = zt::round_keys(ka), rkb = zt::round_keys(kb);  // once per block
  const int items = n + k;
  float gp[kGram], gq[kGram];
#pragma unroll
  for (int e = 0; e < kGram; ++e) gp[e] = gq[e] = 0.f;
  float4* a0 = a + (size_t)(2 * j) * n;
  float4* b0 = b + (size_t)(2 * j) * k;
  for (int i = blockIdx.x * kFacThreads + threadIdx.x; i < items; i += gridDim.x * kFacThreads) {
    float v[4];
    if (i < n) {
#pragma unroll
      for (int r = 0; r < 4; ++r) v[r] = zt::gauss_rk((uint32_t)(4 * i + r), rka);
      zt::Dt<DT>::round2(v[0], v[1]);
      zt::Dt<DT>::round2(v[2], v[3]);
      const float4 f = make_float4(v[0], v[1], v[2], v[3]);
      a0[i] = f;
      a0[i + n] = f;
      if (a_ext) {  // 32-byte K-slab row: [A, A, 0 x 8] or [0 x 8, A, A]
        const uint2 av = make_uint2(bf16x2(v[0], v[1]), bf16x2(v[2], v[3]));
        const uint4 nz = make_uint4(av.x, av.y, av.x, av.y), z = make_uint4(0u, 0u, 0u, 0u);
        uint4* r0 = a_ext + 2 * ((size_t)(2 * j) * n + i);
        uint4* r1 = r0 + 2 * (size_t)n;
        r0[0] = ext_slot ? z : nz;
        r0[1] = ext_slot ? nz : z;
        r1[0] = ext_slot ? z : nz;
        r1[1] = ext_slot ? nz : z;
      }
      gram_add(gp, v);
    } else {
      const int t = i - n;
#pragma unroll
      for (int r = 0; r < 4; ++r) v[r] = zt::gauss_rk((uint32_t)(r * k + t), rkb);
      zt::Dt<DT>::round2(v[0], v[1]);
      zt::Dt<DT>::round2(v[2], v[3]);
      const float4 f = make_float4(v[0], v[1], v[2], v[3]);
      b0[t] = f;
      b0[t + k] = f;
      if (b_ext) {  // B^T rows of both members: [member][b_ext_row + r][t]
        __nv_bfloat16* e0 = b_ext + ((size_t)(2 * j) * 16 + b_ext_row) * k + t;
        __nv_bfloat16* e1 = e0 + (size_t)16 * k;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const __nv_bfloat16 h = __float2bfloat16_rn(v[r]);
          e0[(size_t)r * k] = h;
          e1[(size_t)r * k] = h;
        }
      }
      gram_add(gq, v);
    }
  }
  __shared__ float red[kFacThreads / 32][2 * kGram];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int e = 0; e < kGram; ++e) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      gp[e] += __shfl_xor_sync(0xffffffffu, gp[e], o);
      gq[e] += __shfl_xor_sync(0xffffffffu, gq[e], o);
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int e = 0; e < kGram; ++e) {
      red[warp][e] = gp[e];
      red[warp][kGram + e] = gq[e];
    }
  }
  __syncthreads();
  if (threadIdx.x < 2 * kGram) {
    float s = 0.f;
    for (int w = 0; w < kFacThreads / 32; ++w) s += red[w][threadIdx.x];
    part[((size_t)j * gridDim.x + blockIdx.x) * (2 * kGram) + threadIdx.x] = s;
  }
}

// Signed scale of both members of pair j (one warp per pair): +-sigma * c_j with
// c_j = sqrt(n*k) / (||P Psi||_F + 1e-7), each step rounded to the parameter dtype as
// the reference's low_rank branch evaluates `z * (numel**0.5 / (z.norm() + 1e-7))`.
// ||P Psi||_F^2 = sum_{r,s} (P^T P)_{rs} (Psi Psi^T)_{rs}.
template <int DT>
__global__ void __launch_bounds__(32) factor_scale_kernel(const float* __restrict__ part, int32_t nblk,
                                                          float sqrt_numel, float sigma, int32_t normalize,
                                                          float* __restrict__ scale) {
  // one warp per pair: lane l sums the partials of blocks l, l + 32 (nblk <= 64) in fp64,
  // then a fixed-order butterfly combines the lanes (deterministic)
  const int j = blockIdx.x, lane = threadIdx.x;
  double g[2 * kGram];
#pragma unroll
  for (int e = 0; e < 2 * kGram; ++e) g[e] = 0.0;
  for (int bi = lane; bi < nblk; bi += 32)
#pragma unroll
    for (int e = 0; e < 2 * kGram; ++e) g[e] += (double)part[((size_t)j * nblk + bi) * (2 * kGram) + e];
#pragma unroll
  for (int e = 0; e < 2 * kGram; ++e)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) g[e] += __shfl_xor_sync(0xffffffffu, g[e], o);
  if (lane != 0) return;
  float c = 1.f;
  if (normalize) {
    double fro2 = 0.0;
#pragma unroll
    for (int e = 0; e < kGram; ++e) {
      const bool diag = (e == 0 || e == 4 || e == 7 || e == 9);
      fro2 += (diag ? 1.0 : 2.0) * g[e] * g[kGram + e];
    }
    const float norm = zt::Dt<DT>::round((float)sqrt(fro2 > 0.0 ? fro2 : 0.0));
    const float t = zt::Dt<DT>::round(norm + 1e-7f);
    c = zt::Dt<DT>::round(__fmul_rn(__fdiv_rn(1.0f, t), sqrt_numel));
  }
  const float s = sigma * c;
  scale[2 * j] = s;
  scale[2 * j + 1] = -s;
}

// ---- RMSNorm with per-member weights -------------------------------------------------

// wm[2j][t] = w[t] + sigma z_j[t], wm[2j+1][t] = w[t] - sigma z_j[t] (fp32 fused
// multiply-add, rounded to bf16), z_j[t] the N(0,1) sample at offset t for key keys[j].
__global__ void __launch_bounds__(256) norm_weights_kernel(const __grid_constant__ PairKeys K, const __nv_bfloat16* __restrict__ w,
                                                           int32_t d, float sigma, __nv_bfloat16* __restrict__ wm) {
  const int j = blockIdx.y;
  const uint32_t key = pair_key_a(K, j);
  for (int t = blockIdx.x * 256 + threadIdx.x; t < d; t += gridDim.x * 256) {
    const float z = zt::gauss((uint32_t)t, key);
    const float wf = __bfloat162float(w[t]);
    wm[(size_t)(2 * j) * d + t] = __float2bfloat16_rn(fmaf(sigma, z, wf));
    wm[(size_t)(2 * j + 1) * d + t] = __float2bfloat16_rn(fmaf(-sigma, z, wf));
  }
}

__device__ __forceinline__ void unpack8(const uint4& u, float f[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return l | (h << 16);
}

__device__ __forceinline__ uint4 pack8(const float f[8]) {
  return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One warp per row: y = wm[member] * bf16(x * rsqrt(mean(x^2) + eps)), the Llama RMSNorm
// (fp32 statistics, normalised row rounded to bf16 before the weight product).
constexpr int kNormRows = 8;
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint4* __restrict__ x, const uint4* __restrict__ wm,
                                                      uint4* __restrict__ y, int64_t rows, int32_t d8,
                                                      int32_t rows_per_member, float inv_d, float eps) {
  const int64_t row = (int64_t)blockIdx.x * kNormRows + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x % 32;
  const uint4* xr = x + row * d8;
  float ss = 0.f;
  for (int c = lane; c < d8; c += 32) {
    float f[8];
    unpack8(xr[c], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss * inv_d + eps);
  const uint4* wr = wm + (int64_t)(row / rows_per_member) * d8;
  uint4* yr = y + row * d8;
  for (int c = lane; c < d8; c += 32) {
    float f[8], g[8];
    unpack8(xr[c], f);
    unpack8(wr[c], g);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = g[e] * bf(f[e] * inv);
    yr[c] = pack8(f);
  }
}

// ---- rotary position embedding, in place --------------------------------------------

// x_embed = x * cos + rotate_half(x) * sin with every product and the sum rounded to bf16
// (the torch evaluation of the Llama rotary embedding on bf16 tensors). One thread owns 8
// consecutive dims i of one head's first half and the matching 8 of its second half.
__global__ void __launch_bounds__(256) rope_kernel(uint4* __restrict__ q, uint4* __restrict__ k,
                                                   const uint4* __restrict__ cs, const uint4* __restrict__ sn,
                                                   int64_t rows, int32_t seq, int32_t hq, int32_t hk, int32_t hd) {
  const int half8 = hd / 16;               // 8-element chunks per half head
  const int per_row = (hq + hk) * half8;
  const int64_t total = rows * per_row;
  const int hd8 = hd / 8;
  for (int64_t it = (int64_t)blockIdx.x * 256 + threadIdx.x; it < total; it += (int64_t)gridDim.x * 256) {
    const int64_t row = it / per_row;
    const int rem = (int)(it - row * per_row);
    const int head = rem / half8, c = rem - head * half8;
    uint4* base = head < hq ? q + (row * hq + head) * hd8 : k + (row * hk + (head - hq)) * hd8;
    const int64_t pos = row % seq;
    float x1[8], x2[8], c1[8], c2[8], s1[8], s2[8];
    unpack8(base[c], x1);
    unpack8(base[c + half8], x2);
    unpack8(cs[pos * hd8 + c], c1);
    unpack8(cs[pos * hd8 + c + half8], c2);
    unpack8(sn[pos * hd8 + c], s1);
    unpack8(sn[pos * hd8 + c + half8], s2);
    float o1[8], o2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o1[e] = bf(x1[e] * c1[e]) + bf(-x2[e] * s1[e]);
      o2[e] = bf(x2[e] * c2[e]) + bf(x1[e] * s2[e]);
    }
    base[c] = pack8(o1);
    base[c + half8] = pack8(o2);
  }
}

// ---- SwiGLU ---------------------------------------------------------------------------

// y = bf16(bf16(silu(g)) * u), silu(x) = x / (1 + exp(-x)) in fp32 (torch's bf16 SiLU
// followed by a bf16 product).
__global__ void __launch_bounds__(256) swiglu_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u,
                                                     uint4* __restrict__ y, int64_t n8) {
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n8; i += (int64_t)gridDim.x * 256) {
    float a[8], b[8];
    unpack8(g[i], a);
    unpack8(u[i], b);
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] = bf(a[e] / (1.0f + expf(-a[e]))) * b[e];
    y[i] = pack8(a);
  }
}

// ---- operands of the evolution-strategies update GEMM ------------------------------------

// Row o < n of a_cat: for pair j, columns 8j..8j+3 = hi(v), 8j+4..8j+7 = lo(v) with
// v = coef_j * (scale_2j / sigma) * A_2j[o]; row t < k of b_cat: B_2j[t] twice. One thread
// per (row, pair): consecutive threads write consecutive 16-byte pieces of a row.
__global__ void __launch_bounds__(256) update_operands_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                                              const float* __restrict__ scale,
                                                              const float* __restrict__ coef, int32_t pairs, int64_t n,
                                                              int64_t k, float sigma, uint4* __restrict__ a_cat,
                                                              uint4* __restrict__ b_cat) {
  const int64_t total = (n + k) * pairs;
  for (int64_t it = (int64_t)blockIdx.x * 256 + threadIdx.x; it < total; it += (int64_t)gridDim.x * 256) {
    const int64_t row = it / pairs;
    const int j = (int)(it - row * pairs);
    if (row < n) {
      const float f = coef[j] * (scale[2 * j] / sigma);
      const float4 v = a[(size_t)(2 * j) * n + row];
      const float x[4] = {f * v.x, f * v.y, f * v.z, f * v.w};
      __nv_bfloat16 h[4], l[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        h[r] = __float2bfloat16_rn(x[r]);
        l[r] = __float2bfloat16_rn(x[r] - __bfloat162float(h[r]));
      }
      a_cat[row * pairs + j] = make_uint4(
          (uint32_t)__bfloat16_as_ushort(h[0]) | ((uint32_t)__bfloat16_as_ushort(h[1]) << 16),
          (uint32_t)__bfloat16_as_ushort(h[2]) | ((uint32_t)__bfloat16_as_ushort(h[3]) << 16),
          (uint32_t)__bfloat16_as_ushort(l[0]) | ((uint32_t)__bfloat16_as_ushort(l[1]) << 16),
          (uint32_t)__bfloat16_as_ushort(l[2]) | ((uint32_t)__bfloat16_as_ushort(l[3]) << 16));
    } else {
      const int64_t t = row - n;
      const float4 v = b[(size_t)(2 * j) * k + t];
      const uint32_t p0 = bf16x2(v.x, v.y), p1 = bf16x2(v.z, v.w);
      b_cat[t * pairs + j] = make_uint4(p0, p1, p0, p1);
    }
  }
}

// ---- LoRA adapter tail ----------------------------------------------------------------

// out[t, c] = bf16(out[t, c] + bf16(scale * sum_r xa[t, r] B[c, r])), the tail of a LoRA
// linear (lora_B(lora_A(x)) * scaling cast to bf16 and added to the base output) in one
// pass. A block owns 256*C columns and a band of kLoraBand rows whose xa rows it stages in
// shared memory once; each thread keeps the B rows of its C adjacent columns in registers
// and walks the band 16 rows at a time, the 16 x C outputs loaded together (4-byte
// accesses for C = 2) before the arithmetic.
constexpr int kLoraBand = 128, kLoraStep = 16;

// PARTS = 3: xa holds three partial products per row, [rows, 3R], summed in fp32 in order
// ((p0 + p1) + p2) while the band is staged.
template <int R, int C, int PARTS = 1>
__global__ void __launch_bounds__(256) lora_add_kernel(__nv_bfloat16* __restrict__ out, const float* __restrict__ xa,
                                                       const float* __restrict__ bw, float scale, int64_t rows,
                                                       int32_t n) {
  __shared__ __align__(16) float sxa[kLoraBand][R];
  const int64_t band0 = (int64_t)blockIdx.y * kLoraBand;
  const int nb = (int)((rows - band0) < kLoraBand ? (rows - band0) : kLoraBand);
  for (int i = threadIdx.x; i < kLoraBand * R; i += 256) {
    const int row = i / R, col = i % R;
    float v = 0.f;
    if (row < nb) {
      const float* p = xa + (band0 + row) * (PARTS * R) + col;
      v = PARTS == 1 ? p[0] : __fadd_rn(__fadd_rn(p[0], p[R]), p[2 * R]);
    }
    sxa[row][col] = v;
  }
  __syncthreads();
  const int c0 = (blockIdx.x * 256 + threadIdx.x) * C;
  if (c0 >= n) return;  // n % C == 0: a thread's columns are all in range or all out
  float b[C][R];
#pragma unroll
  for (int j = 0; j < C; ++j)
#pragma unroll
    for (int r = 0; r < R; r += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(bw + (size_t)(c0 + j) * R + r));
      b[j][r] = v.x; b[j][r + 1] = v.y; b[j][r + 2] = v.z; b[j][r + 3] = v.w;
    }
  __nv_bfloat16* ob = out + band0 * n + c0;
  for (int i0 = 0; i0 < nb; i0 += kLoraStep) {
    float o[kLoraStep][C];
#pragma unroll
    for (int i = 0; i < kLoraStep; ++i) {  // independent loads, in flight together
      if (C == 2) {
        const __nv_bfloat162 h = i0 + i < nb ? *reinterpret_cast<const __nv_bfloat162*>(ob + (int64_t)(i0 + i) * n)
                                             : __floats2bfloat162_rn(0.f, 0.f);
        o[i][0] = __low2float(h);
        o[i][C - 1] = __high2float(h);
      } else {
        o[i][0] = i0 + i < nb ? __bfloat162float(ob[(int64_t)(i0 + i) * n]) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < kLoraStep; ++i) {
      float v[C];
#pragma unroll
      for (int j = 0; j < C; ++j) v[j] = 0.f;
#pragma unroll
      for (int r = 0; r < R; r += 4) {
        const float4 xv = *reinterpret_cast<const float4*>(&sxa[i0 + i][r]);
#pragma unroll
        for (int j = 0; j < C; ++j)
          v[j] = fmaf(xv.w, b[j][r + 3], fmaf(xv.z, b[j][r + 2], fmaf(xv.y, b[j][r + 1], fmaf(xv.x, b[j][r], v[j]))));
      }
      if (i0 + i < nb) {
        float y[C];
#pragma unroll
        for (int j = 0; j < C; ++j) y[j] = o[i][j] + __bfloat162float(__float2bfloat16_rn(v[j] * scale));
        if (C == 2)
          *reinterpret_cast<__nv_bfloat162*>(ob + (int64_t)(i0 + i) * n) = __floats2bfloat162_rn(y[0], y[C - 1]);
        else
          ob[(int64_t)(i0 + i) * n] = __float2bfloat16_rn(y[0]);
      }
    }
  }
}

int stream_grid(int64_t items, int per_sm) {
  const int64_t want = (items + 255) / 256;
  const int64_t cap = (int64_t)zt::sm_count() * per_sm;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// The same tail with the rank-R product on the tensor cores: mma.sync m16n8k8 on TF32
// operands, each fp32 input split as hi = tf32(v), lo = tf32(v - hi) and the product
// taken as lo*hi + hi*lo + hi*hi (the dropped lo*lo term and the TF32 rounding of lo
// leave ~2^-22 relative, far inside the bf16 rounding that follows). A block owns a band
// of 64 rows and walks up to kBandChunks chunks of 128 columns: the band of xa (the three
// partial products summed in order when PARTS = 3) is staged once as TF32 hi / lo parts
// and kept in registers as MMA fragments; per chunk, the chunk's 128 rows of b are staged
// the same way, warp w computes rows 16*(w/2) .. +16 and columns 64*(w%2) .. +64 and
// writes bf16(scale * delta) to a shared tile (rows padded to 136 bf16: conflict-free
// fragment writes), and every thread updates 8 consecutive outputs of a row with one
// 16-byte read and write of out. The next chunk's out tile and b rows are requested
// before the current chunk is multiplied, so HBM reads overlap the arithmetic.
constexpr int kMmaRows = 64, kMmaCols = 128, kMmaLdd = kMmaCols + 8;
constexpr int kBandChunks = 8;

__device__ __forceinline__ uint32_t tf32_of(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <int R, int PARTS>
__global__ void __launch_bounds__(256, 2) lora_add_mma_kernel(__nv_bfloat16* __restrict__ out,
                                                              const float* __restrict__ xa,
                                                              const float* __restrict__ bw, float scale,
                                                              int64_t rows, int32_t n, int32_t chunks_per_block) {
  static_assert(R % 8 == 0 && R <= 16, "k steps of 8; the staged operands fit 48 KB up to R = 16");
  constexpr int KS = R / 8;
  constexpr int LD = R + 4;  // padded rows: conflict-free fragment reads
  constexpr int R4 = R / 4;
  constexpr int BV = (kMmaCols * R4 + 255) / 256;  // b float4 pieces per thread per chunk
  // operands staged as their TF32 hi / lo parts (bit patterns)
  __shared__ uint32_t sah[kMmaRows][LD], sal[kMmaRows][LD];
  __shared__ uint32_t sbh[kMmaCols][LD], sbl[kMmaCols][LD];
  __shared__ __align__(16) __nv_bfloat16 sd[kMmaRows][kMmaLdd];
  const int64_t row0 = (int64_t)blockIdx.y * kMmaRows;
  const int nr = (int)((rows - row0) < kMmaRows ? (rows - row0) : kMmaRows);
  const int n_chunks = (n + kMmaCols - 1) / kMmaCols;
  const int c_begin = blockIdx.x * chunks_per_block;
  const int c_end = min(c_begin + chunks_per_block, n_chunks);
  const int cq = (threadIdx.x % 16) * 8, q0 = threadIdx.x / 16;
  uint4 ov[kMmaRows / 16], ovn[kMmaRows / 16];
  float4 bv[BV], bvn[BV];
  // out tile (16 threads per row, 8 columns each; n % 8 == 0: a group is wholly in or out
  // of range) and b rows of chunk c into registers
  auto load_chunk = [&](int c, uint4 (&o)[kMmaRows / 16], float4 (&b)[BV]) {
    const int col0 = c * kMmaCols;
    const int nc = (n - col0) < kMmaCols ? (n - col0) : kMmaCols;
#pragma unroll
    for (int j = 0; j < kMmaRows / 16; ++j)
      if (q0 + 16 * j < nr && cq < nc) o[j] = *reinterpret_cast<const uint4*>(out + (row0 + q0 + 16 * j) * n + col0 + cq);
#pragma unroll
    for (int v = 0; v < BV; ++v) {
      const int i = threadIdx.x + 256 * v;
      const int cc = i / R4, k = (i % R4) * 4;
      b[v] = (i < kMmaCols * R4 && cc < nc) ? __ldg(reinterpret_cast<const float4*>(bw + (size_t)(col0 + cc) * R + k))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  if (c_begin >= c_end) return;
  load_chunk(c_begin, ov, bv);
  // the band of xa, once per block
  for (int i = threadIdx.x; i < kMmaRows * R4; i += 256) {
    const int rr = i / R4, k = (i % R4) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rr < nr) {
      const float* p = xa + (row0 + rr) * (PARTS * R) + k;
      v = *reinterpret_cast<const float4*>(p);
      if (PARTS == 3) {
        const float4 v1 = *reinterpret_cast<const float4*>(p + R);
        const float4 v2 = *reinterpret_cast<const float4*>(p + 2 * R);
        v = make_float4(__fadd_rn(__fadd_rn(v.x, v1.x), v2.x), __fadd_rn(__fadd_rn(v.y, v1.y), v2.y),
                        __fadd_rn(__fadd_rn(v.z, v1.z), v2.z), __fadd_rn(__fadd_rn(v.w, v1.w), v2.w));
      }
    }
    const float e4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t h = tf32_of(e4[e]);
      sah[rr][k + e] = h;
      sal[rr][k + e] = tf32_of(__fsub_rn(e4[e], __uint_as_float(h)));
    }
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, t = lane % 4;
  const int wr = (warp / 2) * 16, wc = (warp % 2) * 64;
  uint32_t ahi[KS][4], alo[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const int kb = ks * 8;
    ahi[ks][0] = sah[wr + g][kb + t];     alo[ks][0] = sal[wr + g][kb + t];
    ahi[ks][1] = sah[wr + g + 8][kb + t]; alo[ks][1] = sal[wr + g + 8][kb + t];
    ahi[ks][2] = sah[wr + g][kb + t + 4]; alo[ks][2] = sal[wr + g][kb + t + 4];
    ahi[ks][3] = sah[wr + g + 8][kb + t + 4];
    alo[ks][3] = sal[wr + g + 8][kb + t + 4];
  }
  for (int c = c_begin; c < c_end; ++c) {
    const int col0 = c * kMmaCols;
    const int nc = (n - col0) < kMmaCols ? (n - col0) : kMmaCols;
    __syncthreads();  // the previous chunk is done with sbh / sbl and sd
#pragma unroll
    for (int v = 0; v < BV; ++v) {
      const int i = threadIdx.x + 256 * v;
      if (i >= kMmaCols * R4) continue;
      const int cc = i / R4, k = (i % R4) * 4;
      const float e4[4] = {bv[v].x, bv[v].y, bv[v].z, bv[v].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t h = tf32_of(e4[e]);
        sbh[cc][k + e] = h;
        sbl[cc][k + e] = tf32_of(__fsub_rn(e4[e], __uint_as_float(h)));
      }
    }
    if (c + 1 < c_end) load_chunk(c + 1, ovn, bvn);   // in flight while this chunk is multiplied
    __syncthreads();
#pragma unroll
    for (int ni = 0; ni < 8; ++ni) {
      const int cb = wc + ni * 8;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const uint32_t bhi[2] = {sbh[cb + g][ks * 8 + t], sbh[cb + g][ks * 8 + t + 4]};
        const uint32_t blo[2] = {sbl[cb + g][ks * 8 + t], sbl[cb + g][ks * 8 + t + 4]};
        mma_tf32(acc, alo[ks], bhi);
        mma_tf32(acc, ahi[ks], blo);
        mma_tf32(acc, ahi[ks], bhi);
      }
      // acc: rows wr + g and wr + g + 8, columns cb + 2t, cb + 2t + 1
      *reinterpret_cast<__nv_bfloat162*>(&sd[wr + g][cb + 2 * t]) = __floats2bfloat162_rn(acc[0] * scale, acc[1] * scale);
      *reinterpret_cast<__nv_bfloat162*>(&sd[wr + g + 8][cb + 2 * t]) =
          __floats2bfloat162_rn(acc[2] * scale, acc[3] * scale);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kMmaRows / 16; ++j) {
      const int rr = q0 + 16 * j;
      if (rr >= nr || cq >= nc) continue;
      uint4* p = reinterpret_cast<uint4*>(out + (row0 + rr) * n + col0 + cq);
      const uint4 o = ov[j];
      const uint4 dv = *reinterpret_cast<const uint4*>(&sd[rr][cq]);
      const uint32_t ow[4] = {o.x, o.y, o.z, o.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
      uint32_t yw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 of = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ow[e]));
        const float2 df = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dw[e]));
        const __nv_bfloat162 y = __floats2bfloat162_rn(of.x + df.x, of.y + df.y);
        yw[e] = *reinterpret_cast<const uint32_t*>(&y);
      }
      *p = make_uint4(yw[0], yw[1], yw[2], yw[3]);
    }
#pragma unroll
    for (int j = 0; j < kMmaRows / 16; ++j) ov[j] = ovn[j];
#pragma unroll
    for (int v = 0; v < BV; ++v) bv[v] = bvn[v];
  }
}

template <int PARTS>
int lora_add_launch(const char* name, void* out, const float* xa, const float* b, float scale, int64_t rows, int64_t n,
                    int32_t r, void* stream) {
  const std::string nm(name);
  if (rows < 0 || n <= 0) return zt::set_error(ZT_ERR_INVALID, nm + ": bad shape");
  if (rows == 0) return ZT_OK;
  if (!out || !xa || !b) return zt::set_error(ZT_ERR_INVALID, nm + ": null pointer");
  if (n > (int64_t)INT32_MAX) return zt::set_error(ZT_ERR_LIMIT, nm + ": shape too large");
  if (!aligned16(b)) return zt::set_error(ZT_ERR_INVALID, nm + ": b not 16-byte aligned");
  if (r != 4 && r != 8 && r != 16 && r != 32 && r != 64)
    return zt::set_error(ZT_ERR_INVALID, nm + ": rank must be 4, 8, 16, 32 or 64");
  cudaStream_t s = zt::as_stream(stream);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  const int32_t ni = (int32_t)n;
  if ((r == 8 || r == 16) && n % 8 == 0 && aligned16(out) && aligned16(xa)) {  // tensor-core form
    // chunks of 128 columns per block: enough blocks for ~4 per SM, at most kBandChunks
    const int64_t n_chunks = (n + kMmaCols - 1) / kMmaCols, bands = (rows + kMmaRows - 1) / kMmaRows;
    const int64_t want = 4 * (int64_t)zt::sm_count();
    int64_t per = (n_chunks * bands) / want;
    per = per < 1 ? 1 : (per > kBandChunks ? kBandChunks : per);
    const dim3 g2((unsigned)((n_chunks + per - 1) / per), (unsigned)bands);
    if (g2.y > 65535u) return zt::set_error(ZT_ERR_LIMIT, nm + ": too many rows");
    switch (r) {
      case 8: lora_add_mma_kernel<8, PARTS><<<g2, 256, 0, s>>>(o, xa, b, scale, rows, ni, (int32_t)per); break;
      default: lora_add_mma_kernel<16, PARTS><<<g2, 256, 0, s>>>(o, xa, b, scale, rows, ni, (int32_t)per); break;
    }
    return zt::check_cuda(cudaGetLastError(), (nm + " launch").c_str());
  }
  const int cols = (r <= 32 && n % 2 == 0 && ((uintptr_t)out & 3) == 0) ? 2 : 1;   // columns per thread
  const dim3 grid((unsigned)((n + 256 * cols - 1) / (256 * cols)), (unsigned)((rows + kLoraBand - 1) / kLoraBand));
  if (grid.y > 65535u) return zt::set_error(ZT_ERR_LIMIT, nm + ": too many rows");
  if (cols == 2) {
    switch (r) {
      case 4: lora_add_kernel<4, 2, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
      case 8: lora_add_kernel<8, 2, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
      case 16: lora_add_kernel<16, 2, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
      default: lora_add_kernel<32, 2, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
    }
  } else {
    switch (r) {
      case 4: lora_add_kernel<4, 1, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
      case 8: lora_add_kernel<8, 1, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
      case 16: lora_add_kernel<16, 1, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
      case 32: lora_add_kernel<32, 1, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
      default: lora_add_kernel<64, 1, PARTS><<<grid, 256, 0, s>>>(o, xa, b, scale, rows, ni); break;
    }
  }
  return zt::check_cuda(cudaGetLastError(), (nm + " launch").c_str());
}

// out[0:n] = bf16(a), out[n:2n] = bf16(a - a0), out[2n:3n] = bf16((a - a0) - a1): three bf16
// parts that sum to a exactly (a0 + a1 carry 16 of its bits, the rest fits a2), the
// operand of a tensor-core x A^T whose fp32 result equals the fp32 product.
__global__ void __launch_bounds__(256) lora_split_kernel(const float* __restrict__ a, __nv_bfloat16* __restrict__ out,
                                                         int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
    const float v = a[i];
    const __nv_bfloat16 a0 = __float2bfloat16_rn(v);
    const float rest = __fsub_rn(v, __bfloat162float(a0));
    const __nv_bfloat16 a1 = __float2bfloat16_rn(rest);
    out[i] = a0;
    out[n + i] = a1;
    out[2 * n + i] = __float2bfloat16_rn(__fsub_rn(rest, __bfloat162float(a1)));
  }
}

}  // namespace

extern "C" {

int zt_eggroll_factors(const zt_eggroll_factor_args* args, void* stream) {
  zt::clear_error();
  if (!args) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: null args");
  const zt_eggroll_factor_args& A = *args;
  if (A.rank != 4) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: rank must be 4");
  if (A.pairs <= 0 || A.n <= 0 || A.k <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: empty shape");
  if (A.pairs > kMaxPairs) return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_factors: more than ZT_EGGROLL_MAX_PAIRS pairs");
  if (A.n * 4 > (int64_t)ZT_MAX_NUMEL || A.k * 4 > (int64_t)ZT_MAX_NUMEL)
    return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_factors: factor fields beyond 2^31 elements");
  if ((!A.seeds && (!A.keys_a || !A.keys_b)) || !A.a || !A.b || !A.scale || !A.work)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: null pointer");
  if (!aligned16(A.a) || !aligned16(A.b)) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: a, b not 16-byte aligned");
  if (A.dtype != ZT_F32 && A.dtype != ZT_BF16 && A.dtype != ZT_F16)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: unknown dtype");
  const PairKeys K = make_pair_keys(A.keys_a, A.keys_b, A.pairs, A.seeds, A.n_params, A.key_index_a, A.key_index_b);
  const int64_t items = A.n + A.k;
  int64_t nblk = (items + 4 * kFacThreads - 1) / (4 * kFacThreads);
  if (nblk > kFacBlocks) nblk = kFacBlocks;
  const dim3 grid((unsigned)nblk, (unsigned)A.pairs);
  cudaStream_t s = zt::as_stream(stream);
  float4* a4 = reinterpret_cast<float4*>(A.a);
  float4* b4 = reinterpret_cast<float4*>(A.b);
  const float sqrt_numel = (float)sqrt((double)A.n * (double)A.k);
  if (A.a_ext && (!aligned16(A.a_ext) || A.ext_slot < 0 || A.ext_slot > 1))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: a_ext not 16-byte aligned or ext_slot not 0/1");
  uint4* ae = static_cast<uint4*>(A.a_ext);
  if (A.b_ext && (A.b_ext_row < 0 || A.b_ext_row > 12 || A.b_ext_row % 4))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_factors: b_ext_row must be 0, 4, 8 or 12");
  __nv_bfloat16* be = static_cast<__nv_bfloat16*>(A.b_ext);
  switch (A.dtype) {
    case ZT_F32:
      factor_kernel<ZT_F32><<<grid, kFacThreads, 0, s>>>(K, (int32_t)A.n, (int32_t)A.k, a4, b4, A.work, ae, A.ext_slot, be, A.b_ext_row);
      factor_scale_kernel<ZT_F32><<<(unsigned)A.pairs, 32, 0, s>>>(A.work, (int32_t)nblk, sqrt_numel, A.sigma, A.normalize, A.scale);
      break;
    case ZT_BF16:
      factor_kernel<ZT_BF16><<<grid, kFacThreads, 0, s>>>(K, (int32_t)A.n, (int32_t)A.k, a4, b4, A.work, ae, A.ext_slot, be, A.b_ext_row);
      factor_scale_kernel<ZT_BF16><<<(unsigned)A.pairs, 32, 0, s>>>(A.work, (int32_t)nblk, sqrt_numel, A.sigma, A.normalize, A.scale);
      break;
    default:
      factor_kernel<ZT_F16><<<grid, kFacThreads, 0, s>>>(K, (int32_t)A.n, (int32_t)A.k, a4, b4, A.work, ae, A.ext_slot, be, A.b_ext_row);
      factor_scale_kernel<ZT_F16><<<(unsigned)A.pairs, 32, 0, s>>>(A.work, (int32_t)nblk, sqrt_numel, A.sigma, A.normalize, A.scale);
      break;
  }
  return zt::check_cuda(cudaGetLastError(), "zt_eggroll_factors launch");
}

int zt_eggroll_rmsnorm(const zt_eggroll_norm_args* args, void* stream) {
  zt::clear_error();
  if (!args) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rmsnorm: null args");
  const zt_eggroll_norm_args& A = *args;
  if (A.pairs <= 0 || A.m <= 0 || A.d <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rmsnorm: empty shape");
  if (A.pairs > kMaxPairs) return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_rmsnorm: more than ZT_EGGROLL_MAX_PAIRS pairs");
  if (A.d % 8 || A.d > (int64_t)ZT_MAX_NUMEL) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rmsnorm: d must be a multiple of 8");
  if (A.rows_per_member <= 0 || A.m != (int64_t)A.rows_per_member * 2 * A.pairs)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rmsnorm: m must equal rows_per_member * 2 * pairs");
  if ((!A.keys && !A.seeds) || !A.x || !A.w || !A.w_members || !A.y)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rmsnorm: null pointer");
  if (!aligned16(A.x) || !aligned16(A.w_members) || !aligned16(A.y))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rmsnorm: x, w_members, y not 16-byte aligned");
  const PairKeys K = make_pair_keys(A.keys, nullptr, A.pairs, A.seeds, A.n_params, A.key_index, 0u);
  cudaStream_t s = zt::as_stream(stream);
  const dim3 wgrid((unsigned)((A.d + 255) / 256), (unsigned)A.pairs);
  norm_weights_kernel<<<wgrid, 256, 0, s>>>(K, static_cast<const __nv_bfloat16*>(A.w), (int32_t)A.d, A.sigma,
                                            static_cast<__nv_bfloat16*>(A.w_members));
  if (int rc = zt::check_cuda(cudaGetLastError(), "zt_eggroll_rmsnorm: weights launch")) return rc;
  const unsigned grid = (unsigned)((A.m + kNormRows - 1) / kNormRows);
  rmsnorm_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(A.x), static_cast<const uint4*>(A.w_members),
                                      static_cast<uint4*>(A.y), A.m, (int32_t)(A.d / 8), A.rows_per_member,
                                      1.0f / (float)A.d, A.eps);
  return zt::check_cuda(cudaGetLastError(), "zt_eggroll_rmsnorm launch");
}

int zt_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t d, float eps, void* stream) {
  zt::clear_error();
  if (rows < 0 || d <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_rmsnorm: bad shape");
  if (rows == 0) return ZT_OK;
  if (d % 8 || d > (int64_t)ZT_MAX_NUMEL) return zt::set_error(ZT_ERR_INVALID, "zt_rmsnorm: d must be a multiple of 8");
  if (rows > (int64_t)INT32_MAX) return zt::set_error(ZT_ERR_LIMIT, "zt_rmsnorm: more than 2^31-1 rows");
  if (!x || !w || !y) return zt::set_error(ZT_ERR_INVALID, "zt_rmsnorm: null pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y)) return zt::set_error(ZT_ERR_INVALID, "zt_rmsnorm: pointers must be 16-byte aligned");
  // One weight row for all rows: rows_per_member = rows maps every row to member 0.
  const unsigned grid = (unsigned)((rows + kNormRows - 1) / kNormRows);
  rmsnorm_kernel<<<grid, 256, 0, zt::as_stream(stream)>>>(static_cast<const uint4*>(x), static_cast<const uint4*>(w),
                                                          static_cast<uint4*>(y), rows, (int32_t)(d / 8), (int32_t)rows,
                                                          1.0f / (float)d, eps);
  return zt::check_cuda(cudaGetLastError(), "zt_rmsnorm launch");
}

int zt_eggroll_rope(void* q, void* k, const void* cos, const void* sin, int64_t rows, int32_t seq, int32_t q_heads,
                    int32_t k_heads, int32_t head_dim, void* stream) {
  zt::clear_error();
  if (rows <= 0 || seq <= 0 || q_heads <= 0 || k_heads < 0 || head_dim <= 0)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rope: empty shape");
  if (head_dim % 16) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rope: head_dim must be a multiple of 16");
  if (rows % seq) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rope: rows must be a multiple of seq");
  if (!q || (k_heads > 0 && !k) || !cos || !sin) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rope: null pointer");
  if (!aligned16(q) || (k && !aligned16(k)) || !aligned16(cos) || !aligned16(sin))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_rope: pointers must be 16-byte aligned");
  const int64_t items = rows * (int64_t)(q_heads + k_heads) * (head_dim / 16);
  rope_kernel<<<stream_grid(items, 16), 256, 0, zt::as_stream(stream)>>>(
      static_cast<uint4*>(q), static_cast<uint4*>(k), static_cast<const uint4*>(cos), static_cast<const uint4*>(sin),
      rows, seq, q_heads, k_heads, head_dim);
  return zt::check_cuda(cudaGetLastError(), "zt_eggroll_rope launch");
}

int zt_eggroll_swiglu(const void* gate, const void* up, void* out, int64_t n, void* stream) {
  zt::clear_error();
  if (n < 0 || n % 8) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_swiglu: n must be a non-negative multiple of 8");
  if (n == 0) return ZT_OK;
  if (!gate || !up || !out) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_swiglu: null pointer");
  if (!aligned16(gate) || !aligned16(up) || !aligned16(out))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_swiglu: pointers must be 16-byte aligned");
  swiglu_kernel<<<stream_grid(n / 8, 16), 256, 0, zt::as_stream(stream)>>>(
      static_cast<const uint4*>(gate), static_cast<const uint4*>(up), static_cast<uint4*>(out), n / 8);
  return zt::check_cuda(cudaGetLastError(), "zt_eggroll_swiglu launch");
}

int zt_eggroll_update_operands(const float* a, const float* b, const float* scale, const float* coef, int32_t pairs,
                               int64_t n, int64_t k, float sigma, void* a_cat, void* b_cat, void* stream) {
  zt::clear_error();
  if (pairs <= 0 || n <= 0 || k <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_update_operands: empty shape");
  if (pairs > kMaxPairs) return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_update_operands: more than ZT_EGGROLL_MAX_PAIRS pairs");
  if (!a || !b || !scale || !coef || !a_cat || !b_cat)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_update_operands: null pointer");
  if (!aligned16(a) || !aligned16(b) || !aligned16(a_cat) || !aligned16(b_cat))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_update_operands: a, b, a_cat, b_cat not 16-byte aligned");
  if (!(sigma > 0.f)) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_update_operands: sigma must be positive");
  update_operands_kernel<<<stream_grid((n + k) * (int64_t)pairs, 16), 256, 0, zt::as_stream(stream)>>>(
      reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), scale, coef, pairs, n, k, sigma,
      static_cast<uint4*>(a_cat), static_cast<uint4*>(b_cat));
  return zt::check_cuda(cudaGetLastError(), "zt_eggroll_update_operands launch");
}

int zt_lora_add(void* out, const float* xa, const float* b, float scale, int64_t rows, int64_t n, int32_t r,
                void* stream) {
  zt::clear_error();
  return lora_add_launch<1>("zt_lora_add", out, xa, b, scale, rows, n, r, stream);
}

int zt_lora_add3(void* out, const float* xa3, const float* b, float scale, int64_t rows, int64_t n, int32_t r,
                 void* stream) {
  zt::clear_error();
  return lora_add_launch<3>("zt_lora_add3", out, xa3, b, scale, rows, n, r, stream);
}

int zt_lora_split(const float* a, void* out, int64_t n, void* stream) {
  zt::clear_error();
  if (n < 0) return zt::set_error(ZT_ERR_INVALID, "zt_lora_split: n < 0");
  if (n == 0) return ZT_OK;
  if (!a || !out) return zt::set_error(ZT_ERR_INVALID, "zt_lora_split: null pointer");
  lora_split_kernel<<<stream_grid(n, 8), 256, 0, zt::as_stream(stream)>>>(a, static_cast<__nv_bfloat16*>(out), n);
  return zt::check_cuda(cudaGetLastError(), "zt_lora_split launch");
}

}  // extern "C"
