// Counter-based Gaussian noise, bit-compatible with the reference's noise source.
//
// The reference draws every perturbation element with Triton's
// `tl.random.randn(seed, offs)` (zotitan/train_zo.py:18-28), where `offs` is the
// element's int32 offset inside its parameter tensor and `seed` is the per-tensor
// key `(pair_seed * n_params + i) & 0x7FFFFFFF` (zotitan/train_zo.py:302).
// Triton 3.6.0 (third party, triton/language/random.py) defines that as:
//   * Philox4x32 with 10 rounds (Salmon et al., SC'11), counter (offs, 0, 0, 0),
//     key (seed_lo, seed_hi) = (seed, 0) because the key is below 2^31
//     (random.py:12-42 philox_impl, :45-69 philox, :88-110 randint4x);
//   * words 0 and 1 mapped to uniforms: bitcast to int32, negative x -> -x-1,
//     then int->fp32 (round to nearest) times fp32(4.6566127342e-10) (random.py:126-143);
//   * one Box-Muller branch: u1 = max(1e-7, u1), r = sqrt(-2 log u1),
//     n = r * cos(fp32(2*pi) * u2); words 2, 3 and the sine half are dropped
//     (random.py:181-203).
// The Philox constants below are the published Philox4x32 multipliers and Weyl
// key increments; the uniform scale and clamp are the values the reference's
// Triton version uses.
#pragma once
#include <stdint.h>

#ifndef ZT_SQRT_MODE
// 0: IEEE sqrtf, 1: sqrt.approx.f32 (hand-written PTX), 2: sqrt.approx.ftz.f32
#define ZT_SQRT_MODE 1
#endif

namespace zt {

constexpr uint32_t kPhiloxM0 = 0xD2511F53u;   // round multiplier applied to word 0
constexpr uint32_t kPhiloxM1 = 0xCD9E8D57u;   // round multiplier applied to word 2
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u;   // key increment, word 0 (golden ratio)
constexpr uint32_t kPhiloxW1 = 0xBB67AE85u;   // key increment, word 1 (sqrt(3)-1)

// The 64-bit product m * c as its high and low words. Written as __umulhi plus a 32-bit
// multiply rather than one widening multiply: the integer-multiply pipe is the busiest one
// in the noise passes, and this form measured 6-7.5 % faster there (same values).
__device__ __forceinline__ void mul_hilo(uint32_t m, uint32_t c, uint32_t& hi, uint32_t& lo) {
  hi = __umulhi(m, c);
  lo = m * c;
}

// Words 0 and 1 of Philox4x32-10 at counter (ctr, 0, 0, 0), key (key, 0).
// Written with the zero counter/key words explicit so the compiler folds the
// first two rounds.
__device__ __forceinline__ void philox_w01(uint32_t ctr, uint32_t key, uint32_t& w0, uint32_t& w1) {
  uint32_t c0 = ctr, c1 = 0u, c2 = 0u, c3 = 0u;
  uint32_t k0 = key, k1 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t h0, l0, h1, l1;
    mul_hilo(kPhiloxM0, c0, h0, l0);
    mul_hilo(kPhiloxM1, c2, h1, l1);
    const uint32_t n0 = h1 ^ c1 ^ k0;
    const uint32_t n2 = h0 ^ c3 ^ k1;
    c1 = l1;
    c3 = l0;
    c0 = n0;
    c2 = n2;
    k0 += kPhiloxW0;
    k1 += kPhiloxW1;
  }
  w0 = c0;
  w1 = c1;
}

// Round keys of the key-schedule word 0: rk[r] = key + r * kPhiloxW0. Word 1 of the key
// is 0, so its schedule r * kPhiloxW1 is a compile-time constant. Computing rk once per
// (stream, tensor) and sharing it across a thread's elements removes the per-element
// key additions.
struct RoundKeys {
  uint32_t k[10];
};

__device__ __forceinline__ RoundKeys round_keys(uint32_t key) {
  RoundKeys rk;
#pragma unroll
  for (int r = 0; r < 10; ++r) rk.k[r] = key + (uint32_t)r * kPhiloxW0;
  return rk;
}

__device__ __forceinline__ void philox_w01_rk(uint32_t ctr, const RoundKeys& rk, uint32_t& w0, uint32_t& w1) {
  uint32_t c0 = ctr, c1 = 0u, c2 = 0u, c3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t h0, l0, h1, l1;
    mul_hilo(kPhiloxM0, c0, h0, l0);
    mul_hilo(kPhiloxM1, c2, h1, l1);
    const uint32_t n0 = h1 ^ c1 ^ rk.k[r];
    const uint32_t n2 = h0 ^ c3 ^ ((uint32_t)r * kPhiloxW1);
    c1 = l1;
    c3 = l0;
    c0 = n0;
    c2 = n2;
  }
  w0 = c0;
  w1 = c1;
}

// All four words (test entry points only).
__device__ __forceinline__ void philox_w4(uint32_t ctr, uint32_t key, uint32_t w[4]) {
  uint32_t c0 = ctr, c1 = 0u, c2 = 0u, c3 = 0u;
  uint32_t k0 = key, k1 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t h0, l0, h1, l1;
    mul_hilo(kPhiloxM0, c0, h0, l0);
    mul_hilo(kPhiloxM1, c2, h1, l1);
    const uint32_t n0 = h1 ^ c1 ^ k0;
    const uint32_t n2 = h0 ^ c3 ^ k1;
    c1 = l1;
    c3 = l0;
    c0 = n0;
    c2 = n2;
    k0 += kPhiloxW0;
    k1 += kPhiloxW1;
  }
  w[0] = c0; w[1] = c1; w[2] = c2; w[3] = c3;
}

// uint32 word -> uniform in [0, 1): x as int32, x<0 -> -x-1 (== ~x == x ^ (x>>31)).
__device__ __forceinline__ float word_to_uniform(uint32_t w) {
  int32_t x = (int32_t)w;
  x ^= (x >> 31);
  return __int2float_rn(x) * 4.6566127342e-10f;
}

__device__ __forceinline__ float zt_sqrt(float x) {
#if ZT_SQRT_MODE == 0
  return sqrtf(x);
#elif ZT_SQRT_MODE == 1
  float y;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
#else
  float y;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
#endif
}

// Box-Muller cosine branch on the two uniforms.
__device__ __forceinline__ float box_muller_cos(float u1, float u2) {
  u1 = fmaxf(1.0e-7f, u1);
  const float th = 6.283185307179586f * u2;
  const float r = zt_sqrt(-2.0f * logf(u1));
  return r * cosf(th);
}

// N(0,1) sample for element `ctr` of the tensor keyed `key`.
__device__ __forceinline__ float gauss(uint32_t ctr, uint32_t key) {
  uint32_t w0, w1;
  philox_w01(ctr, key, w0, w1);
  return box_muller_cos(word_to_uniform(w0), word_to_uniform(w1));
}

__device__ __forceinline__ float gauss_rk(uint32_t ctr, const RoundKeys& rk) {
  uint32_t w0, w1;
  philox_w01_rk(ctr, rk, w0, w1);
  return box_muller_cos(word_to_uniform(w0), word_to_uniform(w1));
}

// Per-tensor key: (pair_seed * n_params + index) & 0x7FFFFFFF, with uint64
// wrap-around (equal to the reference's Python big-int result after the mask).
__host__ __device__ __forceinline__ uint32_t param_key(uint64_t seed, uint32_t n_params, uint32_t index) {
  return (uint32_t)((seed * (uint64_t)n_params + (uint64_t)index) & 0x7FFFFFFFull);
}

}  // namespace zt
