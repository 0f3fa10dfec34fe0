/* Oracle (test infrastructure only): plain-C restatement of the reference's
 * noise source and of the elementwise arithmetic of its optimizer passes.
 *
 * Noise: the reference's `_philox_randn(seed, n)` (zotitan/train_zo.py:18-28)
 * evaluates Triton 3.6.0's `tl.random.randn(seed, offs)`:
 *   philox_impl  triton/language/random.py:12-42  (Philox4x32, 10 rounds)
 *   philox       random.py:45-69                  (key = (seed_lo, seed_hi))
 *   randint4x    random.py:88-110                 (counter = (offs, 0, 0, 0))
 *   uint_to_uniform_float random.py:126-143       (int32, x<0 -> -x-1, * 4.6566127342e-10)
 *   pair_uniform_to_normal random.py:181-187      (u1 = max(1e-7, u1); sqrt(-2 log u1) cos(2 pi u2))
 * The Philox words are reproduced exactly. The transcendental functions are
 * evaluated in double precision and rounded once to fp32 (the mathematically
 * intended value); sqrt is the IEEE fp32 square root.
 *
 * Passes: each `zo_*` elementwise routine below is one torch op of the
 * reference's update path, evaluated with fp32 opmath and rounded once to the
 * parameter dtype, as torch does for an in-place op on a bf16/fp16/fp32 tensor.
 * `a + alpha*b` forms use a fused multiply-add (ATen's vectorised add kernel
 * uses fmadd). Citations are on each routine.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ZO_F32 0
#define ZO_BF16 1
#define ZO_F16 2

static const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
static const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;

static void philox4(uint32_t ctr, uint32_t key, uint32_t out[4]) {
  uint32_t c0 = ctr, c1 = 0, c2 = 0, c3 = 0, k0 = key, k1 = 0;
  for (int r = 0; r < 10; ++r) {
    uint64_t a = (uint64_t)M0 * c0;
    uint64_t b = (uint64_t)M1 * c2;
    uint32_t n0 = (uint32_t)(b >> 32) ^ c1 ^ k0;
    uint32_t n2 = (uint32_t)(a >> 32) ^ c3 ^ k1;
    c1 = (uint32_t)b;
    c3 = (uint32_t)a;
    c0 = n0;
    c2 = n2;
    k0 += W0;
    k1 += W1;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

static float to_uniform(uint32_t w) {
  int32_t x = (int32_t)w;
  if (x < 0) x = -(x + 1);           /* -x-1 without signed overflow */
  return (float)x * 4.6566127342e-10f;
}

static float gauss(uint32_t ctr, uint32_t key) {
  uint32_t w[4];
  philox4(ctr, key, w);
  float u1 = to_uniform(w[0]), u2 = to_uniform(w[1]);
  if (u1 < 1.0e-7f) u1 = 1.0e-7f;
  float th = 6.283185307179586f * u2;
  float lg = (float)log((double)u1);
  float r = sqrtf(-2.0f * lg);
  float c = (float)cos((double)th);
  return r * c;
}

/* zotitan/train_zo.py:302 — per-tensor key with uint64 wrap-around, masked. */
uint32_t zo_param_key(uint64_t seed, uint32_t n_params, uint32_t index) {
  return (uint32_t)((seed * (uint64_t)n_params + index) & 0x7FFFFFFFull);
}

void zo_philox_words(uint32_t key, const uint32_t* offs, int64_t n, uint32_t* out4) {
  for (int64_t i = 0; i < n; ++i) philox4(offs[i], key, out4 + 4 * i);
}

/* zotitan/train_zo.py:25-28: fp32 N(0,1) for offsets off0 .. off0+n-1. */
void zo_randn(uint32_t key, int64_t off0, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = gauss((uint32_t)(off0 + i), key);
}

void zo_randn_at(uint32_t key, const uint32_t* offs, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = gauss(offs[i], key);
}

/* ---- rounding to the parameter dtype --------------------------------------- */

static float round_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) {  /* NaN: quiet, keep sign */
    u = (u | 0x00400000u) & 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
  }
  memcpy(&f, &u, 4);
  return f;
}

static float round_f16(float f) { return (float)(_Float16)f; }

static inline float rnd(int dt, float x) {
  return dt == ZO_BF16 ? round_bf16(x) : dt == ZO_F16 ? round_f16(x) : x;
}

/* Values are carried as fp32 arrays; bf16/fp16 values are exact in fp32. */
void zo_round(int dt, float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = rnd(dt, x[i]);
}

/* p.add_(x, alpha=a): zotitan/train_zo.py:351 (_apply_z), :345 (momentum replay),
 * :399 (SGD step), :419 (stored EMA), :556/:577 (grad_est accumulation). */
void zo_add_scaled(int dt, float* p, const float* x, float a, int64_t n) {
  for (int64_t i = 0; i < n; ++i) p[i] = rnd(dt, fmaf(x[i], a, p[i]));
}

/* out = x * s (torch._foreach_mul(z, proj_grad), zotitan/train_zo.py:552; also
 * foreach_mul_ with a scalar at :402, :418, :424, :457). */
void zo_mul_scalar(int dt, float* out, const float* x, float s, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = rnd(dt, x[i] * s);
}

/* out = x / s (torch._foreach_div(v, bc2) at :394; m / (bc + eps) at :331). */
void zo_div_scalar(int dt, float* out, const float* x, float s, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = rnd(dt, x[i] / s);
}

/* v.addcmul_(t, t, value=c): zotitan/train_zo.py:425. torch evaluates
 * self + value * t1 * t2 left to right with the last multiply-add fused. */
void zo_addcmul(int dt, float* v, const float* t1, const float* t2, float c, int64_t n) {
  for (int64_t i = 0; i < n; ++i) v[i] = rnd(dt, fmaf(c * t1[i], t2[i], v[i]));
}

/* sqrt_ then add_(eps): zotitan/train_zo.py:395-396. */
void zo_sqrt_add(int dt, float* x, float eps, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float s = rnd(dt, sqrtf(x[i]));
    x[i] = rnd(dt, s + eps);
  }
}

/* p.addcdiv_(g, d, value=c): zotitan/train_zo.py:397, CPU order (c*g)/d. */
void zo_addcdiv(int dt, float* p, const float* g, const float* d, float c, int64_t n) {
  for (int64_t i = 0; i < n; ++i) p[i] = rnd(dt, p[i] + (c * g[i]) / d[i]);
}

/* Anchored weight decay, zotitan/train_zo.py:403-407:
 *   diff = p - p0 (param dtype); p.sub_(sign(diff) | diff, alpha=lam). */
void zo_anchored(int dt, float* p, const float* p0, float lam, int l1, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float d = rnd(dt, p[i] - p0[i]);
    float x = l1 ? (float)((d > 0.0f) - (d < 0.0f)) : d;
    p[i] = rnd(dt, fmaf(x, -lam, p[i]));
  }
}
