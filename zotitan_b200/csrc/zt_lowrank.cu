// Low-rank perturbation directions (distribution "low_rank") as fused tensor-core passes.
//
// The reference draws, for a 2-D parameter i of shape [m, n] and pair seed `seed`
// (zotitan/train_zo.py:295-322, _sample_z):
//   P   = randn(key(i + 2N), m r).view(m, r).to(dtype)          r = min(rank, m)
//   Psi = randn(key(i + N),  r n).view(r, n).to(dtype)
//   z   = P @ Psi                                   (dtype GEMM, fp32 accumulation)
//   z   = z * (sqrt(m n) / (||z||_F + 1e-7))        (torch scalar ops, each rounded to dtype)
// and applies it with _apply_z (:350-351), theta <- round(theta + a z), or folds it into
// the grad estimate (:550-556, :575-577). Materialised, every use of z writes and re-reads
// an m x n tensor several times. Here z never reaches HBM:
//   zt_lowrank_prepare  generates P and Psi^T of S streams into K-major buffers padded to a
//                       multiple of 64 in K with zeros (exact: zero products), runs the
//                       product on tcgen05 CTA pairs with an epilogue that only sums the
//                       squares of the rounded product (per-warp partials, fixed order), and
//                       a small kernel turns each stream's sum into the rounded scale with
//                       torch's op sequence (norm, + 1e-7, reciprocal, * sqrt(m n));
//   zt_lowrank_apply    runs the product again, tile by tile, and in the epilogue reads the
//                       parameter (and grad-estimate) rows, applies the chained
//                       coefficients of every stream in stream order with one rounding per
//                       step, and writes them back: HBM sees the parameter once.
// Streams of one tile run back to back inside one CTA pair, so a tile's rows are updated
// in stream order (the grad estimate sums pairs in the reference's order).
//
// The product z = round(P Psi) is the fp32 sum of r exact bf16/f16 products in K order
// (16 per MMA); cuBLAS may order the sum differently, so an element can differ from the
// reference's materialised product by one unit in the last place where the fp32 sum sits
// on a rounding boundary. The norm is summed in fp32 per thread and in double across
// threads, in a fixed order (deterministic, identical on every rank).
//
// Every mbarrier wait is bounded; on expiry the kernel records an error code
// (zt_lowrank_take_error), raises both CTAs' abort flags, drains its own copies and MMAs
// and frees its tensor memory.
#include "zt_philox.cuh"
#include "zt_tc.cuh"

namespace {

using namespace zt::tc;

constexpr int kThreads = 576;  // warp 0 TMA, warp 1 MMA (leader), warps 2-17 epilogue
constexpr int kEpiWarps = 16;
constexpr int kWarpCols = 256 / (kEpiWarps / 4);  // columns of a tile per epilogue warp (64)
constexpr uint32_t kHalfRows = 128;
constexpr uint32_t kStageA = kHalfRows * kBK * 2;
constexpr uint32_t kStageBytes = 2 * kStageA;
constexpr uint32_t kTile = 256;
constexpr uint32_t kTmemCols = 2 * kTile;
// Per parameter dtype: the A/B stages, and the apply epilogue's staging of the scaled
// direction (each warp's 32 rows x 64 columns in shared memory, rows padded by 16 bytes so
// the row-per-thread writes hit distinct banks). fp32 parameters keep z in fp32.
template <int DT> struct Cfg {
  static constexpr int kStages = DT == ZT_F32 ? 2 : 4;
  static constexpr uint32_t kEsz = DT == ZT_F32 ? 4 : 2;
  static constexpr uint32_t kZRow = kWarpCols * kEsz + 16;
  static constexpr uint32_t kZWarp = 32 * kZRow;
  static constexpr size_t kSmem = 1024 + kStages * kStageBytes + kEpiWarps * kZWarp + 256;
};
constexpr int kGroupN = 16;
constexpr int kPartials = 2 * kEpiWarps;  // per (tile, stream): one per epilogue warp of the pair
constexpr uint32_t kIdescBf16 = idesc_bf16(256, 256);
constexpr uint32_t kIdescF16 = idesc_f16(256, 256);

__device__ int g_lowrank_error = 0;

// 16-bit storage <-> fp32 and rounding of the parameter dtypes (fp32: no rounding).
template <int DT> struct H;
template <> struct H<ZT_F32> {
  __device__ static __forceinline__ float round(float x) { return x; }
  __device__ static __forceinline__ void round2(float&, float&) {}
};
template <> struct H<ZT_BF16> {
  __device__ static __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  __device__ static __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ static __forceinline__ uint16_t bits(float x) {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    return *reinterpret_cast<const uint16_t*>(&h);
  }
  __device__ static __forceinline__ float val(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
  __device__ static __forceinline__ float round(float x) { return zt::Dt<ZT_BF16>::round(x); }
  __device__ static __forceinline__ void round2(float& a, float& b) { zt::Dt<ZT_BF16>::round2(a, b); }
};
template <> struct H<ZT_F16> {
  __device__ static __forceinline__ float lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu))); }
  __device__ static __forceinline__ float hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ static __forceinline__ uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  __device__ static __forceinline__ float val(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  __device__ static __forceinline__ float round(float x) { return zt::Dt<ZT_F16>::round(x); }
  __device__ static __forceinline__ void round2(float& a, float& b) { zt::Dt<ZT_F16>::round2(a, b); }
};

// ---- factors ----------------------------------------------------------------------------

struct FactorKeys {
  uint32_t p[ZT_LOWRANK_MAX_STREAMS];
  uint32_t psi[ZT_LOWRANK_MAX_STREAMS];
};

// Part `part` (0, 1, 2) of the exact three-way bf16 split of an fp32 value: x = hi + mid
// + lo with hi = bf16(x), mid = bf16(x - hi), lo = x - hi - mid (each difference exact in
// fp32, and lo has at most 8 significant bits, so it is exact in bf16).
__device__ __forceinline__ float split3(float x, int part) {
  const float hi = zt::Dt<ZT_BF16>::round(x);
  if (part == 0) return hi;
  const float r1 = __fsub_rn(x, hi);
  const float mid = zt::Dt<ZT_BF16>::round(r1);
  if (part == 1) return mid;
  return __fsub_rn(r1, mid);
}

// Factor value at K position kk of a row: the factor itself for 16-bit parameters
// (k = kk < r, else 0); for fp32 parameters the 9-block split layout, block (a, b) =
// kk / r holding part a of P on the P rows and part b of Psi on the Psi rows, so that the
// product of the two buffers sums all nine exact cross products.
template <int DT>
__device__ __forceinline__ float factor_at(int32_t kk, int32_t r, bool is_p, uint32_t ctr_base, uint32_t ctr_step,
                                           uint32_t key) {
  if (DT != ZT_F32) return kk < r ? zt::gauss(ctr_base + (uint32_t)kk * ctr_step, key) : 0.0f;
  if (kk >= 9 * r) return 0.0f;
  const int32_t blk = kk / r, k = kk - blk * r;
  return split3(zt::gauss(ctr_base + (uint32_t)k * ctr_step, key), is_p ? blk / 3 : blk % 3);
}

// Row `row` of the stacked factor buffers, 8 consecutive K positions per thread:
// rows [0, S m) are P (stream row / m, element i = row % m: P[i, k] = noise(i r + k)),
// rows [S m, S (m + n)) are Psi^T (element j: Psi[k, j] = noise(k n + j)); the operand
// format is the parameter's (bf16 splits for fp32 parameters).
template <int DT>
__global__ void __launch_bounds__(256) lr_factor_kernel(const __grid_constant__ FactorKeys K, uint16_t* __restrict__ p,
                                                        uint16_t* __restrict__ psi_t, int32_t S, int32_t m, int32_t n,
                                                        int32_t r, int32_t kp) {
  constexpr int OT = DT == ZT_F16 ? ZT_F16 : ZT_BF16;  // operand type
  const int32_t groups = kp / 8;
  const int64_t rows = (int64_t)S * ((int64_t)m + n);
  const int64_t total = rows * groups;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = g / groups;
    const int32_t k0 = (int32_t)(g - row * groups) * 8;
    uint32_t w[4];
    if (row < (int64_t)S * m) {
      const int32_t s = (int32_t)(row / m), i = (int32_t)(row - (int64_t)s * m);
      const uint32_t key = K.p[s];
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        w[e / 2] = H<OT>::pack(factor_at<DT>(k0 + e, r, true, (uint32_t)(i * r), 1u, key),
                               factor_at<DT>(k0 + e + 1, r, true, (uint32_t)(i * r), 1u, key));
      *reinterpret_cast<uint4*>(p + row * kp + k0) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      const int64_t rr = row - (int64_t)S * m;
      const int32_t s = (int32_t)(rr / n), j = (int32_t)(rr - (int64_t)s * n);
      const uint32_t key = K.psi[s];
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        w[e / 2] = H<OT>::pack(factor_at<DT>(k0 + e, r, false, (uint32_t)j, (uint32_t)n, key),
                               factor_at<DT>(k0 + e + 1, r, false, (uint32_t)j, (uint32_t)n, key));
      *reinterpret_cast<uint4*>(psi_t + rr * kp + k0) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// ---- the product with a fused epilogue ------------------------------------------------

// kernel roles: the norm pass, and the apply pass writing the parameter, the grad
// estimate, or both (one specialisation each keeps the epilogue loop small)
enum : int { kModeNorm = 0, kModeTheta = 1, kModeGe = 2, kModeBoth = 3 };

struct LrParams {
  CUtensorMap tmap_a;  // stacked P    [S m, kp], box {64, 128}
  CUtensorMap tmap_b;  // stacked Psi^T [S n, kp], box {64, 128}
  const void* src;      // parameter read by stream 0 (later streams read dst)
  void* dst;            // parameter written (nullptr: no parameter update)
  void* ge;             // grad estimate (nullptr: none)
  const float* scale;   // [S] rounded scale of each stream's direction
  float* partial;       // norm mode: [tiles * S][kPartials]
  float alpha[3];
  int32_t n_alpha;
  int32_t ge_init;      // 1: stream 0 sets ge = round(c0 z) instead of accumulating
  int32_t m, n, k_blocks, m_tiles, n_tiles, n_streams;
  int32_t vec;          // rows are 8-element multiples at 16-byte aligned addresses: vector path
  int32_t stall_loads;  // test hook: the loader issues no copies (every wait then expires)
  long long wait_cycles;
  float coef[ZT_LOWRANK_MAX_STREAMS];
};

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int per_group = kGroupN * m_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int rem = n_tiles - g * kGroupN;
  const int gn = rem < kGroupN ? rem : kGroupN;
  mt = r / gn;
  nt = g * kGroupN + r % gn;
}

// Phase 1 of the apply epilogue: 32 accumulator columns of this thread's row ->
// zs = round(round(acc) * sc) into the warp's staging row (packed 16-bit values, or fp32
// for fp32 parameters, where nothing is rounded).
template <int DT>
__device__ __forceinline__ void stage_chunk(const uint32_t (&acc)[32], float sc, uint4* dst) {
  if constexpr (DT == ZT_F32) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dst[i] = make_uint4(__float_as_uint(__fmul_rn(__uint_as_float(acc[4 * i]), sc)),
                          __float_as_uint(__fmul_rn(__uint_as_float(acc[4 * i + 1]), sc)),
                          __float_as_uint(__fmul_rn(__uint_as_float(acc[4 * i + 2]), sc)),
                          __float_as_uint(__fmul_rn(__uint_as_float(acc[4 * i + 3]), sc)));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = 4 * i + k;
        float za = __uint_as_float(acc[2 * j]), zb = __uint_as_float(acc[2 * j + 1]);
        H<DT>::round2(za, zb);
        za = __fmul_rn(za, sc);
        zb = __fmul_rn(zb, sc);
        w[k] = H<DT>::pack(za, zb);   // the second rounding
      }
      dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Phase 2 on 8 consecutive elements (one 16-byte group of the parameter, the grad
// estimate and the staged direction): theta = round(theta + a zs) for each chained
// coefficient, g = round(g + c zs) (g = round(c zs) when `init`).
template <int DT, bool TH, bool GE, typename PT>
__device__ __forceinline__ void apply8(uint4& th, uint4& gv, const uint4 zs, const PT& P, float c, bool init) {
  uint32_t tw[4] = {th.x, th.y, th.z, th.w};
  uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
  const uint32_t zw[4] = {zs.x, zs.y, zs.z, zs.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float za = H<DT>::lo(zw[k]), zb = H<DT>::hi(zw[k]);
    if (TH) {
      float xa = H<DT>::lo(tw[k]), xb = H<DT>::hi(tw[k]);
#pragma unroll
      for (int t = 0; t < 3; ++t) {
        if (t < P.n_alpha) {
          xa = __fmaf_rn(za, P.alpha[t], xa);
          xb = __fmaf_rn(zb, P.alpha[t], xb);
          H<DT>::round2(xa, xb);
        }
      }
      tw[k] = H<DT>::pack(xa, xb);
    }
    if (GE) {
      const float ga = init ? __fmul_rn(za, c) : __fmaf_rn(za, c, H<DT>::lo(gw[k]));
      const float gb = init ? __fmul_rn(zb, c) : __fmaf_rn(zb, c, H<DT>::hi(gw[k]));
      gw[k] = H<DT>::pack(ga, gb);
    }
  }
  th = make_uint4(tw[0], tw[1], tw[2], tw[3]);
  gv = make_uint4(gw[0], gw[1], gw[2], gw[3]);
}

// The same on 8 fp32 elements (two 16-byte words each): no rounding, fused multiply-adds.
template <bool TH, bool GE, typename PT>
__device__ __forceinline__ void apply8_f32(uint4 (&th)[2], uint4 (&gv)[2], const uint4 (&zs)[2], const PT& P, float c,
                                           bool init) {
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const float z[4] = {__uint_as_float(zs[w].x), __uint_as_float(zs[w].y), __uint_as_float(zs[w].z),
                        __uint_as_float(zs[w].w)};
    float x[4] = {__uint_as_float(th[w].x), __uint_as_float(th[w].y), __uint_as_float(th[w].z),
                  __uint_as_float(th[w].w)};
    float g[4] = {__uint_as_float(gv[w].x), __uint_as_float(gv[w].y), __uint_as_float(gv[w].z),
                  __uint_as_float(gv[w].w)};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (TH) {
#pragma unroll
        for (int t = 0; t < 3; ++t)
          if (t < P.n_alpha) x[e] = __fmaf_rn(z[e], P.alpha[t], x[e]);
      }
      if (GE) g[e] = init ? __fmul_rn(z[e], c) : __fmaf_rn(z[e], c, g[e]);
    }
    th[w] = make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3]));
    gv[w] = make_uint4(__float_as_uint(g[0]), __float_as_uint(g[1]), __float_as_uint(g[2]), __float_as_uint(g[3]));
  }
}

template <int DT, bool TH, bool GE, int VW, typename PT>
__device__ __forceinline__ void apply8v(uint4 (&th)[VW], uint4 (&gv)[VW], const uint4 (&zs)[VW], const PT& P, float c,
                                        bool init) {
  if constexpr (DT == ZT_F32)
    apply8_f32<TH, GE>(th, gv, zs, P, c, init);
  else
    apply8<DT, TH, GE>(th[0], gv[0], zs[0], P, c, init);
}

// The same element by element for columns below `n` (rows whose length is not a multiple
// of 8 or buffers not 16-byte aligned); row pointers and the staged row as bytes.
template <int DT, typename PT>
__device__ __forceinline__ void apply_scalar8(const uint8_t* srow, uint8_t* drow, uint8_t* grow, int col,
                                              const uint8_t* zrow, const PT& P, float c, bool init) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if (col + e >= P.n) continue;
    if constexpr (DT == ZT_F32) {
      const float z = reinterpret_cast<const float*>(zrow)[e];
      if (drow) {
        float x = reinterpret_cast<const float*>(srow)[col + e];
        for (int t = 0; t < P.n_alpha; ++t) x = __fmaf_rn(z, P.alpha[t], x);
        reinterpret_cast<float*>(drow)[col + e] = x;
      }
      if (grow) {
        float* g = reinterpret_cast<float*>(grow) + col + e;
        *g = init ? __fmul_rn(z, c) : __fmaf_rn(z, c, *g);
      }
    } else {
      const float z = H<DT>::val(reinterpret_cast<const uint16_t*>(zrow)[e]);
      if (drow) {
        float x = H<DT>::val(reinterpret_cast<const uint16_t*>(srow)[col + e]);
        for (int t = 0; t < P.n_alpha; ++t) x = H<DT>::round(__fmaf_rn(z, P.alpha[t], x));
        reinterpret_cast<uint16_t*>(drow)[col + e] = H<DT>::bits(x);
      }
      if (grow) {
        uint16_t* g = reinterpret_cast<uint16_t*>(grow) + col + e;
        const float gv = init ? __fmul_rn(z, c) : __fmaf_rn(z, c, H<DT>::val(*g));
        *g = H<DT>::bits(gv);
      }
    }
  }
}

template <int DT, int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    lr_gemm_kernel(const __grid_constant__ LrParams P) {
  constexpr int kStages = Cfg<DT>::kStages;
  constexpr uint32_t kZRow = Cfg<DT>::kZRow, kZWarp = Cfg<DT>::kZWarp, kEsz = Cfg<DT>::kEsz;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint8_t* zstage = smem + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(zstage + kEpiWarps * kZWarp);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* accf = bars + 2 * kStages;
  uint64_t* acce = bars + 2 * kStages + 2;
  uint64_t* drain = bars + 2 * kStages + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], 2 * kEpiWarps); }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t peer_abort = peer_addr((const void*)abort, rank ^ 1u);
  const long long wl = P.wait_cycles;

  const int n_tiles = P.m_tiles * P.n_tiles;
  const int S = P.n_streams;
  const int cid = (int)cluster_id_x(), ncl = (int)n_clusters_x();
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs): for each tile, every stream's K blocks
      int last_phase[kStages];
      for (int s = 0; s < kStages; ++s) last_phase[s] = -1;
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < n_tiles; tile += ncl) {
        int mt, nt;
        tile_coords(tile, P.m_tiles, P.n_tiles, mt, nt);
        for (int st = 0; ok && st < S; ++st) {
          for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
            const int s = it % kStages;
            const uint32_t round = it / kStages;
            if (!mbar_wait_pair(&empty[s], (round & 1) ^ 1, abort, peer_abort, &g_lowrank_error, 1, wl)) {
              ok = false;
              break;
            }
            if (P.stall_loads) continue;
            uint8_t* sa = stage_base + s * kStageBytes;
            const uint32_t leader_full = peer_addr(&full[s], 0);
            if (leader) mbar_expect_tx(&full[s], 2 * kStageBytes);
            tma_load_2d_pair(sa, &P.tmap_a, leader_full, kb * kBK,
                             st * P.m + mt * (int)kTile + (int)rank * (int)kHalfRows);
            tma_load_2d_pair(sa + kStageA, &P.tmap_b, leader_full, kb * kBK,
                             st * P.n + nt * (int)kTile + (int)rank * (int)kHalfRows);
            last_phase[s] = (int)(round & 1);
          }
        }
      }
      if (leader)
        for (int s = 0; s < kStages; ++s)
          if (last_phase[s] >= 0) mbar_drain(&full[s], (uint32_t)last_phase[s]);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ---- MMA issuer (leader CTA only)
      uint32_t it = 0, tcount = 0;
      bool ok = true, issued = false;
      for (int tile = cid; ok && tile < n_tiles; tile += ncl) {
        for (int st = 0; ok && st < S; ++st, ++tcount) {
          const uint32_t b = tcount & 1;
          if (!mbar_wait_pair(&acce[b], ((tcount >> 1) & 1) ^ 1, abort, peer_abort, &g_lowrank_error, 2, wl)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t tmem_d = tmem_base + b * kTile;
          for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
            const int s = it % kStages;
            if (!mbar_wait_pair(&full[s], (it / kStages) & 1, abort, peer_abort, &g_lowrank_error, 3, wl)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_u32(stage_base + s * kStageBytes);
            const uint32_t sb = sa + kStageA;
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              if (DT != ZT_F16)  // bf16 operands (bf16 splits for fp32 parameters)
                umma_bf16_pair<kIdescBf16>(tmem_d, umma_desc(sa + k * kUmmaK * 2),
                                                     umma_desc(sb + k * kUmmaK * 2), (kb | k) != 0);
              else
                umma_bf16_pair<kIdescF16>(tmem_d, umma_desc(sa + k * kUmmaK * 2),
                                                    umma_desc(sb + k * kUmmaK * 2), (kb | k) != 0);
            }
            issued = true;
            umma_commit_pair(&empty[s]);
          }
          if (!ok) break;
          umma_commit_pair(&accf[b]);
        }
      }
      if (issued) {
        umma_commit_pair_local(drain);
        mbar_drain(drain, 0);
      }
    }
  } else {  // ---- epilogue: warps 2..17 of both CTAs; a warp owns 32 rows x 64 columns
    const int ew = warp - 2;
    const int q = warp & 3;       // tensor-memory lane quadrant this warp may read
    const int quarter = ew >> 2;  // column quarter of the tile
    const int row_local = q * 32 + lane;
    const uint32_t leader_acce0 = peer_addr(&acce[0], 0), leader_acce1 = peer_addr(&acce[1], 0);
    const bool vec = P.vec != 0;
    uint32_t tcount = 0;
    bool ok = true;
    for (int tile = cid; ok && tile < n_tiles; tile += ncl) {
      int mt, nt;
      tile_coords(tile, P.m_tiles, P.n_tiles, mt, nt);
      const int row = mt * (int)kTile + (int)rank * (int)kHalfRows + row_local;
      const bool row_ok = row < P.m;
      for (int st = 0; st < S; ++st, ++tcount) {
        const uint32_t b = tcount & 1;
        const int colh = nt * (int)kTile + quarter * kWarpCols;
        // apply: the first batch of parameter / estimate rows is requested before the wait
        // for the accumulator (it needs none of it; a later stream of the same tile reads
        // what this thread stored for the previous one, after those stores)
        constexpr bool TH = MODE == kModeTheta || MODE == kModeBoth;
        constexpr bool GE = MODE == kModeGe || MODE == kModeBoth;
        constexpr int kLanesPerRow = kWarpCols / 8, kRowsPerStep = 32 / kLanesPerRow;
        constexpr int kSteps = 32 / kRowsPerStep;
        constexpr int kVW = DT == ZT_F32 ? 2 : 1;  // 16-byte words per 8 elements
        constexpr int kBatch = ((TH && GE) ? kSteps / 2 : kSteps) / kVW;  // row steps in flight per lane
        const bool init = P.ge_init && st == 0;
        const uint8_t* src = static_cast<const uint8_t*>(st == 0 ? P.src : P.dst);
        uint8_t* dstb = static_cast<uint8_t*>(P.dst);
        uint8_t* geb = static_cast<uint8_t*>(P.ge);
        const int rbase = mt * (int)kTile + (int)rank * (int)kHalfRows + q * 32;
        const int cg = (lane % kLanesPerRow) * 8;
        const int rsub = lane / kLanesPerRow;
        const int col = colh + cg;
        const bool col_ok = col < P.n;
        uint4 th[kBatch][kVW], gv[kBatch][kVW];
        auto load_batch = [&](int i0) {
#pragma unroll
          for (int i = 0; i < kBatch; ++i) {
            const int row = rbase + kRowsPerStep * (i0 + i) + rsub;
            if (row < P.m && col_ok) {
              const size_t off = ((size_t)row * P.n + col) * kEsz;
#pragma unroll
              for (int w = 0; w < kVW; ++w) {
                if (TH) th[i][w] = reinterpret_cast<const uint4*>(src + off)[w];
                if (GE && !init) gv[i][w] = reinterpret_cast<const uint4*>(geb + off)[w];
              }
            }
          }
        };
        if (MODE != kModeNorm && vec) load_batch(0);
        int okw = 1;
        if (lane == 0)
          okw = mbar_wait_pair(&accf[b], (tcount >> 1) & 1, abort, peer_abort, &g_lowrank_error, 4, wl) ? 1 : 0;
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) {
          ok = false;
          break;
        }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + b * kTile + (uint32_t)(quarter * kWarpCols);
        if (MODE == kModeNorm) {
          float ssq = 0.0f;
#pragma unroll 1
          for (int c = 0; c < kWarpCols / 32; ++c) {
            uint32_t acc[32];
            tmem_ld32(taddr + (uint32_t)(c * 32), acc);
            const int col0 = colh + c * 32;
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float z = H<DT>::round(__uint_as_float(acc[j]));
                if (col0 + j < P.n) ssq = __fmaf_rn(z, z, ssq);
              }
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
          if (lane == 0)
            P.partial[((size_t)tile * S + st) * kPartials + rank * kEpiWarps + ew] = ssq;
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(b ? leader_acce1 : leader_acce0);
        } else {
          // phase 1: the warp's 32 rows x 64 columns of zs into its staging rows, then the
          // accumulator buffer goes back to the MMA issuer
          uint8_t* zw = zstage + ew * kZWarp;
          const float sc = P.scale[st];
#pragma unroll 1
          for (int c = 0; c < kWarpCols / 32; ++c) {
            uint32_t acc[32];
            tmem_ld32(taddr + (uint32_t)(c * 32), acc);
            stage_chunk<DT>(acc, sc, reinterpret_cast<uint4*>(zw + lane * kZRow + c * 32 * kEsz));
          }
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(b ? leader_acce1 : leader_acce0);
          // phase 2: four rows per step, 8 lanes per row, 8 consecutive columns per lane
          // (coalesced 128- or 256-byte row segments)
          const float c = P.coef[st];
          if (vec) {
#pragma unroll 1
            for (int i0 = 0; i0 < kSteps; i0 += kBatch) {
              if (i0 > 0) load_batch(i0);
#pragma unroll
              for (int i = 0; i < kBatch; ++i) {
                const int rl = kRowsPerStep * (i0 + i) + rsub;
                const int row = rbase + rl;
                if (row < P.m && col_ok) {
                  uint4 zs[kVW];
#pragma unroll
                  for (int w = 0; w < kVW; ++w) zs[w] = reinterpret_cast<const uint4*>(zw + rl * kZRow + cg * kEsz)[w];
                  const size_t off = ((size_t)row * P.n + col) * kEsz;
                  apply8v<DT, TH, GE>(th[i], gv[i], zs, P, c, init);
#pragma unroll
                  for (int w = 0; w < kVW; ++w) {
                    if (TH) reinterpret_cast<uint4*>(dstb + off)[w] = th[i][w];
                    if (GE) reinterpret_cast<uint4*>(geb + off)[w] = gv[i][w];
                  }
                }
              }
            }
          } else {
#pragma unroll 1
            for (int i = 0; i < kSteps; ++i) {
              const int rl = kRowsPerStep * i + rsub;
              const int row = rbase + rl;
              if (row >= P.m || !col_ok) continue;
              const uint8_t* zrow = zw + rl * kZRow + cg * kEsz;
              const size_t roff = (size_t)row * P.n * kEsz;
              apply_scalar8<DT>(TH ? src + roff : nullptr, TH ? dstb + roff : nullptr, GE ? geb + roff : nullptr, col,
                                zrow, P, c, init);
            }
          }
          __syncwarp();  // every lane has read the staging rows before the next item rewrites them
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
}

// Scale of stream blockIdx.x from its partial sums of squares, in torch's op order on the
// parameter dtype: norm = round(sqrt(ss)), den = round(norm + 1e-7), rec = round(1 / den),
// scale = round(rec * sqrt(m n)). The sum runs in double in a fixed order.
template <int DT>
__global__ void __launch_bounds__(256) lr_scale_kernel(const float* __restrict__ partial, int32_t tiles, int32_t S,
                                                       float sqrt_numel, float* __restrict__ scale) {
  __shared__ double red[256];
  const int s = blockIdx.x;
  double acc = 0.0;
  const int64_t count = (int64_t)tiles * kPartials;
  for (int64_t t = threadIdx.x; t < count; t += 256) {
    const int64_t tile = t / kPartials, k = t - tile * kPartials;
    acc += (double)partial[((size_t)tile * S + s) * kPartials + k];
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float ss = (float)red[0];
    const float nrm = H<DT>::round(__fsqrt_rn(ss));
    const float den = H<DT>::round(__fadd_rn(nrm, 1e-7f));
    const float rec = H<DT>::round(__fdiv_rn(1.0f, den));
    scale[s] = H<DT>::round(__fmul_rn(rec, sqrt_numel));
  }
}

// ---- apply with the parameter slice resident in shared memory ---------------------------
//
// For parameters whose rows are whole 16-byte groups at 16-byte aligned addresses. Each
// CTA's 128 x 256 slice of a tile (of the parameter, the grad estimate, or both) comes in
// by TMA one tile ahead of its use. Every stream of the tile is applied to it in shared
// memory, and one TMA store writes it back: HBM sees the parameter once per tile whatever
// the stream count, and the copies run on the TMA engine instead of the epilogue warps.
// The slice is held in the 128-byte-swizzled layout the tile maps use: 16-byte chunk c of
// row r at r * 128 + ((c ^ (r & 7)) << 4) inside each 64-column box.
constexpr int kTStages = 2;
constexpr uint32_t kBoxBytes = 128 * 128;        // 64 columns x 128 rows of 16-bit values
constexpr uint32_t kSliceBytes = 4 * kBoxBytes;  // a CTA's 128 x 256 slice of a tile
constexpr size_t kSmemT = 1024 + kTStages * kStageBytes + 2 * kSliceBytes + 256;

struct LrTileParams {
  CUtensorMap tmap_a;    // stacked P    [S m, kp], box {64, 128}
  CUtensorMap tmap_b;    // stacked Psi^T [S n, kp], box {64, 128}
  CUtensorMap tmap_src;  // parameter read   [m, n], box {64, 128}, 128-byte swizzle
  CUtensorMap tmap_dst;  // parameter written
  CUtensorMap tmap_ge;   // grad estimate (read unless ge_init, written)
  const float* scale;
  float alpha[3];
  int32_t n_alpha;
  int32_t ge_init;
  int32_t m, n, k_blocks, m_tiles, n_tiles, n_streams;
  int32_t stall_loads;
  long long wait_cycles;
  float coef[ZT_LOWRANK_MAX_STREAMS];
};

template <int DT, int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    lr_tile_kernel(const __grid_constant__ LrTileParams P) {
  constexpr bool TH = MODE == kModeTheta || MODE == kModeBoth;
  constexpr bool GE = MODE == kModeGe || MODE == kModeBoth;
  constexpr int kBufs = (TH && GE) ? 1 : 2;  // slices in flight: two, or one of each kind
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint8_t* slices = smem + kTStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(slices + 2 * kSliceBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kTStages;
  uint64_t* accf = bars + 2 * kTStages;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint64_t* tfull = drain + 1;
  uint64_t* tempty = tfull + 2;
  uint64_t* tdone = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tdone + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 2 * kEpiWarps);
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 1);
      mbar_init(&tdone[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t peer_abort = peer_addr((const void*)abort, rank ^ 1u);
  const long long wl = P.wait_cycles;

  const int n_tiles = P.m_tiles * P.n_tiles;
  const int S = P.n_streams;
  const int cid = (int)cluster_id_x(), ncl = (int)n_clusters_x();
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs): the tile's slice, then every stream's K blocks
      int last_phase[kTStages];
      for (int s = 0; s < kTStages; ++s) last_phase[s] = -1;
      int slice_phase[2] = {-1, -1};
      uint32_t it = 0;
      bool ok = true;
      int ti = 0;
      for (int tile = cid; ok && tile < n_tiles; tile += ncl, ++ti) {
        int mt, nt;
        tile_coords(tile, P.m_tiles, P.n_tiles, mt, nt);
        const int tb = kBufs == 2 ? (ti & 1) : 0;
        const uint32_t u = kBufs == 2 ? (uint32_t)(ti >> 1) : (uint32_t)ti;
        if (!mbar_wait_pair(&tempty[tb], (u & 1) ^ 1, abort, peer_abort, &g_lowrank_error, 5, wl)) break;
        uint8_t* th_buf = slices + (kBufs == 2 ? tb * kSliceBytes : 0);
        uint8_t* ge_buf = kBufs == 2 ? th_buf : slices + kSliceBytes;
        const bool load_ge = GE && !P.ge_init;
        const uint32_t bytes = (TH ? kSliceBytes : 0u) + (load_ge ? kSliceBytes : 0u);
        const int x0 = nt * (int)kTile, y0 = mt * (int)kTile + (int)rank * (int)kHalfRows;
        if (bytes) {
          mbar_expect_tx(&tfull[tb], bytes);
#pragma unroll
          for (int box = 0; box < 4; ++box) {
            if (TH) tma_load_2d(th_buf + box * kBoxBytes, &P.tmap_src, &tfull[tb], x0 + box * 64, y0);
            if (load_ge) tma_load_2d(ge_buf + box * kBoxBytes, &P.tmap_ge, &tfull[tb], x0 + box * 64, y0);
          }
          slice_phase[tb] = (int)(u & 1);
        } else {
          mbar_arrive(&tfull[tb]);
        }
        for (int st = 0; ok && st < S; ++st) {
          for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
            const int s = it % kTStages;
            const uint32_t round = it / kTStages;
            if (!mbar_wait_pair(&empty[s], (round & 1) ^ 1, abort, peer_abort, &g_lowrank_error, 1, wl)) {
              ok = false;
              break;
            }
            if (P.stall_loads) continue;
            uint8_t* sa = stage_base + s * kStageBytes;
            const uint32_t leader_full = peer_addr(&full[s], 0);
            if (leader) mbar_expect_tx(&full[s], 2 * kStageBytes);
            tma_load_2d_pair(sa, &P.tmap_a, leader_full, kb * kBK,
                             st * P.m + mt * (int)kTile + (int)rank * (int)kHalfRows);
            tma_load_2d_pair(sa + kStageA, &P.tmap_b, leader_full, kb * kBK,
                             st * P.n + nt * (int)kTile + (int)rank * (int)kHalfRows);
            last_phase[s] = (int)(round & 1);
          }
        }
      }
      for (int b = 0; b < 2; ++b)
        if (slice_phase[b] >= 0) mbar_drain(&tfull[b], (uint32_t)slice_phase[b]);
      if (leader)
        for (int s = 0; s < kTStages; ++s)
          if (last_phase[s] >= 0) mbar_drain(&full[s], (uint32_t)last_phase[s]);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ---- MMA issuer (leader CTA only)
      uint32_t it = 0, tcount = 0;
      bool ok = true, issued = false;
      for (int tile = cid; ok && tile < n_tiles; tile += ncl) {
        for (int st = 0; ok && st < S; ++st, ++tcount) {
          const uint32_t b = tcount & 1;
          if (!mbar_wait_pair(&acce[b], ((tcount >> 1) & 1) ^ 1, abort, peer_abort, &g_lowrank_error, 2, wl)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t tmem_d = tmem_base + b * kTile;
          for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
            const int s = it % kTStages;
            if (!mbar_wait_pair(&full[s], (it / kTStages) & 1, abort, peer_abort, &g_lowrank_error, 3, wl)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_u32(stage_base + s * kStageBytes);
            const uint32_t sb = sa + kStageA;
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              if (DT == ZT_BF16)
                umma_bf16_pair<kIdescBf16>(tmem_d, umma_desc(sa + k * kUmmaK * 2), umma_desc(sb + k * kUmmaK * 2),
                                           (kb | k) != 0);
              else
                umma_bf16_pair<kIdescF16>(tmem_d, umma_desc(sa + k * kUmmaK * 2), umma_desc(sb + k * kUmmaK * 2),
                                          (kb | k) != 0);
            }
            issued = true;
            umma_commit_pair(&empty[s]);
          }
          if (!ok) break;
          umma_commit_pair(&accf[b]);
        }
      }
      if (issued) {
        umma_commit_pair_local(drain);
        mbar_drain(drain, 0);
      }
    }
  } else {  // ---- epilogue: warps 2..17 of both CTAs; a warp owns 32 rows x 64 columns (one box)
    const int ew = warp - 2;
    const int q = warp & 3;
    const int quarter = ew >> 2;
    const int r = q * 32 + lane;  // row of the CTA's slice = tensor-memory lane
    const uint32_t leader_acce0 = peer_addr(&acce[0], 0), leader_acce1 = peer_addr(&acce[1], 0);
    uint32_t tcount = 0;
    bool ok = true;
    int ti = 0;
    for (int tile = cid; ok && tile < n_tiles; tile += ncl, ++ti) {
      int mt, nt;
      tile_coords(tile, P.m_tiles, P.n_tiles, mt, nt);
      const int tb = kBufs == 2 ? (ti & 1) : 0;
      const uint32_t u = kBufs == 2 ? (uint32_t)(ti >> 1) : (uint32_t)ti;
      uint8_t* th_buf = slices + (kBufs == 2 ? tb * kSliceBytes : 0);
      uint8_t* ge_buf = kBufs == 2 ? th_buf : slices + kSliceBytes;
      int okw = 1;
      if (lane == 0) okw = mbar_wait_pair(&tfull[tb], u & 1, abort, peer_abort, &g_lowrank_error, 6, wl) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) break;
      uint8_t* th_row = th_buf + quarter * kBoxBytes + r * 128;
      uint8_t* ge_row = ge_buf + quarter * kBoxBytes + r * 128;
      for (int st = 0; st < S; ++st, ++tcount) {
        const uint32_t b = tcount & 1;
        okw = 1;
        if (lane == 0)
          okw = mbar_wait_pair(&accf[b], (tcount >> 1) & 1, abort, peer_abort, &g_lowrank_error, 4, wl) ? 1 : 0;
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) {
          ok = false;
          break;
        }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + b * kTile + (uint32_t)(quarter * 64);
        const float sc = P.scale[st];
        const float c = P.coef[st];
        const bool init = P.ge_init && st == 0;
#pragma unroll 1
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t acc[32];
          tmem_ld32(taddr + (uint32_t)(c2 * 32), acc);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int off = ((c2 * 4 + k) ^ (r & 7)) << 4;
            uint32_t zw[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              float za = __uint_as_float(acc[8 * k + 2 * w]), zb = __uint_as_float(acc[8 * k + 2 * w + 1]);
              H<DT>::round2(za, zb);
              zw[w] = H<DT>::pack(__fmul_rn(za, sc), __fmul_rn(zb, sc));
            }
            uint4 tv = make_uint4(0u, 0u, 0u, 0u), gv = make_uint4(0u, 0u, 0u, 0u);
            if (TH) tv = *reinterpret_cast<const uint4*>(th_row + off);
            if (GE && !init) gv = *reinterpret_cast<const uint4*>(ge_row + off);
            apply8<DT, TH, GE>(tv, gv, make_uint4(zw[0], zw[1], zw[2], zw[3]), P, c, init);
            if (TH) *reinterpret_cast<uint4*>(th_row + off) = tv;
            if (GE) *reinterpret_cast<uint4*>(ge_row + off) = gv;
          }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(b ? leader_acce1 : leader_acce0);
      }
      if (!ok) break;
      // the slice is complete: every warp's writes made visible to the TMA engine, then
      // one thread stores it once all sixteen warps have arrived
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&tdone[tb]);
      if (ew == 0 && lane == 0) {
        if (!mbar_wait_pair(&tdone[tb], u & 1, abort, peer_abort, &g_lowrank_error, 7, wl)) {
          ok = false;
        } else {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          const int x0 = nt * (int)kTile, y0 = mt * (int)kTile + (int)rank * (int)kHalfRows;
#pragma unroll
          for (int box = 0; box < 4; ++box) {
            if (TH) tma_store_2d(&P.tmap_dst, th_buf + box * kBoxBytes, x0 + box * 64, y0);
            if (GE) tma_store_2d(&P.tmap_ge, ge_buf + box * kBoxBytes, x0 + box * 64, y0);
          }
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          mbar_arrive(&tempty[tb]);
        }
      }
      okw = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0);
      if (!okw) break;
    }
    if (ew == 0 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
}

// ---- host side ----------------------------------------------------------------------------

// CTA pairs of `kern` that fit on the GPU at once (cached per device and kernel).
template <typename Kern>
int pairs_for(Kern kern, size_t smem, int (&cache)[64], int* pairs) {
  static std::mutex mu;
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "zt_lowrank: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return zt::set_error(ZT_ERR_LIMIT, "zt_lowrank: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] <= 0) {
    if (int rc = zt::check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "zt_lowrank: shared memory attribute"))
      return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)(zt::sm_count() / 2));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (int rc = zt::check_cuda(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "zt_lowrank: cudaOccupancyMaxActiveClusters"))
      return rc;
    if (n <= 0) return zt::set_error(ZT_ERR_CUDA, "zt_lowrank: no CTA pair fits on this GPU");
    cache[dev] = n;
  }
  *pairs = cache[dev];
  return ZT_OK;
}

template <int DT, int MODE>
int prepare_gemm(int* pairs) {
  static int cache[64] = {0};
  return pairs_for(lr_gemm_kernel<DT, MODE>, Cfg<DT>::kSmem, cache, pairs);
}

int64_t tiles_of(int64_t m, int64_t n) { return ((m + kTile - 1) / kTile) * ((n + kTile - 1) / kTile); }

int check_desc(const zt_lowrank_desc* d, const char* who) {
  if (!d) return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": null descriptor");
  if (d->m <= 0 || d->n <= 0) return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": m and n must be positive");
  if (d->dtype != ZT_BF16 && d->dtype != ZT_F16 && d->dtype != ZT_F32)
    return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": dtype must be ZT_BF16, ZT_F16 or ZT_F32");
  if (d->kp <= 0 || d->kp % kBK || d->kp > 1024)
    return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": kp must be a positive multiple of 64, at most 1024");
  if (d->r < 1 || d->r > d->kp || d->r > d->m)
    return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": need 1 <= r <= min(kp, m)");
  if (d->dtype == ZT_F32 && !d->factors_given && d->kp < 9 * d->r)
    return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": fp32 factors from the noise source need kp >= 9 r");
  if (d->n_streams < 1 || d->n_streams > ZT_LOWRANK_MAX_STREAMS)
    return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": n_streams must be in [1, ZT_LOWRANK_MAX_STREAMS]");
  const int64_t S = d->n_streams;
  if (d->m * d->r > (int64_t)INT32_MAX || d->n * d->r > (int64_t)INT32_MAX || S * d->m > (int64_t)INT32_MAX - 512 ||
      S * d->n > (int64_t)INT32_MAX - 512 || d->m * d->n > ((int64_t)1 << 40))
    return zt::set_error(ZT_ERR_LIMIT, std::string(who) + ": factor or parameter size above the 32-bit offsets");
  if (!d->p || !d->psi_t || !d->scale) return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": null buffer");
  if (((uintptr_t)d->p & 15) || ((uintptr_t)d->psi_t & 15) || ((uintptr_t)d->scale & 3))
    return zt::set_error(ZT_ERR_INVALID, std::string(who) + ": factor buffers must be 16-byte aligned");
  return ZT_OK;
}

template <int DT, int MODE>
int launch_gemm(const zt_lowrank_desc* d, LrParams& P, cudaStream_t st, const char* who) {
  int pairs = 0;
  if (int rc = prepare_gemm<DT, MODE>(&pairs)) return rc;
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc, who)) return rc;
  const uint64_t S = (uint64_t)d->n_streams;
  if (int rc = make_map_bf16(enc, &P.tmap_a, d->p, S * (uint64_t)d->m, (uint64_t)d->kp, kHalfRows, who)) return rc;
  if (int rc = make_map_bf16(enc, &P.tmap_b, d->psi_t, S * (uint64_t)d->n, (uint64_t)d->kp, kHalfRows, who)) return rc;
  P.m = (int32_t)d->m;
  P.n = (int32_t)d->n;
  P.k_blocks = d->kp / kBK;
  P.m_tiles = (int32_t)((d->m + kTile - 1) / kTile);
  P.n_tiles = (int32_t)((d->n + kTile - 1) / kTile);
  P.n_streams = d->n_streams;
  P.scale = d->scale;
  const int64_t tiles = (int64_t)P.m_tiles * P.n_tiles;
  const int clusters = tiles < pairs ? (int)tiles : pairs;
  lr_gemm_kernel<DT, MODE><<<2 * clusters, kThreads, Cfg<DT>::kSmem, st>>>(P);
  return zt::check_cuda(cudaGetLastError(), (std::string(who) + ": launch").c_str());
}

template <int DT, int MODE>
int launch_tile(const zt_lowrank_desc* d, const zt_lowrank_apply_args* a, cudaStream_t st) {
  const char* who = "zt_lowrank_apply";
  static int cache[64] = {0};
  int pairs = 0;
  if (int rc = pairs_for(lr_tile_kernel<DT, MODE>, kSmemT, cache, &pairs)) return rc;
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc, who)) return rc;
  LrTileParams P;
  memset(&P, 0, sizeof(P));
  const uint64_t S = (uint64_t)d->n_streams, m = (uint64_t)d->m, n = (uint64_t)d->n;
  if (int rc = make_map_bf16(enc, &P.tmap_a, d->p, S * m, (uint64_t)d->kp, kHalfRows, who)) return rc;
  if (int rc = make_map_bf16(enc, &P.tmap_b, d->psi_t, S * n, (uint64_t)d->kp, kHalfRows, who)) return rc;
  if (a->dst) {
    if (int rc = make_map_bf16(enc, &P.tmap_src, a->src, m, n, kHalfRows, who)) return rc;
    if (int rc = make_map_bf16(enc, &P.tmap_dst, a->dst, m, n, kHalfRows, who)) return rc;
  }
  if (a->ge)
    if (int rc = make_map_bf16(enc, &P.tmap_ge, a->ge, m, n, kHalfRows, who)) return rc;
  P.scale = d->scale;
  P.n_alpha = a->n_alpha;
  for (int i = 0; i < 3; ++i) P.alpha[i] = a->alpha[i];
  P.ge_init = a->ge_init ? 1 : 0;
  for (int s = 0; s < d->n_streams; ++s) P.coef[s] = a->coef[s];
  P.m = (int32_t)d->m;
  P.n = (int32_t)d->n;
  P.k_blocks = d->kp / kBK;
  P.m_tiles = (int32_t)((d->m + kTile - 1) / kTile);
  P.n_tiles = (int32_t)((d->n + kTile - 1) / kTile);
  P.n_streams = d->n_streams;
  P.stall_loads = a->test_stall_loads ? 1 : 0;
  P.wait_cycles = a->test_wait_cycles > 0 ? (long long)a->test_wait_cycles : kWaitCycles;
  const int64_t tiles = (int64_t)P.m_tiles * P.n_tiles;
  const int clusters = tiles < pairs ? (int)tiles : pairs;
  lr_tile_kernel<DT, MODE><<<2 * clusters, kThreads, kSmemT, st>>>(P);
  return zt::check_cuda(cudaGetLastError(), "zt_lowrank_apply: launch");
}

template <int DT>
int prepare_impl(const zt_lowrank_desc* d, cudaStream_t st) {
  const char* who = "zt_lowrank_prepare";
  FactorKeys K;
  for (int s = 0; s < d->n_streams; ++s) {
    K.p[s] = d->keys_p[s];
    K.psi[s] = d->keys_psi[s];
  }
  if (!d->factors_given) {
    const int64_t total = (int64_t)d->n_streams * (d->m + d->n) * (d->kp / 8);
    const int64_t want = (total + 255) / 256, cap = (int64_t)zt::sm_count() * 16;
    lr_factor_kernel<DT><<<(unsigned)(want < cap ? want : cap), 256, 0, st>>>(
        K, static_cast<uint16_t*>(d->p), static_cast<uint16_t*>(d->psi_t), d->n_streams, (int32_t)d->m,
        (int32_t)d->n, d->r, d->kp);
    if (int rc = zt::check_cuda(cudaGetLastError(), "zt_lowrank_prepare: factor launch")) return rc;
  }
  LrParams P;
  memset(&P, 0, sizeof(P));
  P.partial = static_cast<float*>(d->workspace);
  P.wait_cycles = kWaitCycles;
  if (int rc = launch_gemm<DT, kModeNorm>(d, P, st, who)) return rc;
  lr_scale_kernel<DT><<<(unsigned)d->n_streams, 256, 0, st>>>(P.partial, (int32_t)tiles_of(d->m, d->n), d->n_streams,
                                                              (float)std::sqrt((double)d->m * (double)d->n), d->scale);
  return zt::check_cuda(cudaGetLastError(), "zt_lowrank_prepare: scale launch");
}

}  // namespace

extern "C" {

int zt_lowrank_workspace_bytes(int64_t m, int64_t n, int32_t n_streams, size_t* bytes) {
  zt::clear_error();
  if (!bytes) return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_workspace_bytes: null pointer");
  if (m <= 0 || n <= 0 || n_streams < 1 || n_streams > ZT_LOWRANK_MAX_STREAMS)
    return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_workspace_bytes: bad shape or stream count");
  *bytes = (size_t)tiles_of(m, n) * (size_t)n_streams * kPartials * sizeof(float);
  return ZT_OK;
}

int zt_lowrank_prepare(const zt_lowrank_desc* d, void* stream) {
  zt::clear_error();
  if (int rc = check_desc(d, "zt_lowrank_prepare")) return rc;
  size_t need = 0;
  if (int rc = zt_lowrank_workspace_bytes(d->m, d->n, d->n_streams, &need)) return rc;
  if (!d->workspace || d->workspace_bytes < need || ((uintptr_t)d->workspace & 15))
    return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_prepare: workspace missing, misaligned or below "
                                         "zt_lowrank_workspace_bytes");
  const cudaStream_t st = zt::as_stream(stream);
  return d->dtype == ZT_BF16 ? prepare_impl<ZT_BF16>(d, st)
         : d->dtype == ZT_F16 ? prepare_impl<ZT_F16>(d, st)
                              : prepare_impl<ZT_F32>(d, st);
}

int zt_lowrank_apply(const zt_lowrank_desc* d, const zt_lowrank_apply_args* a, void* stream) {
  zt::clear_error();
  const char* who = "zt_lowrank_apply";
  if (int rc = check_desc(d, who)) return rc;
  if (!a) return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: null arguments");
  if (a->n_alpha < 0 || a->n_alpha > 3) return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: n_alpha must be 0..3");
  if (a->n_alpha > 0 && (!a->dst || !a->src))
    return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: coefficients given without src and dst");
  if (a->n_alpha == 0 && a->dst)
    return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: dst given without coefficients");
  if (!a->dst && !a->ge) return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: nothing to write");
  const size_t esz = d->dtype == ZT_F32 ? 4 : 2;
  const size_t bytes = (size_t)d->m * (size_t)d->n * esz;
  if (a->src && a->dst && a->src != a->dst) {
    const uintptr_t s0 = (uintptr_t)a->src, d0 = (uintptr_t)a->dst;
    if (s0 < d0 + bytes && d0 < s0 + bytes)
      return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: src and dst overlap without being equal");
  }
  if (a->ge && a->dst) {
    const uintptr_t g0 = (uintptr_t)a->ge, d0 = (uintptr_t)a->dst;
    if (g0 < d0 + bytes && d0 < g0 + bytes) return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: ge overlaps dst");
  }
  for (const void* p : {a->src, (const void*)a->dst, (const void*)a->ge})
    if (((uintptr_t)p & (esz - 1)) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_apply: misaligned parameter buffer");
  LrParams P;
  memset(&P, 0, sizeof(P));
  P.src = a->src;
  P.dst = a->dst;
  P.ge = a->ge;
  P.n_alpha = a->n_alpha;
  for (int i = 0; i < 3; ++i) P.alpha[i] = a->alpha[i];
  P.ge_init = a->ge_init ? 1 : 0;
  for (int s = 0; s < d->n_streams; ++s) P.coef[s] = a->coef[s];
  bool vec = d->n % 8 == 0;
  for (const void* p : {a->src, (const void*)a->dst, (const void*)a->ge})
    if (((uintptr_t)p & 15) != 0) vec = false;
  P.vec = vec ? 1 : 0;
  P.stall_loads = a->test_stall_loads ? 1 : 0;
  P.wait_cycles = a->test_wait_cycles > 0 ? (long long)a->test_wait_cycles : kWaitCycles;
  const cudaStream_t st = zt::as_stream(stream);
  const bool th = a->dst != nullptr, ge = a->ge != nullptr;
  if (d->dtype == ZT_F32)
    return th && ge ? launch_gemm<ZT_F32, kModeBoth>(d, P, st, who)
           : th     ? launch_gemm<ZT_F32, kModeTheta>(d, P, st, who)
                    : launch_gemm<ZT_F32, kModeGe>(d, P, st, who);
  if (vec) {  // whole 16-byte row groups at aligned addresses: the slice-resident kernel
    if (d->dtype == ZT_BF16)
      return th && ge ? launch_tile<ZT_BF16, kModeBoth>(d, a, st)
             : th     ? launch_tile<ZT_BF16, kModeTheta>(d, a, st)
                      : launch_tile<ZT_BF16, kModeGe>(d, a, st);
    return th && ge ? launch_tile<ZT_F16, kModeBoth>(d, a, st)
           : th     ? launch_tile<ZT_F16, kModeTheta>(d, a, st)
                    : launch_tile<ZT_F16, kModeGe>(d, a, st);
  }
  if (d->dtype == ZT_BF16)
    return th && ge ? launch_gemm<ZT_BF16, kModeBoth>(d, P, st, who)
           : th     ? launch_gemm<ZT_BF16, kModeTheta>(d, P, st, who)
                    : launch_gemm<ZT_BF16, kModeGe>(d, P, st, who);
  return th && ge ? launch_gemm<ZT_F16, kModeBoth>(d, P, st, who)
         : th     ? launch_gemm<ZT_F16, kModeTheta>(d, P, st, who)
                  : launch_gemm<ZT_F16, kModeGe>(d, P, st, who);
}

int zt_lowrank_take_error(int32_t* code) {
  zt::clear_error();
  if (!code) return zt::set_error(ZT_ERR_INVALID, "zt_lowrank_take_error: null pointer");
  int v = 0;
  if (int rc = zt::check_cuda(cudaMemcpyFromSymbol(&v, g_lowrank_error, sizeof(int)), "zt_lowrank_take_error: read"))
    return rc;
  const int zero = 0;
  if (int rc = zt::check_cuda(cudaMemcpyToSymbol(g_lowrank_error, &zero, sizeof(int)), "zt_lowrank_take_error: clear"))
    return rc;
  *code = v;
  return ZT_OK;
}

}  // extern "C"
