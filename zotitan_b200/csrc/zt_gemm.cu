// W <- bf16(W + alpha * A B^T) on the tensor cores, W read and written in the epilogue.
//
// The update of the evolution-strategies step: for a 2-D weight W [m, n] and p pairs,
// sum_j coef_j c_j P_j Psi_j is one GEMM of inner dimension 8p over the packed operands of
// zt_eggroll_update_operands (A [m, 8p], B [n, 8p], both bf16 K-major), and the step adds
// -lr times it to W with one rounding. CTA pairs (tcgen05.mma.cta_group::2) compute
// 256 x 256 tiles with fp32 accumulators double-buffered in tensor memory; the epilogue
// thread that owns a row reads 32 bf16 of W at a time (four 16-byte loads), adds
// alpha * acc in fp32 (one fused multiply-add) and writes the bf16 rounding back, so W is
// read and written once and the product never reaches HBM. Every mbarrier wait is bounded;
// on expiry the kernel records an error (zt_gemm_take_error), drains its own copies and
// MMAs and frees its tensor memory.
#include "zt_tc.cuh"

namespace {

using namespace zt::tc;

constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA (leader), warps 2-5 epilogue
constexpr int kStages = 6;
constexpr uint32_t kHalfRows = 128;
constexpr uint32_t kStageA = kHalfRows * kBK * 2;
constexpr uint32_t kStageBytes = 2 * kStageA;
constexpr uint32_t kTile = 256;
constexpr uint32_t kTmemCols = 2 * kTile;
constexpr size_t kSmem = 1024 + kStages * kStageBytes + 256;
constexpr uint32_t kIdesc = idesc_bf16(256, 256);
constexpr int kGroupN = 16;  // N-blocks per rasterisation group (A rows and B slice stay in L2)

__device__ int g_gemm_error = 0;

struct AddtoParams {
  CUtensorMap tmap_a;  // A [m, k], box {64, 128}
  CUtensorMap tmap_b;  // B [n, k], box {64, 128}
  __nv_bfloat16* w;    // [m, n], row stride ldw elements
  int64_t ldw;
  float alpha;
  int32_t m, n, k_blocks, m_tiles, n_tiles;
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

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_addto_kernel(const __grid_constant__ AddtoParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
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
    for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], 2 * 4); }
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

  const int n_tiles = P.m_tiles * P.n_tiles;
  const int cid = (int)cluster_id_x(), ncl = (int)n_clusters_x();
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs)
      int last_phase[kStages];
      for (int s = 0; s < kStages; ++s) last_phase[s] = -1;
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < n_tiles; tile += ncl) {
        int mt, nt;
        tile_coords(tile, P.m_tiles, P.n_tiles, mt, nt);
        for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t round = it / kStages;
          if (!mbar_wait_pair(&empty[s], (round & 1) ^ 1, abort, peer_abort, &g_gemm_error, 1)) { ok = false; break; }
          uint8_t* sa = stage_base + s * kStageBytes;
          const uint32_t leader_full = peer_addr(&full[s], 0);
          if (leader) mbar_expect_tx(&full[s], 2 * kStageBytes);
          tma_load_2d_pair(sa, &P.tmap_a, leader_full, kb * kBK, mt * (int)kTile + (int)rank * (int)kHalfRows);
          tma_load_2d_pair(sa + kStageA, &P.tmap_b, leader_full, kb * kBK, nt * (int)kTile + (int)rank * (int)kHalfRows);
          last_phase[s] = (int)(round & 1);
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
      for (int tile = cid; ok && tile < n_tiles; tile += ncl, ++tcount) {
        const uint32_t b = tcount & 1;
        if (!mbar_wait_pair(&acce[b], ((tcount >> 1) & 1) ^ 1, abort, peer_abort, &g_gemm_error, 2)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tmem_d = tmem_base + b * kTile;
        for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait_pair(&full[s], (it / kStages) & 1, abort, peer_abort, &g_gemm_error, 3)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = smem_u32(stage_base + s * kStageBytes);
          const uint32_t sb = sa + kStageA;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k)
            umma_bf16_pair<kIdesc>(tmem_d, umma_desc(sa + k * kUmmaK * 2), umma_desc(sb + k * kUmmaK * 2),
                                   (kb | k) != 0);
          issued = true;
          umma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair(&accf[b]);
      }
      if (issued) {
        umma_commit_pair_local(drain);
        mbar_drain(drain, 0);
      }
    }
  } else {  // ---- epilogue: warps 2..5 of both CTAs; each thread owns one accumulator row
    const int q = warp & 3;
    const int row_local = q * 32 + lane;
    const uint32_t leader_acce0 = peer_addr(&acce[0], 0), leader_acce1 = peer_addr(&acce[1], 0);
    uint32_t tcount = 0;
    for (int tile = cid; tile < n_tiles; tile += ncl, ++tcount) {
      int mt, nt;
      tile_coords(tile, P.m_tiles, P.n_tiles, mt, nt);
      const uint32_t b = tcount & 1;
      const int row = mt * (int)kTile + (int)rank * (int)kHalfRows + row_local;
      int okw = 1;
      if (lane == 0) okw = mbar_wait_pair(&accf[b], (tcount >> 1) & 1, abort, peer_abort, &g_gemm_error, 4) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) break;
      __syncwarp();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      __nv_bfloat16* wrow = P.w + (size_t)row * (size_t)P.ldw;
      for (int c0 = 0; c0 < (int)kTile; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + b * kTile + (uint32_t)c0, r);
        const int col0 = nt * (int)kTile + c0;
        if (row < P.m && col0 < P.n) {  // n % 32 == 0: a chunk is wholly inside or outside
          uint4* wp = reinterpret_cast<uint4*>(wrow + col0);
          uint4 v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = wp[i];
          uint32_t* words = reinterpret_cast<uint32_t*>(v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float lo = __uint_as_float(words[j] << 16), hi = __uint_as_float(words[j] & 0xffff0000u);
            const __nv_bfloat162 h = __floats2bfloat162_rn(__fmaf_rn(P.alpha, __uint_as_float(r[2 * j]), lo),
                                                           __fmaf_rn(P.alpha, __uint_as_float(r[2 * j + 1]), hi));
            words[j] = *reinterpret_cast<const uint32_t*>(&h);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) wp[i] = v[i];
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(b ? leader_acce1 : leader_acce0);
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

int g_max_pairs[64] = {0};

int prepare(int* pairs) {
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "zt_gemm_addto: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return zt::set_error(ZT_ERR_LIMIT, "zt_gemm_addto: device ordinal >= 64");
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (g_max_pairs[dev] <= 0) {
    if (int rc = zt::check_cuda(cudaFuncSetAttribute(gemm_addto_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)kSmem), "zt_gemm_addto: shared memory attribute"))
      return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)(zt::sm_count() / 2));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    int n = 0;
    if (int rc = zt::check_cuda(cudaOccupancyMaxActiveClusters(&n, gemm_addto_kernel, &cfg),
                                "zt_gemm_addto: cudaOccupancyMaxActiveClusters"))
      return rc;
    if (n <= 0) return zt::set_error(ZT_ERR_CUDA, "zt_gemm_addto: no CTA pair fits on this GPU");
    g_max_pairs[dev] = n;
  }
  *pairs = g_max_pairs[dev];
  return ZT_OK;
}

}  // namespace

extern "C" {

int zt_gemm_addto(void* w, int64_t ldw, const void* a, const void* b, float alpha, int64_t m, int64_t n, int64_t k,
                  void* stream) {
  zt::clear_error();
  if (!w || !a || !b) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_addto: null pointer");
  if (m <= 0 || n <= 0 || k <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_addto: m, n and k must be positive");
  if (n % 32 || k % kBK) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_addto: need n % 32 == 0 and k % 64 == 0");
  if (ldw < n || ldw % 8) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_addto: ldw must be >= n and a multiple of 8");
  if (m > (int64_t)INT32_MAX - 256 || n > (int64_t)INT32_MAX - 256 || k > (int64_t)INT32_MAX)
    return zt::set_error(ZT_ERR_LIMIT, "zt_gemm_addto: dimension above 2^31 - 257");
  for (const void* p : {(const void*)w, a, b})
    if (((uintptr_t)p & 15) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_addto: pointers must be 16-byte aligned");
  int pairs = 0;
  if (int rc = prepare(&pairs)) return rc;
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc, "zt_gemm_addto")) return rc;
  AddtoParams P;
  if (int rc = make_map_bf16(enc, &P.tmap_a, a, (uint64_t)m, (uint64_t)k, kHalfRows, "zt_gemm_addto")) return rc;
  if (int rc = make_map_bf16(enc, &P.tmap_b, b, (uint64_t)n, (uint64_t)k, kHalfRows, "zt_gemm_addto")) return rc;
  P.w = static_cast<__nv_bfloat16*>(w);
  P.ldw = ldw;
  P.alpha = alpha;
  P.m = (int32_t)m;
  P.n = (int32_t)n;
  P.k_blocks = (int32_t)(k / kBK);
  P.m_tiles = (int32_t)((m + kTile - 1) / kTile);
  P.n_tiles = (int32_t)((n + kTile - 1) / kTile);
  const int tiles = P.m_tiles * P.n_tiles;
  const int clusters = tiles < pairs ? tiles : pairs;
  gemm_addto_kernel<<<2 * clusters, kThreads, kSmem, zt::as_stream(stream)>>>(P);
  return zt::check_cuda(cudaGetLastError(), "zt_gemm_addto: launch");
}

int zt_gemm_take_error(int32_t* code) {
  zt::clear_error();
  if (!code) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_take_error: null pointer");
  int v = 0;
  if (int rc = zt::check_cuda(cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)), "zt_gemm_take_error: read")) return rc;
  const int zero = 0;
  if (int rc = zt::check_cuda(cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int)), "zt_gemm_take_error: clear"))
    return rc;
  *code = v;
  return ZT_OK;
}

}  // extern "C"
