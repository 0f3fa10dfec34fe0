// Fused linear cross-entropy: the lm_head GEMM and the per-row cross-entropy statistics
// in one tcgen05 kernel, so no logit reaches HBM.
//
//   logits[r, v] = bf16(X[r, :] . W[v, :])      (fp32 accumulate, one bf16 rounding: the
//                                                 bf16 logits the reference's head produces)
//   lse[r]  = log sum_v exp(logits[r, v]),  loss[r] = lse[r] - logits[r, t_r],
//   correct[r] = (first argmax_v logits[r, v] == t_r)
// as zotitan/losses.py:55-79 evaluates them on the fp32 upcast of the bf16 logits; replaces
// the Liger fused linear cross-entropy of zotitan/losses.py:17-52.
//
// Kernel 1 (lce_gemm_kernel) runs on CTA pairs (tcgen05.mma.cta_group::2, 256 x 256 tiles,
// K-block 64, 6 TMA stages, fp32 accumulators double-buffered in tensor memory). The
// vocabulary is cut into splits of a few 256-column tiles; a work item is (256 rows, one
// split), items are ordered row-block fastest so the pairs in flight share W tiles in L2.
// The epilogue warps own one accumulator row each and keep, across the split's tiles, an
// online (max, sum of exp(x - max)), the first argmax and the target's logit; at the end of
// the item they write these four numbers per row to a small partials buffer.
// Kernel 2 (lce_combine_kernel) merges each row's splits in vocabulary order.
// Every mbarrier wait is bounded; on expiry the kernel records an error
// (zt_linear_xent_take_error), drains its own copies and MMAs and frees its tensor memory.
#include <math.h>

#include "zt_tc.cuh"

namespace {

using namespace zt::tc;

constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA (leader), warps 2-5 epilogue
constexpr int kStages = 6;
constexpr uint32_t kHalfRows = 128;
constexpr uint32_t kStageA = kHalfRows * kBK * 2;  // 16 KB of X
constexpr uint32_t kStageBytes = 2 * kStageA;       // + 16 KB of W (this CTA's half of the N tile)
constexpr uint32_t kTile = 256;
constexpr uint32_t kTmemCols = 2 * kTile;
constexpr size_t kSmem = 1024 + kStages * kStageBytes + 256;
constexpr uint32_t kIdesc = idesc_bf16(256, 256);
constexpr float kLog2e = 1.4426950408889634f;

__device__ int g_lce_error = 0;

struct LceParams {
  CUtensorMap tmap_x;  // X [rows, k], box {64, 128}
  CUtensorMap tmap_w;  // W [vocab, k], box {64, 128}
  const int64_t* targets;
  float4* partials;    // [n_splits][rows_pad]: (max, sum exp(x - max), target logit, argmax bits)
  int32_t rows, vocab, k_blocks;
  int32_t m_tiles, n_tiles, split_tiles, n_splits, rows_pad;
  int32_t stall_loads;    // test hook: the loader issues no copies
  long long wait_cycles;  // bound of every wait
};

__device__ __forceinline__ void item_range(const LceParams& P, int item, int& mt, int& split, int& nt0, int& nt1) {
  split = item / P.m_tiles;
  mt = item - split * P.m_tiles;
  nt0 = split * P.split_tiles;
  nt1 = min(nt0 + P.split_tiles, P.n_tiles);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    lce_gemm_kernel(const __grid_constant__ LceParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;                    // [kStages], used in the leader
  uint64_t* empty = bars + kStages;         // [kStages]
  uint64_t* accf = bars + 2 * kStages;      // [2]
  uint64_t* acce = bars + 2 * kStages + 2;  // [2], used in the leader
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
  if (warp == 0) {  // warp 0 of both CTAs allocates the pair's tensor memory
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA signal
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t peer_abort = peer_addr((const void*)abort, rank ^ 1u);

  const int n_items = P.m_tiles * P.n_splits;
  const int cid = (int)cluster_id_x(), ncl = (int)n_clusters_x();
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs)
      int last_phase[kStages];
      for (int s = 0; s < kStages; ++s) last_phase[s] = -1;
      uint32_t it = 0;
      bool ok = !P.stall_loads;
      for (int item = cid; ok && item < n_items; item += ncl) {
        int mt, split, nt0, nt1;
        item_range(P, item, mt, split, nt0, nt1);
        for (int nt = nt0; ok && nt < nt1; ++nt) {
          for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
            const int s = it % kStages;
            const uint32_t round = it / kStages;
            if (!mbar_wait_pair(&empty[s], (round & 1) ^ 1, abort, peer_abort, &g_lce_error, 1, P.wait_cycles)) { ok = false; break; }
            uint8_t* sa = stage_base + s * kStageBytes;
            const uint32_t leader_full = peer_addr(&full[s], 0);
            if (leader) mbar_expect_tx(&full[s], 2 * kStageBytes);
            tma_load_2d_pair(sa, &P.tmap_x, leader_full, kb * kBK, mt * (int)kTile + (int)rank * (int)kHalfRows);
            tma_load_2d_pair(sa + kStageA, &P.tmap_w, leader_full, kb * kBK, nt * (int)kTile + (int)rank * (int)kHalfRows);
            last_phase[s] = (int)(round & 1);
          }
        }
      }
      // Drain (leader): each armed phase of a full barrier completes only when both CTAs'
      // copies for it have landed, so no copy is in flight when the pair leaves.
      if (leader)
        for (int s = 0; s < kStages; ++s)
          if (last_phase[s] >= 0) mbar_drain(&full[s], (uint32_t)last_phase[s]);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ---- MMA issuer (leader CTA only)
      uint32_t it = 0, tcount = 0;
      bool ok = true, issued = false;
      for (int item = cid; ok && item < n_items; item += ncl) {
        int mt, split, nt0, nt1;
        item_range(P, item, mt, split, nt0, nt1);
        for (int nt = nt0; ok && nt < nt1; ++nt, ++tcount) {
          const uint32_t b = tcount & 1;
          if (!mbar_wait_pair(&acce[b], ((tcount >> 1) & 1) ^ 1, abort, peer_abort, &g_lce_error, 2, P.wait_cycles)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t tmem_d = tmem_base + b * kTile;
          for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
            const int s = it % kStages;
            if (!mbar_wait_pair(&full[s], (it / kStages) & 1, abort, peer_abort, &g_lce_error, 3, P.wait_cycles)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_u32(stage_base + s * kStageBytes);
            const uint32_t sb = sa + kStageA;
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k)
              umma_bf16_pair<kIdesc>(tmem_d, umma_desc(sa + k * kUmmaK * 2), umma_desc(sb + k * kUmmaK * 2),
                                     (kb | k) != 0);
            issued = true;
            umma_commit_pair(&empty[s]);  // stage s is free in both CTAs once these MMAs have read it
          }
          if (!ok) break;
          umma_commit_pair(&accf[b]);  // accumulator b is complete in both CTAs
        }
      }
      if (issued) {  // wait (bounded) for every MMA issued by this thread before exit
        umma_commit_pair_local(drain);
        mbar_drain(drain, 0);
      }
    }
  } else {  // ---- epilogue: warps 2..5 of both CTAs; each thread owns one accumulator row
    const int q = warp & 3;
    const int row_local = q * 32 + lane;
    const uint32_t leader_acce0 = peer_addr(&acce[0], 0), leader_acce1 = peer_addr(&acce[1], 0);
    uint32_t tcount = 0;
    bool ok = true;
    for (int item = cid; ok && item < n_items; item += ncl) {
      int mt, split, nt0, nt1;
      item_range(P, item, mt, split, nt0, nt1);
      const int row = mt * (int)kTile + (int)rank * (int)kHalfRows + row_local;
      const int64_t t = row < P.rows ? __ldg(P.targets + row) : -1;
      float m = -INFINITY, s = 0.f, tgt = __int_as_float(0x7fc00000);  // NaN: target not in this split
      int amax = -1;
      for (int nt = nt0; nt < nt1; ++nt, ++tcount) {
        const uint32_t b = tcount & 1;
        int okw = 1;
        if (lane == 0) okw = mbar_wait_pair(&accf[b], (tcount >> 1) & 1, abort, peer_abort, &g_lce_error, 4, P.wait_cycles) ? 1 : 0;
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) { ok = false; break; }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int c0 = 0; c0 < (int)kTile; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + b * kTile + (uint32_t)c0, r);
          const int col0 = nt * (int)kTile + c0;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {  // the bf16 logits, as fp32
            const __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
            const uint32_t w = *reinterpret_cast<const uint32_t*>(&h);
            v[j] = __uint_as_float(w << 16);
            v[j + 1] = __uint_as_float(w & 0xffff0000u);
          }
          if (col0 + 32 > P.vocab) {  // the padded columns of the last tile
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j >= P.vocab) v[j] = -INFINITY;
          }
          float cm = v[0];
#pragma unroll
          for (int j = 1; j < 32; ++j) cm = fmaxf(cm, v[j]);
          if (cm > m) {  // a new maximum: its first column, and the sum rescaled to it
            int jj = 31;
#pragma unroll
            for (int j = 31; j >= 0; --j)
              if (v[j] == cm) jj = j;
            amax = col0 + jj;
            s = (m == -INFINITY) ? 0.f : s * ex2((m - cm) * kLog2e);
            m = cm;
          }
          if (m != -INFINITY) {
            const float ml = m * kLog2e;
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) acc += ex2(__fmaf_rn(v[j], kLog2e, -ml));
            s += acc;
          }
          if ((uint64_t)(t - col0) < 32u) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j == t) tgt = v[j];
          }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(b ? leader_acce1 : leader_acce0);  // accumulator b may be overwritten
      }
      if (ok && row < P.rows) P.partials[(size_t)split * P.rows_pad + row] = make_float4(m, s, tgt, __int_as_float(amax));
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it or read its shared memory
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
}

// One thread per row: merge the row's splits in vocabulary order.
__global__ void lce_combine_kernel(const float4* __restrict__ partials, int32_t n_splits, int32_t rows_pad,
                                   int32_t rows, int32_t vocab, const int64_t* __restrict__ targets,
                                   float* __restrict__ loss, float* __restrict__ lse, int32_t* __restrict__ correct) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const int64_t t = __ldg(targets + row);
  if (t < 0) {  // ignored position
    loss[row] = 0.f;
    if (lse) lse[row] = 0.f;
    if (correct) correct[row] = 0;
    return;
  }
  float M = -INFINITY;
  for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldg(partials + (size_t)sp * rows_pad + row).x);
  float S = 0.f, tgt = __int_as_float(0x7fc00000);
  int amax = -1;
  for (int sp = 0; sp < n_splits; ++sp) {
    const float4 p = __ldg(partials + (size_t)sp * rows_pad + row);
    if (p.x != -INFINITY) S += p.y * expf(p.x - M);
    if (!isnan(p.z)) tgt = p.z;
    if (amax < 0 && p.x == M) amax = __float_as_int(p.w);  // the first split holding the maximum
  }
  const float ls = logf(S);
  loss[row] = t >= vocab ? __int_as_float(0x7fc00000) : -((tgt - M) - ls);
  if (lse) lse[row] = M + ls;
  if (correct) correct[row] = (amax == t) ? 1 : 0;
}

// Per-device kernel attributes and the number of CTA pairs resident at once.
int g_max_pairs[64] = {0};

int prepare(int dev) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (g_max_pairs[dev] > 0) return ZT_OK;
  if (int rc = zt::check_cuda(cudaFuncSetAttribute(lce_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)kSmem), "zt_linear_xent: shared memory attribute"))
    return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)(zt::sm_count() / 2));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  int n = 0;
  if (int rc = zt::check_cuda(cudaOccupancyMaxActiveClusters(&n, lce_gemm_kernel, &cfg),
                              "zt_linear_xent: cudaOccupancyMaxActiveClusters"))
    return rc;
  if (n <= 0) return zt::set_error(ZT_ERR_CUDA, "zt_linear_xent: no CTA pair fits on this GPU");
  g_max_pairs[dev] = n;
  return ZT_OK;
}

// Vocabulary split: the split length (in 256-column tiles) whose round-robin schedule over
// `pairs` CTA pairs has the smallest longest queue, preferring longer splits on ties.
struct Split {
  int32_t m_tiles, n_tiles, split_tiles, n_splits, rows_pad;
};

Split choose_split(int64_t rows, int64_t vocab, int pairs) {
  Split sp;
  sp.m_tiles = (int32_t)((rows + kTile - 1) / kTile);
  sp.n_tiles = (int32_t)((vocab + kTile - 1) / kTile);
  sp.rows_pad = sp.m_tiles * (int32_t)kTile;
  long long best = -1;
  sp.split_tiles = sp.n_tiles;
  for (int st = 1; st <= sp.n_tiles && st <= 64; ++st) {
    const long long splits = (sp.n_tiles + st - 1) / st;
    const long long items = splits * sp.m_tiles;
    const long long queue = (items + pairs - 1) / pairs * st;
    if (best < 0 || queue <= best) {
      best = queue;
      sp.split_tiles = st;
    }
  }
  sp.n_splits = (sp.n_tiles + sp.split_tiles - 1) / sp.split_tiles;
  return sp;
}

int device_pairs(int* dev, int* pairs) {
  if (int rc = zt::check_cuda(cudaGetDevice(dev), "zt_linear_xent: cudaGetDevice")) return rc;
  if (*dev < 0 || *dev >= 64) return zt::set_error(ZT_ERR_LIMIT, "zt_linear_xent: device ordinal >= 64");
  if (int rc = prepare(*dev)) return rc;
  *pairs = g_max_pairs[*dev];
  return ZT_OK;
}

int check_shape(int64_t rows, int64_t vocab, int64_t k) {
  if (rows <= 0 || rows > (int64_t)INT32_MAX - 256) return zt::set_error(ZT_ERR_INVALID, "zt_linear_xent: rows outside [1, 2^31 - 257]");
  if (vocab <= 0 || vocab > (int64_t)INT32_MAX - 256)
    return zt::set_error(ZT_ERR_INVALID, "zt_linear_xent: vocab outside [1, 2^31 - 257]");
  if (k <= 0 || k % kBK != 0) return zt::set_error(ZT_ERR_INVALID, "zt_linear_xent: k must be a positive multiple of 64");
  return ZT_OK;
}

}  // namespace

extern "C" {

size_t zt_linear_xent_workspace_bytes(int64_t rows, int64_t vocab, int64_t k) {
  zt::clear_error();
  if (check_shape(rows, vocab, k)) return 0;
  int dev = 0, pairs = 0;
  if (device_pairs(&dev, &pairs)) return 0;
  const Split sp = choose_split(rows, vocab, pairs);
  return sizeof(float4) * (size_t)sp.n_splits * (size_t)sp.rows_pad;
}

int zt_linear_xent(const zt_lce_args* a, void* stream) {
  zt::clear_error();
  if (!a || !a->x || !a->w || !a->targets || !a->loss || !a->workspace)
    return zt::set_error(ZT_ERR_INVALID, "zt_linear_xent: null pointer");
  if (int rc = check_shape(a->rows, a->vocab, a->k)) return rc;
  auto mis16 = [](const void* p) { return ((uintptr_t)p & 15u) != 0; };
  if (mis16(a->x) || mis16(a->w) || mis16(a->workspace))
    return zt::set_error(ZT_ERR_INVALID, "zt_linear_xent: x, w and workspace must be 16-byte aligned");
  int dev = 0, pairs = 0;
  if (int rc = device_pairs(&dev, &pairs)) return rc;
  const Split sp = choose_split(a->rows, a->vocab, pairs);
  const size_t need = sizeof(float4) * (size_t)sp.n_splits * (size_t)sp.rows_pad;
  if (a->workspace_bytes < need) return zt::set_error(ZT_ERR_INVALID, "zt_linear_xent: workspace too small");
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc, "zt_linear_xent")) return rc;
  LceParams P;
  if (int rc = make_map_bf16(enc, &P.tmap_x, a->x, (uint64_t)a->rows, (uint64_t)a->k, kHalfRows, "zt_linear_xent"))
    return rc;
  if (int rc = make_map_bf16(enc, &P.tmap_w, a->w, (uint64_t)a->vocab, (uint64_t)a->k, kHalfRows, "zt_linear_xent"))
    return rc;
  P.targets = a->targets;
  P.partials = static_cast<float4*>(a->workspace);
  P.rows = (int32_t)a->rows;
  P.vocab = (int32_t)a->vocab;
  P.k_blocks = (int32_t)(a->k / kBK);
  P.m_tiles = sp.m_tiles;
  P.n_tiles = sp.n_tiles;
  P.split_tiles = sp.split_tiles;
  P.n_splits = sp.n_splits;
  P.rows_pad = sp.rows_pad;
  P.stall_loads = a->test_stall_loads ? 1 : 0;
  P.wait_cycles = a->test_wait_cycles > 0 ? (long long)a->test_wait_cycles : kWaitCycles;
  const int items = sp.m_tiles * sp.n_splits;
  const int clusters = items < pairs ? items : pairs;
  cudaStream_t s = zt::as_stream(stream);
  lce_gemm_kernel<<<2 * clusters, kThreads, kSmem, s>>>(P);
  if (int rc = zt::check_cuda(cudaGetLastError(), "zt_linear_xent: gemm launch")) return rc;
  const int tb = 256;
  lce_combine_kernel<<<(unsigned)((a->rows + tb - 1) / tb), tb, 0, s>>>(
      P.partials, sp.n_splits, sp.rows_pad, P.rows, P.vocab, a->targets, a->loss, a->lse, a->correct);
  return zt::check_cuda(cudaGetLastError(), "zt_linear_xent: combine launch");
}

int zt_linear_xent_take_error(int32_t* code) {
  zt::clear_error();
  if (!code) return zt::set_error(ZT_ERR_INVALID, "zt_linear_xent_take_error: null pointer");
  int v = 0;
  if (int rc = zt::check_cuda(cudaMemcpyFromSymbol(&v, g_lce_error, sizeof(int)), "zt_linear_xent_take_error: read"))
    return rc;
  const int zero = 0;
  if (int rc = zt::check_cuda(cudaMemcpyToSymbol(g_lce_error, &zero, sizeof(int)), "zt_linear_xent_take_error: clear"))
    return rc;
  *code = v;
  return ZT_OK;
}

}  // extern "C"
