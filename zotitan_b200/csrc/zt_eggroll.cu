// EGGROLL population linear layer on the 5th-generation tensor cores.
//
//   Y[m, :] = X[m, :] W^T + sigma_i * (X[m, :] B_i) A_i^T,   i = m / rows_per_member
//
// X [M, K] bf16 holds the activations of a whole population chunk (member i owns rows
// [i*T, (i+1)*T)), W [N, K] bf16 is the shared base weight, A_i [N, 4] and B_i [K, 4]
// (fp32) are member i's rank-4 factors and sigma_i its signed scale. The base GEMM runs
// on tcgen05 tensor cores with TMA-staged tiles; the rank-4 correction is added in the
// epilogue from X B_i (computed by a bandwidth-bound pre-pass) and the member's A_i
// tile, so W is never perturbed or copied per member.
//
// GEMM structure (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: 128x64 X tile + 256x64 W tile per stage, 4 stages,
//               128-byte swizzle, completion tracked by mbarrier transaction bytes;
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256, K=16, bf16 in,
//               fp32 accumulate in tensor memory) and tcgen05.commit to free stages;
//   warps 2..5  epilogue: tcgen05.ld of the 128x256 fp32 accumulator (each warp reads
//               its 32-lane quarter), rank-4 correction, bf16 store. The accumulator is
//               double-buffered in tensor memory (2 x 256 columns) so the epilogue of one
//               tile overlaps the MMAs of the next.
// Every mbarrier wait is bounded by a clock deadline; on expiry the kernel records an
// error code, stops issuing, drains its own copies and MMAs (again bounded), frees its
// tensor memory and returns.
#include "zt_tc.cuh"

namespace {

using namespace zt::tc;

constexpr int kBM = 128, kBN = 256, kStages = 4;
constexpr int kThreadsEgg = 192;  // 6 warps
constexpr uint32_t kStageA = kBM * kBK * 2;   // 16 KB
constexpr uint32_t kStageB = kBN * kBK * 2;   // 32 KB
constexpr uint32_t kStageBytes = kStageA + kStageB;
constexpr uint32_t kTmemCols = 2 * kBN;       // two fp32 accumulators of 128 x 256
constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + kStages * kStageBytes + 256 /*barriers, flags*/;
constexpr int kGroupN = 16;  // N-blocks per rasterisation group

// Tile order: groups of kGroupN N-blocks; inside a group the M-blocks are swept with the
// N-block fastest. The ~150 tiles in flight then touch ~10 M-blocks of X and one group's
// slice of W, both of which stay in L2, instead of streaming all of W per wave.
__device__ __forceinline__ void tile_coords(int tile, int m_blocks, int n_blocks, int& mb, int& nb) {
  const int per_group = kGroupN * m_blocks;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int rem = n_blocks - g * kGroupN;
  const int gn = rem < kGroupN ? rem : kGroupN;
  mb = r / gn;
  nb = g * kGroupN + r % gn;
}

__device__ int g_eggroll_error = 0;

struct EggParams {
  CUtensorMap tmap_x;  // X [M, K], box {64, 128}
  CUtensorMap tmap_w;  // W [N, K], box {64, 256} (single CTA) or {64, 128} (CTA pair)
  CUtensorMap tmap_y;  // Y [M, N], box {32, 32}, 64-byte swizzle (CTA-pair epilogue stores)
  CUtensorMap tmap_w2; // gated pair: W_up [N, K], box {64, 128} (tmap_w holds W_gate)
  const float* a2;     // gated: A of the up projection [members, N, 4]
  const float* sigma2; // gated: [members]
  const float* xb2;    // gated: X B_up [M, 4]
  CUtensorMap tmap_xe;  // K-slab: X_ext [M, 16] bf16, box {16, 128}, 32-byte swizzle
  CUtensorMap tmap_we;  // K-slab: W_ext [members * N, 16] bf16 (gated: of the gate projection)
  CUtensorMap tmap_we2; // gated K-slab: W_ext of the up projection
  const float* a;      // [members, N, 4]
  const float* sigma;  // [members]
  const float* xb;     // [M, 4]
  __nv_bfloat16* y;    // [M, N]
  int32_t m_blocks, n_blocks, k_blocks;
  int32_t n;
  int32_t rows_per_member;
  int32_t stall_loads;  // test hook: the loader issues no copies (zt_eggroll_args.test_stall_loads)
};

// The library's common mbarrier / TMA / tcgen05 helpers (zt_tc.cuh) with this file's
// error flag, instruction descriptor and wait bound.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  return zt::tc::mbar_wait(bar, parity, abort, &g_eggroll_error, code);
}

// Instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = idesc_bf16(kBM, kBN);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  zt::tc::umma_bf16<kIdesc>(tmem_d, adesc, bdesc, accumulate);
}

__global__ void __launch_bounds__(kThreadsEgg, 1) eggroll_gemm_kernel(const __grid_constant__ EggParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;                 // [kStages]
  uint64_t* empty = bars + kStages;      // [kStages]
  uint64_t* accf = bars + 2 * kStages;   // [2]
  uint64_t* acce = bars + 2 * kStages + 2;  // [2]
  uint64_t* drain = bars + 2 * kStages + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], 4 * 32); }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // the whole warp allocates tensor memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = P.m_blocks * P.n_blocks;
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      int last_phase[kStages];
      for (int s = 0; s < kStages; ++s) last_phase[s] = -1;
      uint32_t it = 0;
      bool ok = true;
      if (P.stall_loads) ok = false;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, P.m_blocks, P.n_blocks, mb, nb);
        for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t round = it / kStages;
          if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort, 1)) { ok = false; break; }
          uint8_t* sa = stage_base + s * kStageBytes;
          mbar_expect_tx(&full[s], kStageBytes);
          tma_load_2d(sa, &P.tmap_x, &full[s], kb * kBK, mb * kBM);
          tma_load_2d(sa + kStageA, &P.tmap_w, &full[s], kb * kBK, nb * kBN);
          last_phase[s] = (int)(round & 1);
        }
      }
      // Drain: every issued copy must have landed before the CTA can exit.
      for (int s = 0; s < kStages; ++s)
        if (last_phase[s] >= 0) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[s], (uint32_t)last_phase[s]) && clock64() - t0 < kWaitCycles) {
          }
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      uint32_t it = 0, tcount = 0;
      bool ok = true, issued = false;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++tcount) {
        const uint32_t b = tcount & 1;
        if (!mbar_wait(&acce[b], ((tcount >> 1) & 1) ^ 1, abort, 2)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tmem_d = tmem_base + b * kBN;
        for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, abort, 3)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = smem_u32(stage_base + s * kStageBytes);
          const uint32_t sb = sa + kStageA;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k)
            umma_bf16(tmem_d, umma_desc(sa + k * kUmmaK * 2), umma_desc(sb + k * kUmmaK * 2), (kb | k) != 0);
          issued = true;
          umma_commit(&empty[s]);  // stage s is free once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&accf[b]);  // accumulator b is complete
      }
      if (issued) {  // wait (bounded) for every MMA issued by this thread before exit
        umma_commit(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {  // ---- epilogue: warps 2..5
    // No barrier among the epilogue threads: each reads the member's A_i columns from
    // global memory at warp-uniform addresses (one L1 broadcast per load), so a thread
    // that gives up on a wait can leave without stranding the others.
    const int q = warp & 3;            // tensor-memory lane quarter this warp may read
    const int row = q * 32 + lane;     // row of the 128-row tile
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++tcount) {
      int mb, nb;
      tile_coords(tile, P.m_blocks, P.n_blocks, mb, nb);
      const uint32_t b = tcount & 1;
      const int m = mb * kBM + row;
      const int member = (mb * kBM) / P.rows_per_member;
      const float4* a_tile = reinterpret_cast<const float4*>(P.a + ((size_t)member * P.n + (size_t)nb * kBN) * 4);
      const float sg = __ldg(P.sigma + member);
      const float4 xb = __ldg(reinterpret_cast<const float4*>(P.xb) + m);
      const float x0 = sg * xb.x, x1 = sg * xb.y, x2 = sg * xb.z, x3 = sg * xb.w;
      // One lane waits and the warp follows its verdict, so the warp stays converged for
      // the .sync.aligned tensor-memory loads even when a wait gives up.
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&accf[b], (tcount >> 1) & 1, abort, 4) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      __syncwarp();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      __nv_bfloat16* yrow = P.y + (size_t)m * P.n + (size_t)nb * kBN;
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + b * kBN + c0, r);
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float4 a0 = __ldg(a_tile + c0 + j);
          const float4 a1 = __ldg(a_tile + c0 + j + 1);
          const float v0 = __uint_as_float(r[j]) + (x0 * a0.x + x1 * a0.y + x2 * a0.z + x3 * a0.w);
          const float v1 = __uint_as_float(r[j + 1]) + (x0 * a1.x + x1 * a1.y + x2 * a1.z + x3 * a1.w);
          const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
          packed[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
        }
        uint4* dst = reinterpret_cast<uint4*>(yrow + c0);
#pragma unroll
        for (int v = 0; v < 4; ++v)
          dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&acce[b]);  // accumulator b may be overwritten
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
}

// ---- the same GEMM on CTA pairs (tcgen05 cta_group::2) ------------------------------
//
// A cluster of two CTAs on two SMs computes a 256 x 256 tile: CTA r (r = 0, 1) loads rows
// [r*128, r*128+128) of the X tile and rows [r*128, r*128+128) of the W tile into its own
// shared memory, and the leader (r = 0) issues tcgen05.mma.cta_group::2 (M = 256, N = 256),
// which reads A from each CTA's own half and B from both halves and writes each CTA's 128
// accumulator rows into that CTA's tensor memory. Per SM this moves half the W bytes of
// the single-CTA tile through shared memory for the same tensor work. The loads carry no
// multicast: each CTA fetches its own halves, and the copies' byte counts land on the
// leader's full barrier, which the leader alone arms with both CTAs' bytes. The leader's
// commits free each stage and publish each accumulator in both CTAs (commit multicast);
// both CTAs' epilogue warps release an accumulator on the leader's barrier.
constexpr int kStages2 = 6;
constexpr uint32_t kHalfRows = 128;
constexpr uint32_t kStageA2 = kHalfRows * kBK * 2;  // 16 KB of X
constexpr uint32_t kStageB2 = kHalfRows * kBK * 2;  // 16 KB of W (this CTA's half of the N tile)
constexpr uint32_t kStageBytes2 = kStageA2 + kStageB2;
constexpr uint32_t kExtTile = kHalfRows * 16 * 2;     // 128 rows of a 16-column bf16 K-slab
constexpr uint32_t kOutChunk = 32 * 32 * 2;           // one warp's 32 x 32 bf16 output chunk
constexpr uint32_t kOutBytes2 = 4 * 2 * kOutChunk;     // 4 epilogue warps x 2 buffers
constexpr size_t kSmemBytes2 = 1024 + kStages2 * kStageBytes2 + kOutBytes2 + 256;
constexpr uint32_t kIdesc2 = idesc_bf16(256, 256);

__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  zt::tc::umma_bf16_pair<kIdesc2>(tmem_d, adesc, bdesc, accumulate);
}

// Bounded wait that also raises the peer CTA's abort flag when it gives up.
__device__ __forceinline__ bool mbar_wait_pair(uint64_t* bar, uint32_t parity, volatile int* abort, uint32_t peer_abort,
                                               int code) {
  return zt::tc::mbar_wait_pair(bar, parity, abort, peer_abort, &g_eggroll_error, code);
}

// GATED: the pair computes the Llama MLP's gate and up projections of the same 128
// output features at once: CTA 0 stages W_gate rows and CTA 1 W_up rows, so accumulator
// columns 0..127 hold G and 128..255 hold U for features [nb*128, nb*128+128), and the
// epilogue writes bf16(bf16(silu(bf16(G))) * bf16(U)) -- the rounding torch applies to
// act_fn(gate_proj(x)) * up_proj(x) -- without G or U ever reaching global memory.
// EXT: the rank-4 term runs on the tensor cores as one more K = 16 slab per tile,
// X_ext [hi, lo of sigma_i X B_i] against W_ext [A_i, A_i] (gated: gate columns 0-7, up
// columns 8-15), so the epilogue only converts (and, gated, applies the SwiGLU).
// EXT without SLAB: no rank-4 term at all, the plain GEMM (gated: gate, up and SwiGLU of
// an unperturbed Llama MLP in one kernel).
template <bool GATED, bool EXT, bool SLAB = EXT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsEgg, 1)
    eggroll_gemm_pair_kernel(const __grid_constant__ EggParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint8_t* out_base = smem + kStages2 * kStageBytes2;  // 1024-byte aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_base + kOutBytes2);
  uint64_t* full = bars;                    // [kStages2], used in the leader
  uint64_t* empty = bars + kStages2;        // [kStages2]
  uint64_t* accf = bars + 2 * kStages2;     // [2]
  uint64_t* acce = bars + 2 * kStages2 + 2; // [2], used in the leader
  uint64_t* drain = bars + 2 * kStages2 + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages2 + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
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

  const int m_tiles = P.m_blocks / 2;  // 256-row tiles
  const int n_tiles = m_tiles * P.n_blocks;
  const int cid = (int)cluster_id_x(), ncl = (int)n_clusters_x();
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs)
      int last_phase[kStages2];
      for (int s = 0; s < kStages2; ++s) last_phase[s] = -1;
      uint32_t it = 0;
      for (int tile = cid; !P.stall_loads && tile < n_tiles; tile += ncl) {
        int mb, nb;
        tile_coords(tile, m_tiles, P.n_blocks, mb, nb);
        bool ok = true;
        for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
          const int s = it % kStages2;
          const uint32_t round = it / kStages2;
          if (!mbar_wait_pair(&empty[s], (round & 1) ^ 1, abort, peer_abort, 1)) { ok = false; break; }
          uint8_t* sa = stage_base + s * kStageBytes2;
          const uint32_t leader_full = peer_addr(&full[s], 0);
          if (leader) mbar_expect_tx(&full[s], 2 * kStageBytes2);
          tma_load_2d_pair(sa, &P.tmap_x, leader_full, kb * kBK, mb * 256 + (int)rank * 128);
          if (GATED)
            tma_load_2d_pair(sa + kStageA2, rank ? &P.tmap_w2 : &P.tmap_w, leader_full, kb * kBK, nb * 128);
          else
            tma_load_2d_pair(sa + kStageA2, &P.tmap_w, leader_full, kb * kBK, nb * kBN + (int)rank * 128);
          last_phase[s] = (int)(round & 1);
        }
        if (ok && SLAB) {  // the rank-4 K-slab of this tile
          const int s = it % kStages2;
          const uint32_t round = it / kStages2;
          if (!mbar_wait_pair(&empty[s], (round & 1) ^ 1, abort, peer_abort, 1)) {
            ok = false;
          } else {
            uint8_t* sa = stage_base + s * kStageBytes2;
            const uint32_t leader_full = peer_addr(&full[s], 0);
            const int member = (mb * 256) / P.rows_per_member;
            if (leader) mbar_expect_tx(&full[s], 2 * 2 * kExtTile);
            tma_load_2d_pair(sa, &P.tmap_xe, leader_full, 0, mb * 256 + (int)rank * 128);
            if (GATED)
              tma_load_2d_pair(sa + kStageA2, rank ? &P.tmap_we2 : &P.tmap_we, leader_full, 0, member * P.n + nb * 128);
            else
              tma_load_2d_pair(sa + kStageA2, &P.tmap_we, leader_full, 0, member * P.n + nb * kBN + (int)rank * 128);
            last_phase[s] = (int)(round & 1);
            ++it;
          }
        }
        if (!ok) break;
      }
      // Drain (leader): each armed phase of a full barrier completes only when both CTAs'
      // copies for it have landed, so no copy is in flight when the pair leaves.
      if (leader)
        for (int s = 0; s < kStages2; ++s)
          if (last_phase[s] >= 0) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], (uint32_t)last_phase[s]) && clock64() - t0 < kWaitCycles) {
            }
          }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ---- MMA issuer (leader CTA only)
      uint32_t it = 0, tcount = 0;
      bool ok = true, issued = false;
      for (int tile = cid; ok && tile < n_tiles; tile += ncl, ++tcount) {
        const uint32_t b = tcount & 1;
        if (!mbar_wait_pair(&acce[b], ((tcount >> 1) & 1) ^ 1, abort, peer_abort, 2)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tmem_d = tmem_base + b * kBN;
        for (int kb = 0; kb < P.k_blocks; ++kb, ++it) {
          const int s = it % kStages2;
          if (!mbar_wait_pair(&full[s], (it / kStages2) & 1, abort, peer_abort, 3)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = smem_u32(stage_base + s * kStageBytes2);
          const uint32_t sb = sa + kStageA2;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k)
            umma_bf16_pair(tmem_d, umma_desc(sa + k * kUmmaK * 2), umma_desc(sb + k * kUmmaK * 2), (kb | k) != 0);
          issued = true;
          umma_commit_pair(&empty[s]);  // stage s is free in both CTAs once these MMAs have read it
        }
        if (ok && SLAB) {  // + (sigma_i X B_i) A_i^T as one K = 16 MMA
          const int s = it % kStages2;
          if (!mbar_wait_pair(&full[s], (it / kStages2) & 1, abort, peer_abort, 3)) {
            ok = false;
          } else {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_u32(stage_base + s * kStageBytes2);
            umma_bf16_pair(tmem_d, umma_desc32(sa), umma_desc32(sa + kStageA2), 1);
            umma_commit_pair(&empty[s]);
            ++it;
          }
        }
        if (!ok) break;
        umma_commit_pair(&accf[b]);  // accumulator b is complete in both CTAs
      }
      if (issued) {  // wait (bounded) for every MMA issued by this thread before exit
        umma_commit_pair_local(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {  // ---- epilogue: warps 2..5 of both CTAs, each on its own 128 rows
    // Each warp turns its 32 rows x 32 columns of the accumulator into bf16 in a shared
    // buffer (64-byte swizzle: conflict-free 16-byte writes) and one lane stores the chunk
    // with a TMA bulk tensor store; two buffers per warp let a store drain while the next
    // chunk is converted.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t leader_acce0 = peer_addr(&acce[0], 0), leader_acce1 = peer_addr(&acce[1], 0);
    uint8_t* obuf = out_base + q * 2 * kOutChunk;
    uint32_t tcount = 0, chunk = 0;
    for (int tile = cid; tile < n_tiles; tile += ncl, ++tcount) {
      int mb, nb;
      tile_coords(tile, m_tiles, P.n_blocks, mb, nb);
      const uint32_t b = tcount & 1;
      const int row0 = mb * 256 + (int)rank * 128;
      const int m = row0 + row;
      const int member = row0 / P.rows_per_member;
      const int col0 = nb * (GATED ? 128 : kBN);  // first output column of the tile
      const float4* a_tile = EXT ? nullptr : reinterpret_cast<const float4*>(P.a + ((size_t)member * P.n + (size_t)col0) * 4);
      const float sg = EXT ? 0.f : __ldg(P.sigma + member);
      const float4 xb = EXT ? make_float4(0.f, 0.f, 0.f, 0.f) : __ldg(reinterpret_cast<const float4*>(P.xb) + m);
      const float x0 = sg * xb.x, x1 = sg * xb.y, x2 = sg * xb.z, x3 = sg * xb.w;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_pair(&accf[b], (tcount >> 1) & 1, abort, peer_abort, 4) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      __syncwarp();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int out_cols = GATED ? 128 : kBN;
      const float4* a2_tile = nullptr;
      float u0 = 0.f, u1 = 0.f, u2 = 0.f, u3 = 0.f;
      if (GATED && !EXT) {
        a2_tile = reinterpret_cast<const float4*>(P.a2 + ((size_t)member * P.n + (size_t)nb * 128) * 4);
        const float sg2 = __ldg(P.sigma2 + member);
        const float4 xb2 = __ldg(reinterpret_cast<const float4*>(P.xb2) + m);
        u0 = sg2 * xb2.x; u1 = sg2 * xb2.y; u2 = sg2 * xb2.z; u3 = sg2 * xb2.w;
      }
      for (int c0 = 0; c0 < out_cols; c0 += 32, ++chunk) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + b * kBN + c0, r);
        uint32_t packed[16];
        if (GATED) {
          uint32_t ru[32];
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + b * kBN + 128 + c0, ru);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float h[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float4 ag = EXT ? make_float4(0.f, 0.f, 0.f, 0.f) : __ldg(a_tile + c0 + j + e);
              const float4 au = EXT ? make_float4(0.f, 0.f, 0.f, 0.f) : __ldg(a2_tile + c0 + j + e);
              const float cg = EXT ? 0.f : (x0 * ag.x + x1 * ag.y + x2 * ag.z + x3 * ag.w);
              const float cu = EXT ? 0.f : (u0 * au.x + u1 * au.y + u2 * au.z + u3 * au.w);
              const float g = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[j + e]) + cg));
              const float u = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ru[j + e]) + cu));
              h[e] = __bfloat162float(__float2bfloat16_rn(g / (1.0f + expf(-g)))) * u;
            }
            const __nv_bfloat162 hv = __floats2bfloat162_rn(h[0], h[1]);
            packed[j / 2] = *reinterpret_cast<const uint32_t*>(&hv);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float v0 = __uint_as_float(r[j]), v1 = __uint_as_float(r[j + 1]);
            if (!EXT) {
              const float4 a0 = __ldg(a_tile + c0 + j);
              const float4 a1 = __ldg(a_tile + c0 + j + 1);
              v0 += x0 * a0.x + x1 * a0.y + x2 * a0.z + x3 * a0.w;
              v1 += x0 * a1.x + x1 * a1.y + x2 * a1.z + x3 * a1.w;
            }
            const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
            packed[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        uint8_t* buf = obuf + (chunk & 1) * kOutChunk;
        if (chunk >= 2) {  // the store issued from this buffer two chunks ago has read it
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
        }
#pragma unroll
        for (int v = 0; v < 4; ++v) {  // 16-byte piece v of this row, 64-byte swizzle
          const uint32_t off = (uint32_t)lane * 64 + (uint32_t)((v ^ ((lane >> 1) & 3)) * 16);
          *reinterpret_cast<uint4*>(buf + off) =
              make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          asm volatile(
              "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n\t"
              "cp.async.bulk.commit_group;"
              ::"l"(reinterpret_cast<uint64_t>(&P.tmap_y)), "r"(col0 + c0), "r"(row0 + q * 32), "r"(smem_u32(buf))
              : "memory");
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(b ? leader_acce1 : leader_acce0);  // accumulator b may be overwritten
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // all stores complete
    __syncwarp();
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

// XB_s[m, r] = sum_k X[m, k] * B_{s,i}[k, r] (fp32) for up to 3 factor sets s that share
// X (q/k/v, or gate/up): X is read once for all of them. One CTA per 64 rows of one
// member (8 warps x 8 rows). B_{s,i} is staged in shared memory in chunks of 512 k,
// transposed to [s][r][k], so lane l reads the float4 at k = 4l + 128j (consecutive
// 16-byte words across the warp: no bank conflicts) and the same B values serve the
// warp's 8 rows. X moves as 8-byte loads of 4 bf16 (256 contiguous bytes per warp and row).
constexpr int kXbRows = 64, kXbRowsPerWarp = 8, kXbChunk = 512, kXbMaxSeg = 3;
static_assert(kXbRows == 8 * kXbRowsPerWarp, "8 warps per CTA");

struct XbSegs {
  const float* b[kXbMaxSeg];      // [members, k, 4]
  float* xb[kXbMaxSeg];           // [m, 4] fp32 (or NULL)
  const float* sigma[kXbMaxSeg];  // [members] (read when xe is set)
  uint4* xe[kXbMaxSeg];           // [m, 16] bf16 K-slab rows (or NULL)
  int32_t xe_slot[kXbMaxSeg];
};

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

// K-slab row of sigma * X B: v = hi + lo with hi = bf16(v), lo = bf16(v - hi).
__device__ __forceinline__ void write_xe(uint4* row, int slot, float sg, const float acc[4]) {
  __nv_bfloat16 h[4], l[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float v = sg * acc[r];
    h[r] = __float2bfloat16_rn(v);
    l[r] = __float2bfloat16_rn(v - __bfloat162float(h[r]));
  }
  const uint4 hl = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(l[0], l[1]),
                              pack_bf16x2(l[2], l[3]));
  if (slot == 0) {
    row[0] = hl;
    row[1] = make_uint4(0u, 0u, 0u, 0u);
  } else {
    row[slot - 1] = hl;
  }
}

template <int NSEG>
__global__ void __launch_bounds__(256, 1) eggroll_xb_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const __grid_constant__ XbSegs S, int32_t k,
                                                            int32_t rows_per_member) {
  __shared__ __align__(16) float bt[NSEG][4][kXbChunk];
  const int64_t row0 = (int64_t)blockIdx.x * kXbRows;
  const int member = (int)(row0 / rows_per_member);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t wrow = row0 + warp * kXbRowsPerWarp;
  float acc[NSEG][kXbRowsPerWarp][4];
#pragma unroll
  for (int s = 0; s < NSEG; ++s)
#pragma unroll
    for (int i = 0; i < kXbRowsPerWarp; ++i) acc[s][i][0] = acc[s][i][1] = acc[s][i][2] = acc[s][i][3] = 0.f;
  for (int kc = 0; kc < k; kc += kXbChunk) {
    const int len = (k - kc) < kXbChunk ? (k - kc) : kXbChunk;
    __syncthreads();
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      const float4* bm = reinterpret_cast<const float4*>(S.b[s] + (size_t)member * k * 4) + kc;
      for (int t = threadIdx.x; t < len; t += 256) {
        const float4 v = __ldg(bm + t);
        bt[s][0][t] = v.x; bt[s][1][t] = v.y; bt[s][2][t] = v.z; bt[s][3][t] = v.w;
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kXbChunk / 128; ++j) {
      const int t = 4 * lane + 128 * j;
      if (t < len) {  // len % 4 == 0
        float xf[kXbRowsPerWarp][4];
#pragma unroll
        for (int i = 0; i < kXbRowsPerWarp; ++i) {
          const uint2 w = __ldcs(reinterpret_cast<const uint2*>(x + (wrow + i) * (int64_t)k + kc + t));
          xf[i][0] = __uint_as_float(w.x << 16);
          xf[i][1] = __uint_as_float(w.x & 0xffff0000u);
          xf[i][2] = __uint_as_float(w.y << 16);
          xf[i][3] = __uint_as_float(w.y & 0xffff0000u);
        }
#pragma unroll
        for (int s = 0; s < NSEG; ++s)
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float4 bv = *reinterpret_cast<const float4*>(&bt[s][r][t]);
#pragma unroll
            for (int i = 0; i < kXbRowsPerWarp; ++i)
              acc[s][i][r] = fmaf(xf[i][0], bv.x, fmaf(xf[i][1], bv.y, fmaf(xf[i][2], bv.z, fmaf(xf[i][3], bv.w, acc[s][i][r]))));
          }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < NSEG; ++s)
#pragma unroll
    for (int i = 0; i < kXbRowsPerWarp; ++i) {
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[s][i][r] += __shfl_xor_sync(0xffffffffu, acc[s][i][r], o);
      if (lane == 0) {
        if (S.xb[s])
          reinterpret_cast<float4*>(S.xb[s])[wrow + i] = make_float4(acc[s][i][0], acc[s][i][1], acc[s][i][2], acc[s][i][3]);
        if (S.xe[s]) write_xe(S.xe[s] + 2 * (wrow + i), S.xe_slot[s], __ldg(S.sigma[s] + member), acc[s][i]);
      }
    }
}

// ---- X B on the tensor cores (K-slab path) ---------------------------------------------
//
// One CTA per 128-row tile of one member: XB[128, 16] = X[tile, K] Bt[member]^T with
// Bt [members, 16, K] bf16 (set s in rows 4s..4s+3), tcgen05.mma M = 128, N = 16 into 16
// tensor-memory columns; X and Bt tiles arrive by TMA (128-byte swizzle) through a
// 4-stage ring. The epilogue turns each set's 4 columns into K-slab rows
// [hi, lo] of sigma_i X B (and fp32 X B if asked). X is read once for all sets, at HBM rate.
constexpr int kXtStages = 4;
constexpr uint32_t kXtA = 128 * kBK * 2;   // 16 KB of X
constexpr uint32_t kXtB = 16 * kBK * 2;    // 2 KB of Bt
constexpr uint32_t kXtStage = kXtA + 2048;  // 1024-aligned stages
constexpr size_t kXtSmem = 1024 + kXtStages * kXtStage + 256;
constexpr uint32_t kXtIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(16 >> 3) << 17) |
                              ((uint32_t)(128 >> 4) << 24);

struct XbtParams {
  CUtensorMap tmap_x;   // X [M, K], box {64, 128}
  CUtensorMap tmap_bt;  // Bt [members * 16, K], box {64, 16}
  XbSegs S;
  int32_t n_seg;
  int32_t k_blocks;
  int32_t rows_per_member;
};

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kThreadsEgg, 1) eggroll_xbt_kernel(const __grid_constant__ XbtParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kXtStages * kXtStage);
  uint64_t* full = bars;
  uint64_t* empty = bars + kXtStages;
  uint64_t* accf = bars + 2 * kXtStages;
  uint64_t* drain = accf + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row0 = blockIdx.x * 128;
  const int member = row0 / P.rows_per_member;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kXtStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(accf, 1);
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(32)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      int last_phase[kXtStages];
      for (int s = 0; s < kXtStages; ++s) last_phase[s] = -1;
      for (int kb = 0; kb < P.k_blocks; ++kb) {
        const int s = kb % kXtStages;
        const uint32_t round = kb / kXtStages;
        if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort, 5)) break;
        uint8_t* sa = smem + s * kXtStage;
        mbar_expect_tx(&full[s], kXtA + kXtB);
        tma_load_2d(sa, &P.tmap_x, &full[s], kb * kBK, row0);
        tma_load_2d(sa + kXtA, &P.tmap_bt, &full[s], kb * kBK, member * 16);
        last_phase[s] = (int)(round & 1);
      }
      for (int s = 0; s < kXtStages; ++s)
        if (last_phase[s] >= 0) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[s], (uint32_t)last_phase[s]) && clock64() - t0 < kWaitCycles) {
          }
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      bool ok = true, issued = false;
      for (int kb = 0; kb < P.k_blocks; ++kb) {
        const int s = kb % kXtStages;
        if (!mbar_wait(&full[s], (kb / kXtStages) & 1, abort, 6)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t sa = smem_u32(smem + s * kXtStage);
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k) {
          const uint64_t ad = umma_desc(sa + k * kUmmaK * 2), bd = umma_desc(sa + kXtA + k * kUmmaK * 2);
          const uint32_t acc = (kb | k) != 0;
          asm volatile(
              "{\n\t.reg .pred p;\n\t"
              "setp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
              ::"r"(tmem_base), "l"(ad), "l"(bd), "r"(kXtIdesc), "r"(acc)
              : "memory");
        }
        issued = true;
        umma_commit(&empty[s]);
      }
      if (ok && issued) umma_commit(accf);
      if (issued) {
        umma_commit(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {  // ---- epilogue: warps 2..5, one row each
    const int q = warp & 3;
    const int m = row0 + q * 32 + lane;
    int ok = 1;
    if (lane == 0) ok = mbar_wait(accf, 0, abort, 7) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) {
      __syncwarp();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t r[16];
      tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16), r);
      for (int sidx = 0; sidx < P.n_seg; ++sidx) {
        float acc[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c] = __uint_as_float(r[4 * sidx + c]);
        if (P.S.xb[sidx])
          reinterpret_cast<float4*>(P.S.xb[sidx])[m] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (P.S.xe[sidx]) write_xe(P.S.xe[sidx] + 2 * (size_t)m, P.S.xe_slot[sidx], __ldg(P.S.sigma[sidx] + member), acc);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(32) : "memory");
  }
}

int launch_xb(const void* x, const float* const* b, float* const* xb, int nseg, int64_t m, int64_t k,
              int32_t rows_per_member, cudaStream_t s, const float* const* sigma = nullptr,
              void* const* xe = nullptr, const int32_t* xe_slot = nullptr) {
  XbSegs S{};
  for (int i = 0; i < nseg; ++i) {
    S.b[i] = b[i];
    S.xb[i] = xb[i];
    S.sigma[i] = sigma ? sigma[i] : nullptr;
    S.xe[i] = xe ? static_cast<uint4*>(xe[i]) : nullptr;
    S.xe_slot[i] = xe_slot ? xe_slot[i] : 0;
  }
  const unsigned grid = (unsigned)(m / kXbRows);
  const __nv_bfloat16* xp = static_cast<const __nv_bfloat16*>(x);
  switch (nseg) {
    case 1: eggroll_xb_kernel<1><<<grid, 256, 0, s>>>(xp, S, (int32_t)k, rows_per_member); break;
    case 2: eggroll_xb_kernel<2><<<grid, 256, 0, s>>>(xp, S, (int32_t)k, rows_per_member); break;
    default: eggroll_xb_kernel<3><<<grid, 256, 0, s>>>(xp, S, (int32_t)k, rows_per_member); break;
  }
  return zt::check_cuda(cudaGetLastError(), "eggroll xb launch");
}

int get_encode(EncodeFn* fn) { return zt::tc::get_encode(fn, "zt_eggroll_linear"); }

int make_map(EncodeFn enc, CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  return make_map_bf16(enc, map, base, rows, cols, box_rows, "zt_eggroll_linear");
}

// A 16-column bf16 K-slab [rows, 16]: box {16, 128}, 32-byte swizzle.
int make_ext_map(EncodeFn enc, CUtensorMap* map, const void* base, uint64_t rows) {
  const cuuint64_t dims[2] = {16, rows};
  const cuuint64_t strides[1] = {32};
  const cuuint32_t box[2] = {16, kHalfRows};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return zt::set_error(ZT_ERR_CUDA, "eggroll: cuTensorMapEncodeTiled (K-slab) failed");
  return ZT_OK;
}

int make_out_map(EncodeFn enc, CUtensorMap* map, void* base, uint64_t rows, uint64_t cols) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return zt::set_error(ZT_ERR_CUDA, "eggroll: cuTensorMapEncodeTiled (output) failed");
  return ZT_OK;
}

// The dynamic shared-memory limits are per-device function attributes; the number of CTA
// pairs that fit at once (GPC boundaries) is queried once per device.
int g_max_pairs[64] = {0};

int prepare_kernels() {
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "eggroll: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return zt::set_error(ZT_ERR_LIMIT, "eggroll: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return ZT_OK;
  if (int rc = zt::check_cuda(cudaFuncSetAttribute(eggroll_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)kSmemBytes), "eggroll: shared memory attribute"))
    return rc;
  if (int rc = zt::check_cuda(cudaFuncSetAttribute(eggroll_xbt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)kXtSmem), "eggroll: shared memory attribute (xb)"))
    return rc;
  for (auto fn : {eggroll_gemm_pair_kernel<false, false>, eggroll_gemm_pair_kernel<true, false>,
                  eggroll_gemm_pair_kernel<false, true>, eggroll_gemm_pair_kernel<true, true>,
                  eggroll_gemm_pair_kernel<false, true, false>, eggroll_gemm_pair_kernel<true, true, false>})
    if (int rc = zt::check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes2),
                                "eggroll: shared memory attribute (pair)"))
      return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)(zt::sm_count() / 2));
  cfg.blockDim = dim3(kThreadsEgg);
  cfg.dynamicSmemBytes = kSmemBytes2;
  int n = 0;
  if (int rc = zt::check_cuda(cudaOccupancyMaxActiveClusters(&n, eggroll_gemm_pair_kernel<false, false>, &cfg),
                              "eggroll: cudaOccupancyMaxActiveClusters"))
    return rc;
  if (n <= 0) return zt::set_error(ZT_ERR_CUDA, "eggroll: no CTA pair fits on this GPU");
  g_max_pairs[dev] = n;
  done[dev] = true;
  return ZT_OK;
}

// mode 0: rank-4 term in the fp32 epilogue, 1: as a K-slab, 2: no rank-4 term.
template <bool GATED>
int launch_pair(const EggParams& P, int mode, cudaStream_t s) {
  int dev = 0;
  if (int rc = zt::check_cuda(cudaGetDevice(&dev), "eggroll: cudaGetDevice")) return rc;
  const int max_clusters = g_max_pairs[dev];
  const int tiles = (P.m_blocks / 2) * P.n_blocks;
  const int clusters = tiles < max_clusters ? tiles : max_clusters;
  if (mode == 1)
    eggroll_gemm_pair_kernel<GATED, true><<<2 * clusters, kThreadsEgg, kSmemBytes2, s>>>(P);
  else if (mode == 2)
    eggroll_gemm_pair_kernel<GATED, true, false><<<2 * clusters, kThreadsEgg, kSmemBytes2, s>>>(P);
  else
    eggroll_gemm_pair_kernel<GATED, false><<<2 * clusters, kThreadsEgg, kSmemBytes2, s>>>(P);
  return zt::check_cuda(cudaGetLastError(), GATED ? "eggroll: gated gemm launch" : "eggroll: gemm launch (pair)");
}

int xb_tensor_cores(const zt_eggroll_xb_args& A, cudaStream_t s) {
  if (A.n_seg < 1 || A.n_seg > kXbMaxSeg) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: n_seg must be 1, 2 or 3");
  if (A.m <= 0 || A.k <= 0 || A.m % 128 || A.k % kBK)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: the tensor-core form needs m % 128 == 0 and k % 64 == 0");
  if (A.rows_per_member <= 0 || A.rows_per_member % 128 || A.m % A.rows_per_member)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: rows_per_member must divide m and be a multiple of 128");
  if (A.m > (int64_t)INT32_MAX || A.k > (int64_t)INT32_MAX) return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_xb: dimension too large");
  if (!A.x || ((uintptr_t)A.x & 15) || ((uintptr_t)A.bt & 15))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: x / bt null or not 16-byte aligned");
  XbtParams P{};
  for (int i = 0; i < A.n_seg; ++i) {
    if (((uintptr_t)A.xb[i] & 15) || (!A.xb[i] && !A.xe[i]))
      return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: each set needs an aligned xb or xe");
    if (A.xe[i] && (!A.sigma[i] || ((uintptr_t)A.xe[i] & 15) || A.xe_slot[i] < 0 || A.xe_slot[i] > 2))
      return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: xe needs sigma, 16-byte alignment and a slot 0-2");
    P.S.xb[i] = A.xb[i];
    P.S.xe[i] = static_cast<uint4*>(A.xe[i]);
    P.S.sigma[i] = A.sigma[i];
    P.S.xe_slot[i] = A.xe_slot[i];
  }
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc)) return rc;
  if (int rc = make_map(enc, &P.tmap_x, A.x, (uint64_t)A.m, (uint64_t)A.k, 128)) return rc;
  if (int rc = make_map(enc, &P.tmap_bt, A.bt, (uint64_t)(A.m / A.rows_per_member) * 16, (uint64_t)A.k, 16)) return rc;
  P.n_seg = A.n_seg;
  P.k_blocks = (int32_t)(A.k / kBK);
  P.rows_per_member = A.rows_per_member;
  if (int rc = prepare_kernels()) return rc;
  eggroll_xbt_kernel<<<(unsigned)(A.m / 128), kThreadsEgg, kXtSmem, s>>>(P);
  return zt::check_cuda(cudaGetLastError(), "zt_eggroll_xb: tensor-core launch");
}

}  // namespace

extern "C" {

int zt_eggroll_linear(const zt_eggroll_args* args, void* stream) {
  zt::clear_error();
  if (!args) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: null args");
  const zt_eggroll_args& A = *args;
  const bool ext = A.x_ext && A.w_ext;
  if (!A.x || !A.w || !A.y || (!ext && (!A.a || (!A.b && !A.xb_ready) || !A.sigma || !A.xb)))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: null pointer");
  if (ext && (A.m % 256 || A.rows_per_member % 256))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: the K-slab form needs M and rows_per_member % 256 == 0");
  if (A.rank != 4) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: rank must be 4");
  if (A.m <= 0 || A.n <= 0 || A.k <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: empty shape");
  if (A.m % kBM || A.n % kBN || A.k % kBK)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: need M % 128 == 0, N % 256 == 0, K % 64 == 0");
  if (A.rows_per_member <= 0 || A.rows_per_member % kBM || A.m % A.rows_per_member)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: rows_per_member must divide M and be a multiple of 128");
  if (A.m > (int64_t)INT32_MAX || A.n > (int64_t)INT32_MAX || A.k > (int64_t)INT32_MAX)
    return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_linear: dimension above 2^31-1");
  for (const void* p : {A.x, A.w, (const void*)A.a, (const void*)A.b, (const void*)A.xb, (const void*)A.y, A.x_ext,
                        A.w_ext})
    if (((uintptr_t)p & 15) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_linear: pointers must be 16-byte aligned");
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc)) return rc;
  // CTA pairs (cta_group::2) whenever the rows split into 256-row tiles
  const bool pair = (A.m % 256) == 0;
  EggParams P;
  P.stall_loads = A.test_stall_loads ? 1 : 0;
  if (int rc = make_map(enc, &P.tmap_x, A.x, (uint64_t)A.m, (uint64_t)A.k, kBM)) return rc;
  if (int rc = make_map(enc, &P.tmap_w, A.w, (uint64_t)A.n, (uint64_t)A.k, pair ? kHalfRows : kBN)) return rc;
  if (pair)
    if (int rc = make_out_map(enc, &P.tmap_y, A.y, (uint64_t)A.m, (uint64_t)A.n)) return rc;
  if (ext) {
    if (int rc = make_ext_map(enc, &P.tmap_xe, A.x_ext, (uint64_t)A.m)) return rc;
    if (int rc = make_ext_map(enc, &P.tmap_we, A.w_ext, (uint64_t)(A.m / A.rows_per_member) * (uint64_t)A.n)) return rc;
  }
  P.a = A.a;
  P.sigma = A.sigma;
  P.xb = A.xb;
  P.a2 = nullptr;
  P.sigma2 = nullptr;
  P.xb2 = nullptr;
  P.y = static_cast<__nv_bfloat16*>(A.y);
  P.m_blocks = (int32_t)(A.m / kBM);
  P.n_blocks = (int32_t)(A.n / kBN);
  P.k_blocks = (int32_t)(A.k / kBK);
  P.n = (int32_t)A.n;
  P.rows_per_member = A.rows_per_member;
  cudaStream_t s = zt::as_stream(stream);
  if (!A.xb_ready && !ext) {  // m % 128 == 0 and rows_per_member % 128 == 0: each 64-row block lies in one member
    const float* bb[1] = {A.b};
    float* xx[1] = {A.xb};
    if (int rc = launch_xb(A.x, bb, xx, 1, A.m, A.k, A.rows_per_member, s)) return rc;
  }
  if (int rc = prepare_kernels()) return rc;
  if (pair) return launch_pair<false>(P, ext ? 1 : 0, s);
  const int tiles = P.m_blocks * P.n_blocks;
  const int grid = tiles < zt::sm_count() ? tiles : zt::sm_count();
  eggroll_gemm_kernel<<<grid, kThreadsEgg, kSmemBytes, s>>>(P);
  return zt::check_cuda(cudaGetLastError(), "zt_eggroll_linear: gemm launch");
}

int zt_eggroll_gated(const zt_eggroll_gated_args* args, void* stream) {
  zt::clear_error();
  if (!args) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: null args");
  const zt_eggroll_gated_args& A = *args;
  const bool ext = A.x_ext && A.w_ext_gate && A.w_ext_up;
  if (!A.x || !A.w_gate || !A.w_up || !A.y ||
      (!ext && (!A.a_gate || !A.a_up || !A.sigma_gate || !A.sigma_up || !A.xb_gate || !A.xb_up)))
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: null pointer");
  if (ext && A.rows_per_member % 256)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: the K-slab form needs rows_per_member % 256 == 0");
  if (A.rank != 4) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: rank must be 4");
  if (A.m <= 0 || A.n <= 0 || A.k <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: empty shape");
  if (A.m % 256 || A.n % 128 || A.k % kBK)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: need M % 256 == 0, N % 128 == 0, K % 64 == 0");
  if (A.rows_per_member <= 0 || A.rows_per_member % kBM || A.m % A.rows_per_member)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: rows_per_member must divide M and be a multiple of 128");
  if (A.m > (int64_t)INT32_MAX || A.n > (int64_t)INT32_MAX || A.k > (int64_t)INT32_MAX)
    return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_gated: dimension above 2^31-1");
  for (const void* p : {A.x, A.w_gate, A.w_up, (const void*)A.a_gate, (const void*)A.a_up, (const void*)A.xb_gate,
                        (const void*)A.xb_up, (const void*)A.y, A.x_ext, A.w_ext_gate, A.w_ext_up})
    if (((uintptr_t)p & 15) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_gated: pointers must be 16-byte aligned");
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc)) return rc;
  EggParams P;
  P.stall_loads = 0;
  if (int rc = make_map(enc, &P.tmap_x, A.x, (uint64_t)A.m, (uint64_t)A.k, kBM)) return rc;
  if (int rc = make_map(enc, &P.tmap_w, A.w_gate, (uint64_t)A.n, (uint64_t)A.k, kHalfRows)) return rc;
  if (int rc = make_map(enc, &P.tmap_w2, A.w_up, (uint64_t)A.n, (uint64_t)A.k, kHalfRows)) return rc;
  if (int rc = make_out_map(enc, &P.tmap_y, A.y, (uint64_t)A.m, (uint64_t)A.n)) return rc;
  if (ext) {
    const uint64_t wrows = (uint64_t)(A.m / A.rows_per_member) * (uint64_t)A.n;
    if (int rc = make_ext_map(enc, &P.tmap_xe, A.x_ext, (uint64_t)A.m)) return rc;
    if (int rc = make_ext_map(enc, &P.tmap_we, A.w_ext_gate, wrows)) return rc;
    if (int rc = make_ext_map(enc, &P.tmap_we2, A.w_ext_up, wrows)) return rc;
  }
  P.a = A.a_gate;
  P.sigma = A.sigma_gate;
  P.xb = A.xb_gate;
  P.a2 = A.a_up;
  P.sigma2 = A.sigma_up;
  P.xb2 = A.xb_up;
  P.y = static_cast<__nv_bfloat16*>(A.y);
  P.m_blocks = (int32_t)(A.m / kBM);
  P.n_blocks = (int32_t)(A.n / 128);  // tiles of 128 output features
  P.k_blocks = (int32_t)(A.k / kBK);
  P.n = (int32_t)A.n;
  P.rows_per_member = A.rows_per_member;
  if (int rc = prepare_kernels()) return rc;
  return launch_pair<true>(P, ext ? 1 : 0, zt::as_stream(stream));
}

int zt_gemm_swiglu(const void* x, const void* w_gate, const void* w_up, void* y, int64_t m, int64_t n, int64_t k,
                   void* stream) {
  zt::clear_error();
  if (!x || !w_gate || !w_up || !y) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_swiglu: null pointer");
  if (m <= 0 || n <= 0 || k <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_swiglu: empty shape");
  if (m % 256 || n % 128 || k % kBK)
    return zt::set_error(ZT_ERR_INVALID, "zt_gemm_swiglu: need m % 256 == 0, n % 128 == 0, k % 64 == 0");
  if (m > (int64_t)INT32_MAX || n > (int64_t)INT32_MAX || k > (int64_t)INT32_MAX)
    return zt::set_error(ZT_ERR_LIMIT, "zt_gemm_swiglu: dimension above 2^31-1");
  for (const void* p : {x, w_gate, w_up, (const void*)y})
    if (((uintptr_t)p & 15) != 0) return zt::set_error(ZT_ERR_INVALID, "zt_gemm_swiglu: pointers must be 16-byte aligned");
  EncodeFn enc = nullptr;
  if (int rc = get_encode(&enc)) return rc;
  EggParams P;
  P.stall_loads = 0;
  if (int rc = make_map(enc, &P.tmap_x, x, (uint64_t)m, (uint64_t)k, kBM)) return rc;
  if (int rc = make_map(enc, &P.tmap_w, w_gate, (uint64_t)n, (uint64_t)k, kHalfRows)) return rc;
  if (int rc = make_map(enc, &P.tmap_w2, w_up, (uint64_t)n, (uint64_t)k, kHalfRows)) return rc;
  if (int rc = make_out_map(enc, &P.tmap_y, y, (uint64_t)m, (uint64_t)n)) return rc;
  P.a = nullptr;
  P.sigma = nullptr;
  P.xb = nullptr;
  P.a2 = nullptr;
  P.sigma2 = nullptr;
  P.xb2 = nullptr;
  P.y = static_cast<__nv_bfloat16*>(y);
  P.m_blocks = (int32_t)(m / kBM);
  P.n_blocks = (int32_t)(n / 128);
  P.k_blocks = (int32_t)(k / kBK);
  P.n = (int32_t)n;
  P.rows_per_member = (int32_t)m;  // one "member": no rank-4 term is read
  if (int rc = prepare_kernels()) return rc;
  return launch_pair<true>(P, 2, zt::as_stream(stream));
}

int zt_eggroll_xb(const zt_eggroll_xb_args* args, void* stream) {
  zt::clear_error();
  if (!args) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: null args");
  const zt_eggroll_xb_args& A = *args;
  if (A.bt) return xb_tensor_cores(A, zt::as_stream(stream));
  if (A.n_seg < 1 || A.n_seg > kXbMaxSeg) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: n_seg must be 1, 2 or 3");
  if (A.m <= 0 || A.k <= 0) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: empty shape");
  if (A.m % kXbRows || A.k % 4) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: need m % 64 == 0 and k % 4 == 0");
  if (A.rows_per_member <= 0 || A.rows_per_member % kXbRows || A.m % A.rows_per_member)
    return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: rows_per_member must divide m and be a multiple of 64");
  if (A.m > (int64_t)INT32_MAX * kXbRows || A.k > (int64_t)INT32_MAX)
    return zt::set_error(ZT_ERR_LIMIT, "zt_eggroll_xb: dimension too large");
  if (!A.x || ((uintptr_t)A.x & 15)) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: x null or not 16-byte aligned");
  for (int i = 0; i < A.n_seg; ++i) {
    if (!A.b[i] || ((uintptr_t)A.b[i] & 15) || ((uintptr_t)A.xb[i] & 15))
      return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: b null or b/xb not 16-byte aligned");
    if (!A.xb[i] && !A.xe[i]) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: a set with neither xb nor xe");
    if (A.xe[i] && (!A.sigma[i] || ((uintptr_t)A.xe[i] & 15) || A.xe_slot[i] < 0 || A.xe_slot[i] > 2))
      return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_xb: xe needs sigma, 16-byte alignment and a slot 0-2");
  }
  return launch_xb(A.x, A.b, A.xb, A.n_seg, A.m, A.k, A.rows_per_member, zt::as_stream(stream), A.sigma, A.xe,
                   A.xe_slot);
}

int zt_eggroll_take_error(int32_t* code) {
  zt::clear_error();
  if (!code) return zt::set_error(ZT_ERR_INVALID, "zt_eggroll_take_error: null pointer");
  int v = 0;
  if (int rc = zt::check_cuda(cudaMemcpyFromSymbol(&v, g_eggroll_error, sizeof(int)), "zt_eggroll_take_error: read"))
    return rc;
  const int zero = 0;
  if (v != 0) {
    if (int rc = zt::check_cuda(cudaMemcpyToSymbol(g_eggroll_error, &zero, sizeof(int)), "zt_eggroll_take_error: clear"))
      return rc;
  }
  *code = v;
  return ZT_OK;
}

}  // extern "C"
