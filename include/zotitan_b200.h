/* zotitan_b200 — C ABI of the B200-native zeroth-order hot path.
 *
 * Replaces the reference's Triton noise kernel and the torch foreach passes
 * built on it (zotitan/train_zo.py). All functions:
 *   - return 0 on success and a nonzero ZT_ERR_* code on failure; the message is
 *     available from zt_last_error() on the same host thread;
 *   - never allocate device memory; callers own every buffer;
 *   - enqueue work on the CUDA stream passed as `stream` (a cudaStream_t; NULL =
 *     legacy default stream) and never synchronise the host;
 *   - take device pointers for tensor data and host pointers for descriptors.
 *
 * Noise contract (bit-exact with the reference): element `o` of the parameter at
 * position `index` of an `n_params`-long trainable list, for pair seed `seed`, is
 *   Philox4x32-10(counter (o,0,0,0), key (k,0)), k = (seed*n_params+index) & 0x7FFFFFFF,
 *   words 0,1 -> uniforms -> Box-Muller cosine branch,
 * exactly as Triton 3.6.0's tl.random.randn(k, o) evaluates it on a GPU
 * (zotitan/train_zo.py:18-28 and :302).
 */
#ifndef ZOTITAN_B200_H
#define ZOTITAN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ZT_API __attribute__((visibility("default")))
#else
#define ZT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ZT_ABI_VERSION 11

/* dtypes of parameter tensors */
#define ZT_F32 0
#define ZT_BF16 1
#define ZT_F16 2

/* status codes */
#define ZT_OK 0
#define ZT_ERR_INVALID 1   /* bad argument (null pointer, size out of range, ...) */
#define ZT_ERR_CUDA 2      /* a CUDA runtime call or kernel launch failed */
#define ZT_ERR_LIMIT 3     /* a documented maximum was exceeded */

#define ZT_MAX_STREAMS 256      /* noise streams per zt_pass call */
#define ZT_MAX_CHAIN 3          /* perturbation coefficients per stream */
#define ZT_MAX_NUMEL 2147483647 /* per-tensor element limit (int32 offsets, as the reference) */
#define ZT_MAX_PUSH_RANKS 8     /* ranks a pass can push a field to (zt_pass_cfg.zpush) */

/* Last error message of the calling host thread ("" if none). */
ZT_API const char* zt_last_error(void);
ZT_API int zt_abi_version(void);

/* Per-tensor key (zotitan/train_zo.py:302); pure host function. */
ZT_API uint32_t zt_param_key(uint64_t seed, uint32_t n_params, uint32_t index);

/* ---- test entry points: raw noise ------------------------------------------------ */

/* out4[4*i + w] = Philox word w at counter offsets[i] for key `key`.
 * Replaces nothing in the reference (its words are internal to tl.random.randn,
 * triton/language/random.py:88-110); exported to pin bit-exactness. */
ZT_API int zt_philox_words(uint32_t key, const uint32_t* offsets, int64_t n, uint32_t* out4, void* stream);

/* out[i] = N(0,1) sample at offset off0 + i for key `key`.
 * Replaces _philox_randn(seed, n, device) (zotitan/train_zo.py:25-28) with off0 = 0. */
ZT_API int zt_randn(uint32_t key, int64_t off0, int64_t n, float* out, void* stream);

/* out[i] = N(0,1) sample at offsets[i]. */
ZT_API int zt_randn_at(uint32_t key, const uint32_t* offsets, int64_t n, float* out, void* stream);

/* out[j*n + t] = N(0,1) sample at offset t for key keys[j] (host array), j < n_keys <= 1024:
 * many tensors' fields in one launch (the EGGROLL factors of a population chunk). Each
 * row equals zt_randn(keys[j], 0, n). */
ZT_API int zt_randn_keys(const uint32_t* keys, int32_t n_keys, int64_t n, float* out, void* stream);

/* ---- parameter tables -------------------------------------------------------------- */

/* One trainable tensor. `data` is the parameter; the other buffers are optional
 * (NULL when unused) and must have the same dtype and numel:
 *   live   a second copy the model reads while `data` holds the unperturbed master
 *          (seed-sharded multi-GPU mode);
 *   m      stored-EMA first moment   (ZOOptimizer.m,  zotitan/train_zo.py:257-258)
 *   v      second moment             (ZOOptimizer.v,  zotitan/train_zo.py:265-266)
 *   anchor theta_0 for anchored weight decay (zotitan/train_zo.py:273-274)
 *   ge     the gradient estimate accumulated across a step's passes, in the
 *          parameter dtype (grad_est of zotitan/train_zo.py:555-556). */
typedef struct zt_tensor {
  void* data;
  void* live;
  void* m;
  void* v;
  const void* anchor;
  void* ge;
  int64_t numel;
  int32_t dtype;   /* ZT_F32 / ZT_BF16 / ZT_F16 */
  int32_t index;   /* position in the reference's named-parameter list */
} zt_tensor;

/* A table of tensors resident in a caller-provided device workspace. */
typedef struct zt_plan {
  const zt_tensor* tensors;    /* device copy of the descriptors */
  const int64_t* unit_prefix;  /* device: first work unit of each tensor, n_tensors+1 entries */
  int64_t n_units;             /* work units of ZT_UNIT_ELEMS elements (per tensor, rounded up) */
  int64_t numel_total;
  int32_t n_tensors;
  uint32_t n_params;           /* length of the reference's named-parameter list */
  int32_t device;
  int32_t buffers;             /* ZT_HAS_* bits: optional buffers present on every tensor */
  int32_t props;               /* ZT_PLAN_* bits: layout properties every tensor shares */
  int32_t reserved;
} zt_plan;

#define ZT_HAS_LIVE 1
#define ZT_HAS_M 2
#define ZT_HAS_V 4
#define ZT_HAS_ANCHOR 8
#define ZT_HAS_GE 16

/* zt_plan.props. With VEC8 and one uniform dtype, zt_pass runs the pass shapes that
 * dominate a step (one or two plain noise streams; the restore + grad_est accumulate +
 * next-perturb pass) through kernels specialised for that dtype. Results are identical. */
#define ZT_PLAN_VEC8 1       /* every numel a multiple of 8, every present buffer 16-byte aligned */
#define ZT_PLAN_ALL_F32 2
#define ZT_PLAN_ALL_BF16 4
#define ZT_PLAN_ALL_F16 8

#define ZT_UNIT_ELEMS 2048

/* Bytes of device workspace zt_plan_init needs for n_tensors tensors. */
ZT_API size_t zt_plan_workspace_bytes(int32_t n_tensors);

/* Validate `host_tensors`, copy them and their work-unit prefix into `workspace`
 * (device memory of at least zt_plan_workspace_bytes(n_tensors), 16-byte aligned)
 * and fill `plan`. The workspace must outlive every pass that uses the plan. */
ZT_API int zt_plan_init(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params,
                 void* workspace, size_t workspace_bytes, zt_plan* plan, void* stream);

/* ---- the fused pass ----------------------------------------------------------------- */

/* Roles of a noise stream inside one pass (flags). */
#define ZT_STREAM_GE 1   /* contributes ge_coef * z to the gradient estimate */
#define ZT_STREAM_MOM 2  /* contributes mom_coef * z to the reconstructed momentum */
#define ZT_STREAM_GE_DEV 4 /* with ZT_STREAM_GE: ge_coef is computed on the device from
                              cfg->dev_vals (see zt_pass_cfg) instead of taken from ge_coef */
/* Noise cache (cfg->zcache). The Gaussian field costs far more to regenerate (Philox4x32-10,
 * log, cos and sqrt per element) than an fp32 read from HBM, so a pair's field can be
 * written once and read back by the later passes of the same pair. */
#define ZT_STREAM_Z_STORE 8  /* the regenerated z is also written to cfg->zcache */
#define ZT_STREAM_Z_LOAD 16  /* z is read from cfg->zcache instead of regenerated; the cache
                                must hold this stream's field (stored by an earlier pass with
                                the same seed and plan; the library cannot check this) */
#define ZT_STREAM_Z_FIELD 32 /* z is read from slot `zslot` of the field store cfg->zfield
                                instead of regenerated; the store must hold this stream's field
                                on the pass's unit range (the library cannot check this) */

/* One noise stream: z = the Gaussian field of pair seed `seed`. Streams are applied in
 * array order. For each stream, the n_chain perturbations theta <- theta + chain[c] * z
 * (rounded to the parameter dtype after each) come first, then its GE / MOM roles. */
typedef struct zt_stream {
  uint64_t seed;
  float chain[ZT_MAX_CHAIN];
  int32_t n_chain;
  float ge_coef;
  float mom_coef;
  int32_t flags;
  int32_t zslot;   /* ZT_STREAM_Z_FIELD: slot of this stream's field in cfg->zfield, [0, 65535] */
} zt_stream;

/* gradient-estimate accumulation modes */
#define ZT_GE_NONE 0
#define ZT_GE_PRODUCT 1  /* ge = z * coef in fp32 (one stream; zotitan/train_zo.py:552) */
#define ZT_GE_ACCUM 2    /* ge = 0; ge += coef * z rounded to the param dtype (:555-556, :575-577) */

/* first-moment backends (MomentumConfig.momentum_method) */
#define ZT_MOM_NONE 0
#define ZT_MOM_STORED_EMA 1
#define ZT_MOM_SEED_WINDOW 2

/* weight decay (WeightDecayConfig) */
#define ZT_WD_NONE 0
#define ZT_WD_STANDARD 1
#define ZT_WD_ANCHORED_L2 2
#define ZT_WD_ANCHORED_L1 3

/* source / destination buffers of theta */
#define ZT_BUF_DATA 1
#define ZT_BUF_LIVE 2

/* Scalars are fp32 values the caller has already rounded the way torch's
 * CUDA kernels round a Python scalar (fp32 opmath). */
typedef struct zt_pass_cfg {
  int32_t src;          /* ZT_BUF_DATA or ZT_BUF_LIVE: where theta is read */
  int32_t dst;          /* bitmask of ZT_BUF_DATA | ZT_BUF_LIVE: where theta is written */
  int32_t ge_mode;      /* ZT_GE_* */
  int32_t ge_scale_on;  /* multiply ge by ge_scale after accumulation (norm clipping, :457) */
  float ge_scale;
  int32_t momentum;     /* ZT_MOM_*; requires update */
  float beta1;          /* stored EMA: m <- m*beta1; m <- m + one_minus_beta1*ge (:418-419) */
  float one_minus_beta1;
  float m_scale;        /* stored EMA: m_t = m * m_scale, m_scale = fp32(1/fp32(1-beta1^t+denom_eps)):
                         torch's CUDA tensor/scalar division multiplies by the reciprocal (:331) */
  int32_t second_moment;
  float beta2;          /* v <- v*beta2; v <- v + one_minus_beta2*ge*ge (:424-425) */
  float one_minus_beta2;
  float bc2;            /* fp32(1 - beta2^t) (:393) */
  float denom_eps;      /* (:396) */
  int32_t update;       /* apply the parameter update (:376-407) */
  float lr;             /* fp32(lr) */
  int32_t wd;           /* ZT_WD_* */
  float wd_lam;         /* fp32(fp32(lambda) * lr) (:390) */
  float wd_factor;      /* fp32(1 - wd_lam) (:402) */
  /* Gradient-estimate buffer (ZT_GE_ACCUM only): ge_load starts ge from the tensors' ge
   * buffers instead of zero; ge_store writes ge back after the streams. */
  int32_t ge_load;
  int32_t ge_store;
  /* Device-side coefficient of a ZT_STREAM_GE_DEV stream, from the pair's two values
   * v+ = dev_vals[0], v- = dev_vals[1] (device fp32), with the reference's arithmetic:
   *   pg = fp32(v+ - v-) * dev_inv2eps           (train_zo.py:544, CUDA scalar division)
   *   pgc = clamp(pg, -dev_tau, dev_tau)          (:545; dev_tau = +inf when not clipping)
   *   coef = pgc * dev_invz                       (:556, alpha = pgc / z_batch)
   * so passes can accumulate grad_est before the host has read any value. */
  const float* dev_vals;
  float dev_inv2eps;
  float dev_invz;
  float dev_tau;
  int32_t reserved;
  /* Work-unit range [unit_begin, unit_end) of the plan this pass covers; unit_end <= 0
   * means every unit. Units number the plan's tensors' 2048-element blocks in table
   * order, so a range is a contiguous slice when tensors are laid out back to back with
   * each padded to a multiple of ZT_UNIT_ELEMS (the sharded update splits the last pass
   * of a step this way across ranks). */
  int64_t unit_begin;
  int64_t unit_end;
  /* Noise cache for ZT_STREAM_Z_STORE / ZT_STREAM_Z_LOAD streams: plan->n_units *
   * ZT_UNIT_ELEMS fp32, 16-byte aligned, caller-owned; unit u's elements sit at
   * zcache[u * ZT_UNIT_ELEMS ...] (a tensor's last unit is padded). At most one stream
   * of a pass loads and at most one stores, and the loading stream comes first, so a
   * pass may read pair j's field and replace it with pair j+1's in place. NULL when no
   * stream uses it. */
  float* zcache;
  /* Field store for ZT_STREAM_Z_FIELD streams: fields of the pass's unit range only.
   * Unit u of the pass (unit_begin <= u < unit_end) of slot s sits at
   *   zfield[s * zfield_stride + (u - unit_begin) * ZT_UNIT_ELEMS ...]
   * (fp32, 16-byte aligned, zfield_stride a multiple of 4 and at least the range's
   * (unit_end - unit_begin) * ZT_UNIT_ELEMS). The seed-sharded step fills it with the
   * slices of every pair's field that fall on a rank's share of the parameters (pushed by
   * the ranks' +eps passes, zpush below, or copied from their noise caches with
   * zt_copy_async), so its last pass reads every field instead of regenerating it. NULL
   * when no stream uses it. */
  const float* zfield;
  int64_t zfield_stride;
  /* Push of a stored field into the ranks' field stores, from the pass that generates it
   * (zpush_ranks > 0): the ZT_STREAM_Z_STORE stream's field is also written, unit by unit,
   * to the store of the rank that owns the unit, over peer memory (zt_ipc_open mappings):
   * for a flat layout of `zpush_ranks` ranks cut into chunks of zpush_ranks * C units
   * (C = zpush_chunk_units; in chunk k rank p owns units [k*R*C + p*C, k*R*C + (p+1)*C)),
   * unit u of chunk k, offset o in rank p's part, goes to
   *   zpush[p][zpush_slot * zpush_stride + (k * C + o) * ZT_UNIT_ELEMS ...]
   * followed by a system-scope fence. Only the specialised +eps pass (one storing stream,
   * a plan of one dtype with ZT_PLAN_VEC8) takes it; other passes are rejected. */
  float* zpush[ZT_MAX_PUSH_RANKS];
  int32_t zpush_ranks;
  int32_t zpush_slot;
  int64_t zpush_chunk_units;
  int64_t zpush_stride;
} zt_pass_cfg;

/* A pass is rejected (ZT_ERR_INVALID) when cfg reads or writes a buffer (live, m, v,
 * anchor) that some tensor of the plan lacks. Optional buffers must have their
 * tensor's numel and dtype; the library cannot check sizes.
 *
 * One fused pass over every element of every tensor of `plan`:
 *   1. theta = src buffer;
 *   2. for each stream in order: regenerate z in registers (or read it from the noise
 *      cache, ZT_STREAM_Z_LOAD, or from the field store, ZT_STREAM_Z_FIELD), apply its
 *      chain to theta, accumulate its ge / momentum contributions (noise is written to
 *      memory only for a ZT_STREAM_Z_STORE stream);
 *   3. optional ge scaling, optimizer state (m, v) update and parameter update with
 *      weight decay, in the reference's op order (zotitan/train_zo.py:409-425, 376-407);
 *   4. theta to every buffer in `dst`.
 * Replaces, per call, any run of _apply_z (:350-351), the grad_est accumulation
 * (:550-556, :575-577), _update_optimizer_state (:409-425), _get_gradient_ema (:324-346)
 * and _apply_update (:376-407) that the caller fuses. */
ZT_API int zt_pass(const zt_plan* plan, const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams,
            void* stream);

/* ---- EGGROLL population linear layer -------------------------------------------- */

/* One linear layer of a population forward in which member i's weight is perturbed by a
 * rank-4 term: W + sigma_i * A_i B_i^T. With X holding all members' activations (member i
 * owns rows [i*rows_per_member, (i+1)*rows_per_member)):
 *   Y[m, :] = X[m, :] W^T + sigma_i * (X[m, :] B_i) A_i^T,   i = m / rows_per_member.
 * The base GEMM runs on tcgen05 tensor cores (bf16 in, fp32 accumulate, bf16 out); the
 * rank-4 term is added in the GEMM epilogue, so W is shared and never copied per member.
 * The reference has no EGGROLL implementation (it is only named in README.md:11); the
 * perturbation follows its low-rank branch, z = P Psi (zotitan/train_zo.py:304-320),
 * with A_i = P and B_i = Psi^T and the normalisation folded into sigma_i. */
typedef struct zt_eggroll_args {
  const void* x;          /* [m, k] bf16, row-major, 16-byte aligned */
  const void* w;          /* [n, k] bf16, row-major (the layer's weight as torch stores it) */
  const float* a;         /* [members, n, 4] fp32: A_i */
  const float* b;         /* [members, k, 4] fp32: B_i */
  const float* sigma;     /* [members] fp32: signed per-member scale */
  float* xb;              /* [m, 4] fp32 workspace, written by the call: X B_i */
  void* y;                /* [m, n] bf16 output */
  int64_t m, n, k;        /* m % 128 == 0, n % 256 == 0, k % 64 == 0 */
  int32_t rows_per_member;  /* multiple of 128 dividing m */
  int32_t rank;           /* must be 4 */
  int32_t xb_ready;       /* nonzero: xb already holds X B_i (zt_eggroll_xb) and is only read */
  int32_t test_stall_loads; /* test hook, 0 in normal use: the GEMM's loader issues no copies, so
                               its first wait for a loaded stage expires (~2 s) with nothing in
                               flight and the call reports it through zt_eggroll_take_error */
  /* Optional rank-4 K-slab (both non-NULL: a, b, sigma, xb are not read). The correction
   * sigma_i (X B_i) A_i^T then runs on the tensor cores as one extra K = 16 MMA per tile:
   * x_ext [m, 16] bf16 rows [hi(sigma_i X B_i), lo(sigma_i X B_i), 0 x 8] (zt_eggroll_xb,
   * hi + lo = the fp32 value to ~2^-16), w_ext [members, n, 16] bf16 rows [A_i, A_i, 0 x 8]
   * (zt_eggroll_factors). Needs m % 256 == 0 and rows_per_member % 256 == 0. */
  const void* x_ext;
  const void* w_ext;
} zt_eggroll_args;

ZT_API int zt_eggroll_linear(const zt_eggroll_args* args, void* stream);

/* X B_s for up to three factor sets that share the activations X (q/k/v projections,
 * or gate/up), in one read of X: xb[s][m, :] = X[m, :] B_{s,i}, i = m / rows_per_member,
 * fp32. The outputs feed zt_eggroll_linear with xb_ready = 1. */
typedef struct zt_eggroll_xb_args {
  const void* x;          /* [m, k] bf16, 16-byte aligned */
  const float* b[3];      /* per set: [members, k, 4] fp32 (entries >= n_seg unused) */
  float* xb[3];           /* per set: [m, 4] fp32 out (NULL: not written) */
  int64_t m, k;           /* m % 64 == 0, k % 4 == 0 */
  int32_t n_seg;          /* 1, 2 or 3 */
  int32_t rows_per_member;  /* multiple of 64 dividing m */
  const float* sigma[3];  /* per set: [members] signed scale, read when xe[s] is set */
  void* xe[3];            /* per set: optional [m, 16] bf16 K-slab rows of sigma_i X B (NULL: skip) */
  int32_t xe_slot[3];     /* 0: write [hi, lo, 0 x 8]; 1: write [hi, lo] to columns 0-7; 2: to 8-15 */
  int32_t reserved;
  /* Optional: all sets' B_s^T as one bf16 [members, 16, k] tensor (set s in rows 4s..4s+3,
   * the other rows zero; zt_eggroll_factors.b_ext). Then X B runs on the tensor cores
   * (N = 16 per 128-row tile) and b[] is not read; needs m, rows_per_member % 128 == 0 and
   * k % 64 == 0. */
  const void* bt;
} zt_eggroll_xb_args;

ZT_API int zt_eggroll_xb(const zt_eggroll_xb_args* args, void* stream);

/* The Llama MLP's gated product of a population chunk in one GEMM:
 *   G = X W_gate^T + sigma_gate_i (X B_gate,i) A_gate,i^T,  U likewise with the up factors,
 *   y = bf16(bf16(silu(bf16(G))) * bf16(U)),  silu(g) = g / (1 + exp(-g)),
 * the rounding torch applies to act_fn(gate_proj(x)) * up_proj(x) in bf16. G and U are
 * never written: a pair of CTAs computes both for the same 128 features and the epilogue
 * combines them. xb_gate / xb_up come from zt_eggroll_xb (one pass over X for both). */
typedef struct zt_eggroll_gated_args {
  const void* x;          /* [m, k] bf16 */
  const void* w_gate;     /* [n, k] bf16 */
  const void* w_up;       /* [n, k] bf16 */
  const float* a_gate;    /* [members, n, 4] */
  const float* a_up;      /* [members, n, 4] */
  const float* sigma_gate;  /* [members] */
  const float* sigma_up;    /* [members] */
  const float* xb_gate;   /* [m, 4] */
  const float* xb_up;     /* [m, 4] */
  void* y;                /* [m, n] bf16 out */
  int64_t m, n, k;        /* m % 256 == 0, n % 128 == 0, k % 64 == 0 */
  int32_t rows_per_member;  /* multiple of 128 dividing m */
  int32_t rank;           /* must be 4 */
  /* Optional K-slab form of both corrections (all three non-NULL; rows_per_member % 256
   * == 0): x_ext rows [hi_g, lo_g, hi_u, lo_u] (zt_eggroll_xb slots 1 and 2), w_ext_gate
   * rows [A_g, A_g, 0 x 8], w_ext_up rows [0 x 8, A_u, A_u] (zt_eggroll_factors slots 0, 1). */
  const void* x_ext;
  const void* w_ext_gate;
  const void* w_ext_up;
} zt_eggroll_gated_args;

ZT_API int zt_eggroll_gated(const zt_eggroll_gated_args* args, void* stream);

/* Reads and clears the device-side error code of the EGGROLL kernels (0: none; nonzero:
 * a bounded wait inside the GEMM expired and that launch returned early). Synchronous. */
ZT_API int zt_eggroll_take_error(int32_t* code);

/* ---- EGGROLL population forward: factors and element-wise layers ------------------ */

#define ZT_EGGROLL_MAX_PAIRS 512
#define ZT_EGGROLL_FACTOR_BLOCKS 64
#define ZT_EGGROLL_FACTOR_WORK_FLOATS (ZT_EGGROLL_FACTOR_BLOCKS * 20) /* workspace floats per pair */

/* The rank-4 factors of one 2-D tensor [n, k] for a chunk of antithetic pairs: pair j
 * gives members 2j (+sigma) and 2j+1 (-sigma). Replaces the low_rank branch of
 * _sample_z (zotitan/train_zo.py:304-320) for the population forward:
 *   P   = randn(keys_a[j], n*4).view(n, 4)  rounded to dtype  -> A_{2j} = A_{2j+1} = P
 *   Psi = randn(keys_b[j], 4*k).view(4, k)  rounded to dtype  -> B_{2j} = B_{2j+1} = Psi^T
 *   c_j = sqrt(n*k) / (||P Psi||_F + 1e-7), the norm, the sum and the quotient each
 *         rounded to dtype as the reference evaluates them,
 *   scale[2j] = sigma * c_j, scale[2j+1] = -sigma * c_j.
 * The outputs are zt_eggroll_linear's a, b and sigma operands. ||P Psi||_F^2 is
 * evaluated as sum_{r,s} (P^T P)_{rs} (Psi Psi^T)_{rs} from fixed-order partial sums
 * (deterministic); the reference takes the norm of the rounded product P Psi. */
typedef struct zt_eggroll_factor_args {
  const uint32_t* keys_a; /* host [pairs]: key of P = zt_param_key(seed, n_params, index + 2*n_params) */
  const uint32_t* keys_b; /* host [pairs]: key of Psi = zt_param_key(seed, n_params, index + n_params) */
  int32_t pairs;          /* 1 .. ZT_EGGROLL_MAX_PAIRS */
  int32_t rank;           /* must be 4 */
  int64_t n, k;           /* the weight's out_features and in_features; 4*n, 4*k <= ZT_MAX_NUMEL */
  int32_t dtype;          /* parameter dtype (ZT_F32 / ZT_BF16 / ZT_F16) */
  int32_t normalize;      /* 0: c_j = 1 */
  float sigma;
  int32_t reserved;
  float* a;               /* out [2*pairs, n, 4] fp32, 16-byte aligned */
  float* b;               /* out [2*pairs, k, 4] fp32, 16-byte aligned */
  float* scale;           /* out [2*pairs] fp32 */
  float* work;            /* workspace: pairs * ZT_EGGROLL_FACTOR_WORK_FLOATS floats */
  void* a_ext;            /* optional out [2*pairs, n, 16] bf16: A as the B operand of the GEMM's
                             rank-4 K-slab (see zt_eggroll_args.w_ext); NULL to skip */
  int32_t ext_slot;       /* a_ext row: 0 = [A, A, 0 x 8], 1 = [0 x 8, A, A] */
  int32_t reserved2;
  void* b_ext;            /* optional out, rows of [2*pairs, 16, k] bf16: B^T written to rows
                             b_ext_row .. b_ext_row+3 of each member (zt_eggroll_xb.bt); other
                             rows untouched (the caller zeroes the buffer once); NULL to skip */
  int32_t b_ext_row;      /* 0, 4 or 8 */
  int32_t reserved3;
  /* Keys from device memory instead (keys_a / keys_b then unused): with seeds non-NULL,
   * pair j's keys are zt_param_key(seeds[j], n_params, key_index_a / key_index_b),
   * computed by the kernel. Lets a captured CUDA graph be replayed for new pairs after
   * a copy of their seeds into `seeds`. */
  const uint64_t* seeds;  /* device [pairs] pair seeds, or NULL */
  uint32_t n_params;
  uint32_t key_index_a;   /* index + 2*n_params of the tensor (P) */
  uint32_t key_index_b;   /* index + n_params (Psi) */
  int32_t reserved4;
} zt_eggroll_factor_args;

ZT_API int zt_eggroll_factors(const zt_eggroll_factor_args* args, void* stream);

/* Llama RMSNorm of a population chunk with member-perturbed weights (a 1-D tensor gets
 * full Gaussian noise, zotitan/train_zo.py:303, applied as p + alpha*z, :350-351):
 *   w_members[2j]   = bf16(w + sigma * z_j),  w_members[2j+1] = bf16(w - sigma * z_j),
 *   z_j[t] = randn(keys[j], t) (fp32),
 *   y[r] = w_members[r / rows_per_member] * bf16(x[r] * rsqrt(mean(x[r]^2) + eps))
 * in fp32 with bf16 rounding where the transformers LlamaRMSNorm on bf16 rounds. All
 * tensors bf16, rows contiguous, d % 8 == 0, m == rows_per_member * 2 * pairs. */
typedef struct zt_eggroll_norm_args {
  const void* x;          /* [m, d] bf16, 16-byte aligned */
  const void* w;          /* [d] bf16: the norm's unperturbed weight */
  const uint32_t* keys;   /* host [pairs]: zt_param_key(seed, n_params, index) */
  void* w_members;        /* [2*pairs, d] bf16 workspace, written by the call */
  void* y;                /* [m, d] bf16 out (may not alias x) */
  int64_t m, d;
  int32_t pairs;
  int32_t rows_per_member;
  float sigma;
  float eps;
  const uint64_t* seeds;  /* device [pairs] pair seeds, or NULL: with seeds, keys[j] =
                             zt_param_key(seeds[j], n_params, key_index) on the device */
  uint32_t n_params;
  uint32_t key_index;
} zt_eggroll_norm_args;

ZT_API int zt_eggroll_rmsnorm(const zt_eggroll_norm_args* args, void* stream);

/* Llama RMSNorm of x [rows, d] with one weight w [d] (bf16, d % 8 == 0, 16-byte aligned):
 *   y = w * bf16(x * rsqrt(mean(x^2) + eps)),
 * the mean and rsqrt in fp32 (transformers' LlamaRMSNorm.forward on bf16 tensors; only
 * the summation order of a row's squares differs). Replaces that module's forward in a
 * no-grad decoder pass. */
ZT_API int zt_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t d, float eps, void* stream);

/* In-place rotary position embedding of q [rows, q_heads*head_dim] and k [rows,
 * k_heads*head_dim] (bf16, rows contiguous; row r is at position r % seq):
 *   x = x * cos[pos] + rotate_half(x) * sin[pos],  cos, sin [seq, head_dim] bf16,
 * each product and the sum rounded to bf16 (apply_rotary_pos_emb of transformers'
 * Llama on bf16 tensors). head_dim % 16 == 0. */
ZT_API int zt_eggroll_rope(void* q, void* k, const void* cos, const void* sin, int64_t rows, int32_t seq,
                           int32_t q_heads, int32_t k_heads, int32_t head_dim, void* stream);

/* out = bf16(bf16(silu(gate)) * up) over n bf16 elements (n % 8 == 0): the Llama MLP's
 * act_fn(gate_proj(x)) * up_proj(x). */
ZT_API int zt_eggroll_swiglu(const void* gate, const void* up, void* out, int64_t n, void* stream);

/* y [m, n] = bf16(bf16(silu(bf16(x w_gate^T))) * bf16(x w_up^T)) for bf16 x [m, k],
 * w_gate, w_up [n, k] (row-major, 16-byte aligned; m % 256 == 0, n % 128 == 0,
 * k % 64 == 0): the gate and up projections and the SwiGLU of an unperturbed Llama MLP
 * (act_fn(gate_proj(x)) * up_proj(x)) as one tcgen05 GEMM over CTA pairs, the SwiGLU in
 * its epilogue; the rounding points are those of the three torch ops, the fp32
 * accumulation order is the kernel's. */
ZT_API int zt_gemm_swiglu(const void* x, const void* w_gate, const void* w_up, void* y, int64_t m, int64_t n,
                          int64_t k, void* stream);

/* Operands of the EGGROLL evolution-strategies update of one 2-D tensor [n, k] over
 * `pairs` antithetic pairs, from zt_eggroll_factors' a, b, scale (members 2j):
 *   a_cat [n, 8*pairs] bf16: row o, pair j -> [hi(v), lo(v)], v = coef_j (scale_2j / sigma) A_2j[o]
 *   b_cat [k, 8*pairs] bf16: row t, pair j -> [B_2j[t], B_2j[t]]
 * so that a_cat b_cat^T = sum_j coef_j c_j P_j Psi_j to ~2^-16 relative: the update
 * theta -= lr * sum_j coef_j z_j of the reference's low_rank directions (zotitan/train_zo.py:
 * 304-320, 550-556) as one GEMM of inner dimension 8 * pairs. */
ZT_API int zt_eggroll_update_operands(const float* a, const float* b, const float* scale, const float* coef,
                                      int32_t pairs, int64_t n, int64_t k, float sigma, void* a_cat, void* b_cat,
                                      void* stream);

/* w[i, j] <- bf16(w[i, j] + alpha * sum_t a[i, t] b[j, t]) for w [m, n] bf16 (row stride ldw,
 * a multiple of 8), a [m, k] and b [n, k] bf16 row-major (k % 64 == 0, n % 32 == 0, all
 * 16-byte aligned): the product on the tensor cores with fp32 accumulation, w read, updated
 * with one fused multiply-add and rounded once in the epilogue. With a = a_cat, b = b_cat of
 * zt_eggroll_update_operands and alpha = -lr it is the evolution-strategies update
 * theta -= lr * sum_j coef_j z_j of a 2-D tensor (zotitan/train_zo.py:550-556, 376-407 with
 * the low_rank directions of :304-320). */
ZT_API int zt_gemm_addto(void* w, int64_t ldw, const void* a, const void* b, float alpha, int64_t m, int64_t n,
                         int64_t k, void* stream);

/* Reads and clears zt_gemm_addto's device error flag (nonzero: a bounded wait inside the
 * GEMM expired and w is partly updated). Synchronises with the device. */
ZT_API int zt_gemm_take_error(int32_t* code);

/* The tail of a LoRA linear (zotitan/lora.py:77-86) in one pass over the output:
 *   out[t, c] = bf16(out[t, c] + bf16(scale * sum_r xa[t, r] b[c, r]))
 * with out [rows, n] bf16 holding the base layer's output (updated in place), xa [rows, r]
 * fp32 = lora_A(x) and b [n, r] fp32 = lora_B.weight. r in {4, 8, 16, 32, 64}; xa and b
 * row-major and contiguous. For r in {8, 16}, n % 8 == 0 and 16-byte aligned out and xa the
 * sum runs on the tensor cores (mma.sync on TF32 with each fp32 operand split into a hi
 * and a lo part, three products: ~2^-22 relative before the bf16 rounding); otherwise in
 * fp32 FMAs over r in order. */
ZT_API int zt_lora_add(void* out, const float* xa, const float* b, float scale, int64_t rows, int64_t n, int32_t r,
                       void* stream);

/* zt_lora_add with xa given as three partial products xa3 [rows, 3r] fp32 (the columns of
 * x [A0; A1; A2]^T for the split of zt_lora_split), summed in fp32 as ((p0 + p1) + p2)
 * while the kernel stages them: the fp32 x A^T of the reference's lora_A(x.float()). */
ZT_API int zt_lora_add3(void* out, const float* xa3, const float* b, float scale, int64_t rows, int64_t n, int32_t r,
                        void* stream);

/* Three bf16 parts of an fp32 array that sum to it exactly: out [3, n] bf16 with
 * out[0] = bf16(a), out[1] = bf16(a - out[0]), out[2] = bf16(a - out[0] - out[1]) (fp32
 * differences), so a tensor-core product against [out[0]; out[1]; out[2]] gives the fp32
 * product's terms exactly (the LoRA A operand). */
ZT_API int zt_lora_split(const float* a, void* out, int64_t n, void* stream);

/* ---- the scorer: next-token cross-entropy statistics ------------------------------ */

/* Per-row statistics of bf16 logits [rows, vocab] (row stride ld elements, ld % 8 == 0,
 * 16-byte aligned) against int64 targets[rows] (negative = ignored):
 *   lse[r]     = log(sum_v exp(x[r, v]))        (fp32, max-shifted; the z-loss term)
 *   loss[r]    = -((x[r, t] - max_r) - log(sum_v exp(x[r, v] - max_r)))
 *   correct[r] = (first argmax of x[r, :] == t)
 * as torch's cross_entropy / logsumexp / argmax evaluate them on the fp32 upcast of the
 * logits (zotitan/losses.py:55-79; transformers' ForCausalLMLoss). Ignored rows get
 * 0 in all three; a target >= vocab gives NaN. lse and correct may be NULL. Replaces the
 * reference's Liger fused cross-entropy (zotitan/losses.py:17-52) after the lm_head GEMM. */
ZT_API int zt_xent_rows(const void* logits, int64_t ld, int64_t rows, int64_t vocab, const int64_t* targets,
                        float* loss, float* lse, int32_t* correct, void* stream);

/* ---- the scorer: fused linear cross-entropy --------------------------------------- */

/* Arguments of zt_linear_xent. */
typedef struct zt_lce_args {
  const void* x;           /* [rows, k] bf16 hidden states, row-major, 16-byte aligned */
  const void* w;           /* [vocab, k] bf16 lm_head weight (torch's [out, in]), 16-byte aligned */
  const int64_t* targets;  /* [rows] target token ids; negative = ignored position */
  float* loss;             /* [rows] out */
  float* lse;              /* [rows] out, or NULL */
  int32_t* correct;        /* [rows] out, or NULL */
  void* workspace;         /* zt_linear_xent_workspace_bytes(rows, vocab, k) bytes, 16-byte aligned */
  size_t workspace_bytes;
  int64_t rows, vocab, k;  /* k a multiple of 64 */
  /* Test hooks, 0 in normal use. With test_stall_loads the GEMM's loader issues no copies,
   * so the first wait for a loaded stage expires (after test_wait_cycles clock cycles; 0:
   * the default bound of ~2 s) with no copy and no MMA in flight: the kernel records the
   * expiry (zt_linear_xent_take_error), frees its tensor memory and returns, and the
   * outputs are incomplete. It exercises the abort path without a fault. */
  int32_t test_stall_loads;
  int32_t reserved;
  int64_t test_wait_cycles;
} zt_lce_args;

/* The lm_head GEMM and the cross-entropy statistics of zt_xent_rows in one pass, without
 * writing the logits: logits[r, v] = bf16(x[r, :] . w[v, :]) (fp32 accumulation on the
 * tensor cores, one rounding to bf16, as the reference's bf16 lm_head produces them), and
 * from them lse, loss and correct exactly as zt_xent_rows defines them (ignored rows 0 in
 * all three, a target >= vocab gives NaN). Replaces the Liger fused linear cross-entropy
 * of zotitan/losses.py:17-52 (and the lm_head + torch cross-entropy of :55-79). The
 * workspace holds per-row partial statistics of vocabulary splits; its size depends on
 * the current device's SM count. */
ZT_API size_t zt_linear_xent_workspace_bytes(int64_t rows, int64_t vocab, int64_t k);
ZT_API int zt_linear_xent(const zt_lce_args* args, void* stream);

/* Reads and clears the fused scorer's device error flag (nonzero: a bounded wait inside
 * the GEMM expired; its outputs are then incomplete). Synchronises with the device. */
ZT_API int zt_linear_xent_take_error(int32_t* code);

/* ---- low-rank directions (distribution "low_rank") on the tensor cores ----------- */

/* Replaces the materialised direction of _sample_z for a 2-D parameter
 * (zotitan/train_zo.py:295-322): P = randn(key_p, m r).view(m, r).to(dtype),
 * Psi = randn(key_psi, r n).view(r, n).to(dtype), z = P @ Psi, then
 * z * (sqrt(m n) / (||z||_F + 1e-7)), and its uses in _apply_z (:350-351) and the grad
 * estimate (:550-556, :575-577), without z ever being written to memory. One parameter of
 * dtype ZT_BF16, ZT_F16 or ZT_F32 at a time, for n_streams pair seeds at once. The product
 * is the fp32 sum of exact products in K order, rounded to the dtype: an element can differ
 * by one unit in the last place from a library GEMM that sums in another order. The
 * tensor cores take 16-bit operands: for ZT_F32 the factor buffers hold bf16 values, each
 * fp32 factor split exactly into three bf16 parts, and the nine cross products of the
 * parts laid out along K (block (a, b) of width r holds part a of P and part b of Psi),
 * which sum to the fp32 product P Psi. The polar distribution's factors (:307-317, QR and
 * Newton-Schulz) come from the caller (factors_given). */
#define ZT_LOWRANK_MAX_STREAMS 128

typedef struct zt_lowrank_desc {
  int64_t m, n;     /* parameter shape, row-major, contiguous */
  int32_t r;        /* rank used: min(rank, m); 1 <= r <= kp */
  int32_t kp;       /* padded K: a multiple of 64, at most 1024 (>= r; >= 9 r for ZT_F32 factors from keys) */
  int32_t dtype;    /* ZT_BF16, ZT_F16 or ZT_F32: the parameter's */
  int32_t n_streams; /* 1..ZT_LOWRANK_MAX_STREAMS */
  uint32_t keys_p[ZT_LOWRANK_MAX_STREAMS];   /* noise key of P per stream: position i + 2N (:311) */
  uint32_t keys_psi[ZT_LOWRANK_MAX_STREAMS]; /* noise key of Psi per stream: position i + N (:315) */
  void* p;          /* device [n_streams * m, kp] 16-bit (bf16 for ZT_F32), 16-byte aligned: P of each stream, zero-padded */
  void* psi_t;      /* device [n_streams * n, kp], same type: Psi transposed, zero-padded */
  float* scale;     /* device [n_streams]: the dtype-rounded scale of each stream's product */
  void* workspace;  /* device, zt_lowrank_workspace_bytes, 16-byte aligned (zt_lowrank_prepare) */
  size_t workspace_bytes;
  int32_t factors_given; /* 1: p and psi_t already hold the factors (written by the caller in the
                            layout above); zt_lowrank_prepare then only computes the scales */
  int32_t reserved;
} zt_lowrank_desc;

typedef struct zt_lowrank_apply_args {
  const void* src;  /* parameter read by stream 0 (later streams read dst); may equal dst */
  void* dst;        /* parameter written; NULL: the parameter is not updated (n_alpha 0) */
  void* ge;         /* grad estimate [m, n] dtype, or NULL */
  int32_t n_alpha;  /* 0..3: per stream, theta <- round(theta + alpha[t] z) for t < n_alpha */
  float alpha[3];
  int32_t ge_init;  /* 1: stream 0 sets ge = round(coef[0] z); else every stream adds round(ge + coef z) */
  float coef[ZT_LOWRANK_MAX_STREAMS]; /* grad-estimate coefficient per stream */
  int32_t test_stall_loads; /* test hook: the loader issues no copies, every wait expires (0 normally) */
  int32_t reserved;
  int64_t test_wait_cycles; /* bound of each wait in clock cycles; 0: about two seconds */
} zt_lowrank_apply_args;

ZT_API int zt_lowrank_workspace_bytes(int64_t m, int64_t n, int32_t n_streams, size_t* bytes);

/* Writes d->p, d->psi_t and d->scale: the factors of every stream from the noise source,
 * then the product's sum of squares (tensor cores, the product never stored) and the
 * scale in torch's op order on the dtype: round(sqrt(ss)), + 1e-7, reciprocal,
 * * sqrt(m n), each rounded. Deterministic (fixed summation order). */
ZT_API int zt_lowrank_prepare(const zt_lowrank_desc* d, void* stream);

/* For each tile of the parameter and each stream in order: z = round(round(P Psi) * scale),
 * theta <- round(theta + alpha z) for the chained coefficients, ge <- round(ge + coef z).
 * Uses the factors and scales of a zt_lowrank_prepare on the same descriptor. */
ZT_API int zt_lowrank_apply(const zt_lowrank_desc* d, const zt_lowrank_apply_args* a, void* stream);

/* Reads and clears the low-rank GEMMs' device error flag (nonzero: a bounded wait
 * expired and the call's outputs are incomplete). Synchronises with the device. */
ZT_API int zt_lowrank_take_error(int32_t* code);

/* ---- peer mappings for the sharded step's field exchange ------------------------- */

/* The reference runs one process per GPU with no communication (sweeps/runall.py:5), so
 * these have no counterpart there. In the seed-sharded step (one process per GPU) each
 * rank pushes the slices of its own pairs' Gaussian fields into the field stores
 * (zt_pass_cfg.zfield) of the ranks that own those slices, so that the step's last pass
 * reads every pair's field instead of regenerating it. The stores are the caller's
 * device allocations (cudaMalloc-backed, e.g. torch's default allocator); these calls
 * only map them into another process and copy with the copy engines. */
#define ZT_IPC_HANDLE_BYTES 64

/* handle_out (ZT_IPC_HANDLE_BYTES) names the device allocation that contains `ptr`, and
 * offset_out is ptr's byte offset from that allocation's start. */
ZT_API int zt_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);

/* Map another process's allocation (a zt_ipc_export handle) into the current device's
 * address space, with peer access enabled; base_out is the allocation's start (add the
 * exporter's offset). Unmap with zt_ipc_close. */
ZT_API int zt_ipc_open(const void* handle, void** base_out);
ZT_API int zt_ipc_close(void* base);

/* cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream): device-to-device, either
 * side may be a peer mapping (zt_ipc_open); runs on the copy engines. */
ZT_API int zt_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* ---- the fused pass without a caller-provided workspace -------------------------- */

#define ZT_STATIC_MAX_TENSORS 1024

/* zt_pass for callers that cannot allocate device memory. This entry point has no
 * counterpart in the reference. It serves callers that cannot hand the library a
 * workspace: a process whose device memory is held by another allocator that reserved
 * it up front, or host code that must not call cudaMalloc/cudaFree while a step is in
 * flight (those calls synchronise the device and fragment the owner's memory pool).
 *
 * Instead of a zt_plan, it takes the host descriptor table directly, copies it into a
 * fixed array compiled into the library (about 64 KB, kept on every GPU that loads the
 * library until the process exits) and runs the same pass as zt_pass. At most
 * ZT_STATIC_MAX_TENSORS tensors per call; more are rejected with ZT_ERR_LIMIT. It calls
 * no cudaMalloc, cudaFree or other allocating routine.
 *
 * The first call on a device resolves the array's device address (once per device, with
 * that device current); make that first call before any stream capture. The address
 * belongs to the device's primary context: after cudaDeviceReset do not call this entry
 * point again in that process. Every call checks all its arguments first (a rejected
 * call leaves the array as it was), then copies its table into the same array, on
 * `stream`, before its pass; the array keeps the last call's table, so calls whose work
 * can overlap on the GPU (different streams, or unordered host threads on one device)
 * race on it. Order such calls on one stream. The copy goes through a host image owned
 * by the library, which the CUDA runtime stages before the call returns: the caller's
 * table, pinned or not, may be changed or freed as soon as the call returns. A stream
 * that is capturing is refused with ZT_ERR_INVALID (the copy would replay from that
 * reused host image). */
ZT_API int zt_pass_static(const zt_tensor* host_tensors, int32_t n_tensors, uint32_t n_params,
                          const zt_pass_cfg* cfg, const zt_stream* streams, int32_t n_streams, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ZOTITAN_B200_H */
