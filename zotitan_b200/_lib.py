"""ctypes binding of ``libzotitan_b200.so`` (the C ABI in include/zotitan_b200.h).

There is no fallback: if the library is missing or fails to load, every entry
point raises. Structures mirror the header field for field.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libzotitan_b200.so")

ZT_F32, ZT_BF16, ZT_F16 = 0, 1, 2
ZT_OK, ZT_ERR_INVALID, ZT_ERR_CUDA, ZT_ERR_LIMIT = 0, 1, 2, 3
ZT_MAX_STREAMS = 256
ZT_MAX_CHAIN = 3
ZT_MAX_NUMEL = 2**31 - 1
ZT_MAX_PUSH_RANKS = 8
ZT_UNIT_ELEMS = 2048
ZT_STREAM_GE, ZT_STREAM_MOM, ZT_STREAM_GE_DEV = 1, 2, 4
ZT_STREAM_Z_STORE, ZT_STREAM_Z_LOAD, ZT_STREAM_Z_FIELD = 8, 16, 32
ZT_GE_NONE, ZT_GE_PRODUCT, ZT_GE_ACCUM = 0, 1, 2
ZT_MOM_NONE, ZT_MOM_STORED_EMA, ZT_MOM_SEED_WINDOW = 0, 1, 2
ZT_WD_NONE, ZT_WD_STANDARD, ZT_WD_ANCHORED_L2, ZT_WD_ANCHORED_L1 = 0, 1, 2, 3
ZT_BUF_DATA, ZT_BUF_LIVE = 1, 2
ZT_PLAN_VEC8, ZT_PLAN_ALL_F32, ZT_PLAN_ALL_BF16, ZT_PLAN_ALL_F16 = 1, 2, 4, 8

# every function include/zotitan_b200.h declares
EXPORTS = ("zt_last_error", "zt_abi_version", "zt_param_key", "zt_philox_words", "zt_randn",
           "zt_randn_at", "zt_plan_workspace_bytes", "zt_plan_init", "zt_pass", "zt_pass_static",
           "zt_eggroll_linear", "zt_eggroll_take_error", "zt_randn_keys", "zt_eggroll_factors",
           "zt_eggroll_rmsnorm", "zt_eggroll_rope", "zt_eggroll_swiglu", "zt_xent_rows",
           "zt_eggroll_xb", "zt_eggroll_gated", "zt_eggroll_update_operands", "zt_lora_add", "zt_rmsnorm", "zt_gemm_swiglu", "zt_lora_add3", "zt_lora_split",
           "zt_ipc_export", "zt_ipc_open", "zt_ipc_close", "zt_copy_async",
           "zt_linear_xent_workspace_bytes", "zt_linear_xent", "zt_linear_xent_take_error",
           "zt_gemm_addto", "zt_gemm_take_error",
           "zt_lowrank_workspace_bytes", "zt_lowrank_prepare", "zt_lowrank_apply", "zt_lowrank_take_error")
ZT_STATIC_MAX_TENSORS = 1024
ZT_EGGROLL_MAX_PAIRS = 512
ZT_EGGROLL_FACTOR_WORK_FLOATS = 64 * 20
ABI_VERSION = 11
ZT_LOWRANK_MAX_STREAMS = 128
ZT_IPC_HANDLE_BYTES = 64


class ZtTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("live", ctypes.c_void_p), ("m", ctypes.c_void_p),
                ("v", ctypes.c_void_p), ("anchor", ctypes.c_void_p), ("ge", ctypes.c_void_p), ("numel", ctypes.c_int64),
                ("dtype", ctypes.c_int32), ("index", ctypes.c_int32)]


class ZtPlan(ctypes.Structure):
    _fields_ = [("tensors", ctypes.c_void_p), ("unit_prefix", ctypes.c_void_p), ("n_units", ctypes.c_int64),
                ("numel_total", ctypes.c_int64), ("n_tensors", ctypes.c_int32), ("n_params", ctypes.c_uint32),
                ("device", ctypes.c_int32), ("buffers", ctypes.c_int32), ("props", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class ZtStream(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("chain", ctypes.c_float * ZT_MAX_CHAIN), ("n_chain", ctypes.c_int32),
                ("ge_coef", ctypes.c_float), ("mom_coef", ctypes.c_float), ("flags", ctypes.c_int32),
                ("zslot", ctypes.c_int32)]


class ZtPassCfg(ctypes.Structure):
    _fields_ = [("src", ctypes.c_int32), ("dst", ctypes.c_int32), ("ge_mode", ctypes.c_int32),
                ("ge_scale_on", ctypes.c_int32), ("ge_scale", ctypes.c_float), ("momentum", ctypes.c_int32),
                ("beta1", ctypes.c_float), ("one_minus_beta1", ctypes.c_float), ("m_scale", ctypes.c_float),
                ("second_moment", ctypes.c_int32), ("beta2", ctypes.c_float), ("one_minus_beta2", ctypes.c_float),
                ("bc2", ctypes.c_float), ("denom_eps", ctypes.c_float), ("update", ctypes.c_int32),
                ("lr", ctypes.c_float), ("wd", ctypes.c_int32), ("wd_lam", ctypes.c_float),
                ("wd_factor", ctypes.c_float), ("ge_load", ctypes.c_int32), ("ge_store", ctypes.c_int32),
                ("dev_vals", ctypes.c_void_p), ("dev_inv2eps", ctypes.c_float), ("dev_invz", ctypes.c_float),
                ("dev_tau", ctypes.c_float), ("reserved", ctypes.c_int32), ("unit_begin", ctypes.c_int64),
                ("unit_end", ctypes.c_int64), ("zcache", ctypes.c_void_p), ("zfield", ctypes.c_void_p),
                ("zfield_stride", ctypes.c_int64), ("zpush", ctypes.c_void_p * ZT_MAX_PUSH_RANKS),
                ("zpush_ranks", ctypes.c_int32), ("zpush_slot", ctypes.c_int32), ("zpush_chunk_units", ctypes.c_int64),
                ("zpush_stride", ctypes.c_int64)]


class ZtEggrollArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("a", ctypes.c_void_p), ("b", ctypes.c_void_p),
                ("sigma", ctypes.c_void_p), ("xb", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
                ("rows_per_member", ctypes.c_int32), ("rank", ctypes.c_int32), ("xb_ready", ctypes.c_int32),
                ("test_stall_loads", ctypes.c_int32), ("x_ext", ctypes.c_void_p), ("w_ext", ctypes.c_void_p)]


class ZtEggrollGatedArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("w_gate", ctypes.c_void_p), ("w_up", ctypes.c_void_p),
                ("a_gate", ctypes.c_void_p), ("a_up", ctypes.c_void_p), ("sigma_gate", ctypes.c_void_p),
                ("sigma_up", ctypes.c_void_p), ("xb_gate", ctypes.c_void_p), ("xb_up", ctypes.c_void_p),
                ("y", ctypes.c_void_p), ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
                ("rows_per_member", ctypes.c_int32), ("rank", ctypes.c_int32), ("x_ext", ctypes.c_void_p),
                ("w_ext_gate", ctypes.c_void_p), ("w_ext_up", ctypes.c_void_p)]


class ZtEggrollXbArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("b", ctypes.c_void_p * 3), ("xb", ctypes.c_void_p * 3),
                ("m", ctypes.c_int64), ("k", ctypes.c_int64), ("n_seg", ctypes.c_int32),
                ("rows_per_member", ctypes.c_int32), ("sigma", ctypes.c_void_p * 3), ("xe", ctypes.c_void_p * 3),
                ("xe_slot", ctypes.c_int32 * 3), ("reserved", ctypes.c_int32), ("bt", ctypes.c_void_p)]


class ZtEggrollFactorArgs(ctypes.Structure):
    _fields_ = [("keys_a", ctypes.c_void_p), ("keys_b", ctypes.c_void_p), ("pairs", ctypes.c_int32),
                ("rank", ctypes.c_int32), ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("dtype", ctypes.c_int32),
                ("normalize", ctypes.c_int32), ("sigma", ctypes.c_float), ("reserved", ctypes.c_int32),
                ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("work", ctypes.c_void_p),
                ("a_ext", ctypes.c_void_p), ("ext_slot", ctypes.c_int32), ("reserved2", ctypes.c_int32),
                ("b_ext", ctypes.c_void_p), ("b_ext_row", ctypes.c_int32), ("reserved3", ctypes.c_int32),
                ("seeds", ctypes.c_void_p), ("n_params", ctypes.c_uint32), ("key_index_a", ctypes.c_uint32),
                ("key_index_b", ctypes.c_uint32), ("reserved4", ctypes.c_int32)]


class ZtEggrollNormArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("keys", ctypes.c_void_p),
                ("w_members", ctypes.c_void_p), ("y", ctypes.c_void_p), ("m", ctypes.c_int64), ("d", ctypes.c_int64),
                ("pairs", ctypes.c_int32), ("rows_per_member", ctypes.c_int32), ("sigma", ctypes.c_float),
                ("eps", ctypes.c_float), ("seeds", ctypes.c_void_p), ("n_params", ctypes.c_uint32),
                ("key_index", ctypes.c_uint32)]


class ZtLceArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("targets", ctypes.c_void_p),
                ("loss", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("correct", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t), ("rows", ctypes.c_int64),
                ("vocab", ctypes.c_int64), ("k", ctypes.c_int64), ("test_stall_loads", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("test_wait_cycles", ctypes.c_int64)]


class ZtLowrankDesc(ctypes.Structure):
    _fields_ = [("m", ctypes.c_int64), ("n", ctypes.c_int64), ("r", ctypes.c_int32), ("kp", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("n_streams", ctypes.c_int32),
                ("keys_p", ctypes.c_uint32 * 128), ("keys_psi", ctypes.c_uint32 * 128),
                ("p", ctypes.c_void_p), ("psi_t", ctypes.c_void_p), ("scale", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
                ("factors_given", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class ZtLowrankApplyArgs(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("ge", ctypes.c_void_p),
                ("n_alpha", ctypes.c_int32), ("alpha", ctypes.c_float * 3), ("ge_init", ctypes.c_int32),
                ("coef", ctypes.c_float * 128), ("test_stall_loads", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("test_wait_cycles", ctypes.c_int64)]


class ZtError(RuntimeError):
    """A C-ABI call returned a nonzero status."""


_lib = None


def load():
    """Load the library once; raise if it is absent (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ZtError(f"{LIB_PATH} is missing: build it with `python -m zotitan_b200.build` "
                      "(the zeroth-order kernels have no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    P, I32, I64, U32, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64
    lib.zt_last_error.restype = ctypes.c_char_p
    lib.zt_last_error.argtypes = []
    lib.zt_abi_version.restype = ctypes.c_int
    lib.zt_param_key.restype = U32
    lib.zt_param_key.argtypes = [U64, U32, U32]
    for name, args in [("zt_philox_words", [U32, P, I64, P, P]), ("zt_randn", [U32, I64, I64, P, P]),
                       ("zt_randn_at", [U32, P, I64, P, P]),
                       ("zt_plan_init", [ctypes.POINTER(ZtTensor), I32, U32, P, ctypes.c_size_t,
                                         ctypes.POINTER(ZtPlan), P]),
                       ("zt_pass", [ctypes.POINTER(ZtPlan), ctypes.POINTER(ZtPassCfg), ctypes.POINTER(ZtStream),
                                    I32, P]),
                       ("zt_pass_static", [ctypes.POINTER(ZtTensor), I32, U32, ctypes.POINTER(ZtPassCfg),
                                           ctypes.POINTER(ZtStream), I32, P])]:
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = args
    lib.zt_randn_keys.restype = ctypes.c_int
    lib.zt_randn_keys.argtypes = [ctypes.POINTER(ctypes.c_uint32), I32, I64, P, P]
    lib.zt_eggroll_linear.restype = ctypes.c_int
    lib.zt_eggroll_linear.argtypes = [ctypes.POINTER(ZtEggrollArgs), P]
    lib.zt_eggroll_take_error.restype = ctypes.c_int
    lib.zt_eggroll_take_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    lib.zt_eggroll_factors.restype = ctypes.c_int
    lib.zt_eggroll_factors.argtypes = [ctypes.POINTER(ZtEggrollFactorArgs), P]
    lib.zt_eggroll_rmsnorm.restype = ctypes.c_int
    lib.zt_eggroll_rmsnorm.argtypes = [ctypes.POINTER(ZtEggrollNormArgs), P]
    lib.zt_eggroll_rope.restype = ctypes.c_int
    lib.zt_eggroll_rope.argtypes = [P, P, P, P, I64, I32, I32, I32, I32, P]
    lib.zt_eggroll_swiglu.restype = ctypes.c_int
    lib.zt_eggroll_swiglu.argtypes = [P, P, P, I64, P]
    lib.zt_eggroll_xb.restype = ctypes.c_int
    lib.zt_eggroll_xb.argtypes = [ctypes.POINTER(ZtEggrollXbArgs), P]
    lib.zt_eggroll_gated.restype = ctypes.c_int
    lib.zt_eggroll_gated.argtypes = [ctypes.POINTER(ZtEggrollGatedArgs), P]
    lib.zt_eggroll_update_operands.restype = ctypes.c_int
    lib.zt_eggroll_update_operands.argtypes = [P, P, P, P, I32, I64, I64, ctypes.c_float, P, P, P]
    lib.zt_lora_add.restype = ctypes.c_int
    lib.zt_lora_add.argtypes = [P, P, P, ctypes.c_float, I64, I64, I32, P]
    lib.zt_lora_add3.restype = ctypes.c_int
    lib.zt_lora_add3.argtypes = [P, P, P, ctypes.c_float, I64, I64, I32, P]
    lib.zt_lora_split.restype = ctypes.c_int
    lib.zt_lora_split.argtypes = [P, P, I64, P]
    lib.zt_rmsnorm.restype = ctypes.c_int
    lib.zt_rmsnorm.argtypes = [P, P, P, I64, I64, ctypes.c_float, P]
    lib.zt_gemm_swiglu.restype = ctypes.c_int
    lib.zt_gemm_swiglu.argtypes = [P, P, P, P, I64, I64, I64, P]
    lib.zt_xent_rows.restype = ctypes.c_int
    lib.zt_xent_rows.argtypes = [P, I64, I64, I64, P, P, P, P, P]
    lib.zt_ipc_export.restype = ctypes.c_int
    lib.zt_ipc_export.argtypes = [P, P, ctypes.POINTER(U64)]
    lib.zt_ipc_open.restype = ctypes.c_int
    lib.zt_ipc_open.argtypes = [P, ctypes.POINTER(P)]
    lib.zt_ipc_close.restype = ctypes.c_int
    lib.zt_ipc_close.argtypes = [P]
    lib.zt_copy_async.restype = ctypes.c_int
    lib.zt_copy_async.argtypes = [P, P, ctypes.c_size_t, P]
    lib.zt_linear_xent_workspace_bytes.restype = ctypes.c_size_t
    lib.zt_linear_xent_workspace_bytes.argtypes = [I64, I64, I64]
    lib.zt_linear_xent.restype = ctypes.c_int
    lib.zt_linear_xent.argtypes = [ctypes.POINTER(ZtLceArgs), P]
    lib.zt_linear_xent_take_error.restype = ctypes.c_int
    lib.zt_linear_xent_take_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    lib.zt_gemm_addto.restype = ctypes.c_int
    lib.zt_gemm_addto.argtypes = [P, I64, P, P, ctypes.c_float, I64, I64, I64, P]
    lib.zt_gemm_take_error.restype = ctypes.c_int
    lib.zt_gemm_take_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    lib.zt_lowrank_workspace_bytes.restype = ctypes.c_int
    lib.zt_lowrank_workspace_bytes.argtypes = [I64, I64, I32, ctypes.POINTER(ctypes.c_size_t)]
    lib.zt_lowrank_prepare.restype = ctypes.c_int
    lib.zt_lowrank_prepare.argtypes = [ctypes.POINTER(ZtLowrankDesc), P]
    lib.zt_lowrank_apply.restype = ctypes.c_int
    lib.zt_lowrank_apply.argtypes = [ctypes.POINTER(ZtLowrankDesc), ctypes.POINTER(ZtLowrankApplyArgs), P]
    lib.zt_lowrank_take_error.restype = ctypes.c_int
    lib.zt_lowrank_take_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    lib.zt_plan_workspace_bytes.restype = ctypes.c_size_t
    lib.zt_plan_workspace_bytes.argtypes = [I32]
    if lib.zt_abi_version() != ABI_VERSION:
        raise ZtError(f"{LIB_PATH}: ABI version {lib.zt_abi_version()} != {ABI_VERSION}")
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != ZT_OK:
        msg = load().zt_last_error().decode(errors="replace")
        raise ZtError(f"{what} failed with status {rc}: {msg}")
