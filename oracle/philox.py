"""ctypes front end of the C oracle (test infrastructure only; see oracle/__init__.py).

Builds ``oracle/libzo_oracle.so`` from ``philox_oracle.c`` with gcc on first use
(``__graft_entry__.build()`` also builds it) and exposes numpy-level helpers.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "philox_oracle.c")
LIB = os.path.join(HERE, "libzo_oracle.so")

F32, BF16, F16 = 0, 1, 2


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (no fast-math: IEEE fp32, explicit fmaf)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + f".tmp{os.getpid()}"
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-std=gnu11",
                               "-ffp-contract=off", "-o", tmp, SRC, "-lm"])
        os.replace(tmp, LIB)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        P = ctypes.c_void_p
        _lib.zo_param_key.restype = ctypes.c_uint32
        _lib.zo_param_key.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32]
        _lib.zo_philox_words.argtypes = [ctypes.c_uint32, P, ctypes.c_int64, P]
        _lib.zo_randn.argtypes = [ctypes.c_uint32, ctypes.c_int64, ctypes.c_int64, P]
        _lib.zo_randn_at.argtypes = [ctypes.c_uint32, P, ctypes.c_int64, P]
        _lib.zo_round.argtypes = [ctypes.c_int, P, ctypes.c_int64]
        _lib.zo_add_scaled.argtypes = [ctypes.c_int, P, P, ctypes.c_float, ctypes.c_int64]
        _lib.zo_mul_scalar.argtypes = [ctypes.c_int, P, P, ctypes.c_float, ctypes.c_int64]
        _lib.zo_div_scalar.argtypes = [ctypes.c_int, P, P, ctypes.c_float, ctypes.c_int64]
        _lib.zo_addcmul.argtypes = [ctypes.c_int, P, P, P, ctypes.c_float, ctypes.c_int64]
        _lib.zo_sqrt_add.argtypes = [ctypes.c_int, P, ctypes.c_float, ctypes.c_int64]
        _lib.zo_addcdiv.argtypes = [ctypes.c_int, P, P, P, ctypes.c_float, ctypes.c_int64]
        _lib.zo_anchored.argtypes = [ctypes.c_int, P, P, ctypes.c_float, ctypes.c_int, ctypes.c_int64]
    return _lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return ctypes.c_void_p(a.ctypes.data)


def param_key(seed: int, n_params: int, index: int) -> int:
    return int(lib().zo_param_key(seed & 0xFFFFFFFFFFFFFFFF, n_params, index))


def words(key: int, offsets) -> np.ndarray:
    offs = np.ascontiguousarray(np.asarray(offsets, dtype=np.int64).astype(np.uint32))
    out = np.empty((offs.size, 4), dtype=np.uint32)
    lib().zo_philox_words(key, _p(offs), offs.size, _p(out))
    return out


def randn(key: int, n: int, off0: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().zo_randn(key, off0, n, _p(out))
    return out


def randn_at(key: int, offsets) -> np.ndarray:
    offs = np.ascontiguousarray(np.asarray(offsets, dtype=np.int64).astype(np.uint32))
    out = np.empty(offs.size, dtype=np.float32)
    lib().zo_randn_at(key, _p(offs), offs.size, _p(out))
    return out


# --- elementwise ops on fp32 carrier arrays (values exact in the param dtype) ---

def rounded(dt: int, x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().zo_round(dt, _p(y), y.size)
    return y


def add_scaled_(dt, p, x, a):
    lib().zo_add_scaled(dt, _p(p), _p(np.ascontiguousarray(x, dtype=np.float32)), a, p.size)


def mul_scalar(dt, x, s):
    out = np.empty_like(x)
    lib().zo_mul_scalar(dt, _p(out), _p(x), s, x.size)
    return out


def div_scalar(dt, x, s):
    out = np.empty_like(x)
    lib().zo_div_scalar(dt, _p(out), _p(x), s, x.size)
    return out


def addcmul_(dt, v, t1, t2, c):
    lib().zo_addcmul(dt, _p(v), _p(t1), _p(t2), c, v.size)


def sqrt_add_(dt, x, eps):
    lib().zo_sqrt_add(dt, _p(x), eps, x.size)


def addcdiv_(dt, p, g, d, c):
    lib().zo_addcdiv(dt, _p(p), _p(g), _p(d), c, p.size)


def anchored_(dt, p, p0, lam, l1):
    lib().zo_anchored(dt, _p(p), _p(p0), lam, int(bool(l1)), p.size)


def ulp_diff_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in fp32 units-in-the-last-place between two fp32 arrays."""
    def ordered(x):
        bits = np.ascontiguousarray(x, dtype=np.float32).view(np.int32).astype(np.int64)
        return np.where(bits >= 0, bits, -(bits & 0x7FFFFFFF))
    return np.abs(ordered(a) - ordered(b))


def ulp_diff_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 ulps between two arrays whose values are bf16-exact."""
    return ulp_diff_f32(a, b) >> 16


def randn_numpy(key: int, n: int, off0: int = 0) -> np.ndarray:
    """The same Gaussians evaluated the way Triton's interpreter evaluates
    random.py:126-143,181-203 on CPU: exact words, then numpy float32 log, cos and
    sqrt. On one machine this is bit-identical to the reference run with
    TRITON_INTERPRET=1, so it pins the optimizer arithmetic independently of the
    device's transcendental approximations."""
    w = words(key, np.arange(off0, off0 + n, dtype=np.int64))

    def uni(col):
        x = np.ascontiguousarray(col).view(np.int32)
        x = np.where(x < 0, -x - 1, x)
        return x.astype(np.float32) * np.float32(4.6566127342e-10)

    u1 = np.maximum(np.float32(1e-7), uni(w[:, 0]))
    u2 = uni(w[:, 1])
    th = np.float32(6.283185307179586) * u2
    r = np.sqrt(np.float32(-2.0) * np.log(u1))
    return (r * np.cos(th)).astype(np.float32)


def alpha_for(dt_self: int, dt_other: int, a: float) -> float:
    """Scalar alpha of ``self.add_(other, alpha=a)`` as torch's CPU kernel uses it:
    when self and other share a reduced float dtype (bf16/fp16) the alpha is first
    converted to that dtype; otherwise it stays fp32 (opmath)."""
    a = float(np.float32(a))
    if dt_self == dt_other and dt_self in (BF16, F16):
        return float(rounded(dt_self, np.array([a], dtype=np.float32))[0])
    return a
