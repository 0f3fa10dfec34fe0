"""The C-ABI library loads and exports what include/zotitan_b200.h declares (CPU only:
no call here launches GPU work; only argument validation paths run)."""
import ctypes
import os
import re

import pytest

from zotitan_b200 import _lib as L
from zotitan_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build()
    return L.load()


def declared_functions():
    src = open(os.path.join(ROOT, "include", "zotitan_b200.h")).read()
    return sorted(set(re.findall(r"^ZT_API [^(]*?\b(zt_\w+)\(", src, flags=re.M)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert names, "no declarations found"
    assert sorted(L.EXPORTS) == names
    for n in names:
        assert hasattr(lib, n), n


def test_abi_version_and_key(lib):
    assert lib.zt_abi_version() == L.ABI_VERSION == 11
    from oracle import philox as ph
    for seed, n, i in [(0, 1, 0), (1234, 39, 7), (2**40 + 3, 146, 145), (2**64 - 1, 448, 3)]:
        assert lib.zt_param_key(seed, n, i) == ph.param_key(seed, n, i) == (seed * n + i) & 0x7FFFFFFF


def test_struct_layouts_match_header(lib):
    assert ctypes.sizeof(L.ZtTensor) == 64
    assert ctypes.sizeof(L.ZtStream) == 40
    assert ctypes.sizeof(L.ZtPlan) == 56 and L.ZtPlan.props.offset == 48
    assert ctypes.sizeof(L.ZtPassCfg) == 240 and L.ZtPassCfg.dev_vals.offset == 88 and L.ZtPassCfg.unit_begin.offset == 112
    assert L.ZtPassCfg.zcache.offset == 128 and L.ZtPassCfg.zfield.offset == 136 and L.ZtPassCfg.zfield_stride.offset == 144
    assert L.ZtPassCfg.zpush.offset == 152 and L.ZtPassCfg.zpush_ranks.offset == 216 and L.ZtPassCfg.zpush_stride.offset == 232
    assert L.ZtStream.zslot.offset == 36
    assert ctypes.sizeof(L.ZtEggrollArgs) == 112 and L.ZtEggrollArgs.xb_ready.offset == 88
    assert ctypes.sizeof(L.ZtEggrollXbArgs) == 152 and L.ZtEggrollXbArgs.bt.offset == 144
    assert ctypes.sizeof(L.ZtEggrollGatedArgs) == 136 and L.ZtEggrollGatedArgs.x_ext.offset == 112
    assert ctypes.sizeof(L.ZtEggrollFactorArgs) == 144 and L.ZtEggrollFactorArgs.b_ext.offset == 104
    assert L.ZtEggrollFactorArgs.seeds.offset == 120 and L.ZtEggrollFactorArgs.key_index_b.offset == 136
    assert ctypes.sizeof(L.ZtEggrollNormArgs) == 88 and L.ZtEggrollNormArgs.seeds.offset == 72
    assert ctypes.sizeof(L.ZtLowrankDesc) == 1104 and L.ZtLowrankDesc.p.offset == 1056
    assert L.ZtLowrankDesc.factors_given.offset == 1096
    assert ctypes.sizeof(L.ZtLowrankApplyArgs) == 576 and L.ZtLowrankApplyArgs.coef.offset == 44
    assert L.ZtLowrankApplyArgs.test_wait_cycles.offset == 568
    assert lib.zt_plan_workspace_bytes(0) == 8
    assert lib.zt_plan_workspace_bytes(3) == 256 + 8 * 4
    assert lib.zt_plan_workspace_bytes(5) == 512 + 8 * 6


def test_invalid_arguments_are_reported(lib):
    assert lib.zt_randn(1, 0, -1, None, None) == L.ZT_ERR_INVALID
    assert b"negative" in lib.zt_last_error()
    # peer-mapping entry points check their pointers before any CUDA call
    h = (ctypes.c_ubyte * L.ZT_IPC_HANDLE_BYTES)()
    off = ctypes.c_uint64()
    assert lib.zt_ipc_export(None, h, ctypes.byref(off)) == L.ZT_ERR_INVALID
    assert lib.zt_ipc_open(None, None) == L.ZT_ERR_INVALID
    assert lib.zt_ipc_close(None) == L.ZT_ERR_INVALID
    assert lib.zt_copy_async(None, None, 16, None) == L.ZT_ERR_INVALID
    assert lib.zt_copy_async(None, None, 0, None) == L.ZT_OK   # nothing to copy
    assert lib.zt_randn(1, 2**31 - 10, 100, None, None) == L.ZT_ERR_LIMIT
    assert lib.zt_randn(1, 0, 0, None, None) == L.ZT_OK          # empty is a no-op
    assert lib.zt_last_error() == b""
    assert lib.zt_pass(None, None, None, 0, None) == L.ZT_ERR_INVALID
    plan = L.ZtPlan()
    cfg = L.ZtPassCfg()
    cfg.src, cfg.dst = L.ZT_BUF_DATA, L.ZT_BUF_DATA
    assert lib.zt_pass(ctypes.byref(plan), ctypes.byref(cfg), None, 300, None) == L.ZT_ERR_INVALID
    arr = (L.ZtStream * 1)()
    assert lib.zt_pass(ctypes.byref(plan), ctypes.byref(cfg), arr, 300, None) == L.ZT_ERR_LIMIT
    cfg.src = 7
    assert lib.zt_pass(ctypes.byref(plan), ctypes.byref(cfg), arr, 1, None) == L.ZT_ERR_INVALID
    cfg.src, cfg.momentum, cfg.update = L.ZT_BUF_DATA, L.ZT_MOM_STORED_EMA, 0
    assert lib.zt_pass(ctypes.byref(plan), ctypes.byref(cfg), arr, 1, None) == L.ZT_ERR_INVALID
    assert b"require update" in lib.zt_last_error()
    cfg.momentum, cfg.update, cfg.src = L.ZT_MOM_NONE, 1, L.ZT_BUF_LIVE   # plan without live buffers
    assert lib.zt_pass(ctypes.byref(plan), ctypes.byref(cfg), arr, 1, None) == L.ZT_ERR_INVALID
    assert b"live" in lib.zt_last_error()
    cfg.src, cfg.second_moment = L.ZT_BUF_DATA, 1
    assert lib.zt_pass(ctypes.byref(plan), ctypes.byref(cfg), arr, 1, None) == L.ZT_ERR_INVALID
    t = (L.ZtTensor * 1)()
    t[0].numel, t[0].dtype, t[0].index, t[0].data = 2**31, L.ZT_BF16, 0, 16
    out = L.ZtPlan()
    assert lib.zt_plan_init(t, 1, 1, ctypes.c_void_p(256), 4096, ctypes.byref(out), None) == L.ZT_ERR_LIMIT
    t[0].numel, t[0].index = 10, 5
    assert lib.zt_plan_init(t, 1, 1, ctypes.c_void_p(256), 4096, ctypes.byref(out), None) == L.ZT_ERR_INVALID
    assert lib.zt_plan_init(t, 1, 1, ctypes.c_void_p(256), 8, ctypes.byref(out), None) == L.ZT_ERR_INVALID


def test_lowrank_arguments_checked_before_launch(lib):
    """The low-rank entry points reject bad descriptors on the host (no CUDA call)."""
    sz = ctypes.c_size_t()
    assert lib.zt_lowrank_workspace_bytes(300, 520, 3, ctypes.byref(sz)) == L.ZT_OK
    assert sz.value == 2 * 3 * 3 * 32 * 4                       # tiles x streams x partials x fp32
    assert lib.zt_lowrank_workspace_bytes(300, 520, 0, ctypes.byref(sz)) == L.ZT_ERR_INVALID
    d = L.ZtLowrankDesc()
    d.m, d.n, d.r, d.kp, d.dtype, d.n_streams = 256, 512, 64, 64, L.ZT_BF16, 1
    d.p, d.psi_t, d.scale, d.workspace, d.workspace_bytes = 256, 512, 1024, 2048, 1 << 20
    a = L.ZtLowrankApplyArgs()
    a.src, a.dst, a.n_alpha = 4096, 4096, 1
    for field, value, code, msg in [("dtype", 7, L.ZT_ERR_INVALID, b"dtype"),
                                    ("kp", 48, L.ZT_ERR_INVALID, b"multiple of 64"),
                                    ("r", 65, L.ZT_ERR_INVALID, b"r <="),
                                    ("n_streams", 129, L.ZT_ERR_INVALID, b"n_streams"),
                                    ("m", 2**31, L.ZT_ERR_LIMIT, b"32-bit"),
                                    ("p", 8, L.ZT_ERR_INVALID, b"aligned")]:
        old = getattr(d, field)
        setattr(d, field, value)
        assert lib.zt_lowrank_prepare(ctypes.byref(d), None) == code, field
        assert msg in lib.zt_last_error(), (field, lib.zt_last_error())
        assert lib.zt_lowrank_apply(ctypes.byref(d), ctypes.byref(a), None) == code, field
        setattr(d, field, old)
    d.workspace_bytes = 8
    assert lib.zt_lowrank_prepare(ctypes.byref(d), None) == L.ZT_ERR_INVALID
    assert b"workspace" in lib.zt_last_error()
    a.n_alpha = 0
    assert lib.zt_lowrank_apply(ctypes.byref(d), ctypes.byref(a), None) == L.ZT_ERR_INVALID   # dst without alpha
    a.dst = None
    assert lib.zt_lowrank_apply(ctypes.byref(d), ctypes.byref(a), None) == L.ZT_ERR_INVALID   # nothing to write
    a.src, a.dst, a.n_alpha = 4096, 4096 + 1024, 1                                          # partial overlap
    assert lib.zt_lowrank_apply(ctypes.byref(d), ctypes.byref(a), None) == L.ZT_ERR_INVALID
    assert b"overlap" in lib.zt_last_error()


def test_missing_library_raises(tmp_path, monkeypatch):
    """No CPU fallback: a missing library is an error, not a silent torch path."""
    monkeypatch.setattr(L, "_lib", None)
    monkeypatch.setattr(L, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(L.ZtError, match="no CPU fallback"):
        L.load()


def test_optimizer_refuses_cpu_tensors():
    import torch
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer
    p = torch.nn.Parameter(torch.zeros(4))
    with pytest.raises(ValueError, match="CUDA"):
        ZOOptimizer([("w", p)], ZOConfig(), score_fn=None)


def test_eggroll_companions_validate_before_launch(lib):
    """Shape checks of the population element-wise entry points fail on the host."""
    import numpy as np
    keys = (ctypes.c_uint32 * 2)(1, 2)
    fa = L.ZtEggrollFactorArgs(ctypes.addressof(keys), ctypes.addressof(keys), 2, 3, 256, 256, L.ZT_BF16, 1, 1e-3, 0,
                               16, 16, 16, 16, None, 0, 0, None, 0, 0)
    assert lib.zt_eggroll_factors(ctypes.byref(fa), None) == L.ZT_ERR_INVALID and b"rank" in lib.zt_last_error()
    fa.rank, fa.pairs = 4, L.ZT_EGGROLL_MAX_PAIRS + 1
    assert lib.zt_eggroll_factors(ctypes.byref(fa), None) == L.ZT_ERR_LIMIT
    fa.pairs, fa.n = 2, 2**30
    assert lib.zt_eggroll_factors(ctypes.byref(fa), None) == L.ZT_ERR_LIMIT
    fa.n, fa.a = 256, 8
    assert lib.zt_eggroll_factors(ctypes.byref(fa), None) == L.ZT_ERR_INVALID and b"aligned" in lib.zt_last_error()
    na = L.ZtEggrollNormArgs(16, 16, ctypes.addressof(keys), 16, 16, 1000, 64, 2, 128, 1e-3, 1e-5)
    assert lib.zt_eggroll_rmsnorm(ctypes.byref(na), None) == L.ZT_ERR_INVALID and b"rows_per_member" in lib.zt_last_error()
    na.m, na.d = 512, 60
    assert lib.zt_eggroll_rmsnorm(ctypes.byref(na), None) == L.ZT_ERR_INVALID
    assert lib.zt_eggroll_rope(16, 16, 16, 16, 64, 64, 4, 4, 24, None) == L.ZT_ERR_INVALID
    assert lib.zt_eggroll_rope(16, 16, 16, 16, 65, 64, 4, 4, 64, None) == L.ZT_ERR_INVALID
    assert lib.zt_eggroll_swiglu(16, 16, 16, 12, None) == L.ZT_ERR_INVALID
    assert lib.zt_eggroll_swiglu(None, None, None, 0, None) == L.ZT_OK
    del np
