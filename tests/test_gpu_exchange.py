"""GPU tests of the field store (ZT_STREAM_Z_FIELD, zt_pass_cfg.zfield) and of the
sharded step's field exchange (zotitan_b200.exchange).

Kernel level: a rank's share of a flat layout is replayed (every pair's +eps / -2eps /
+eps chain, its grad_est term, the SGD update) once with every field regenerated and
once with the fields read from a field store filled by the exchange's push plan from
noise caches; every element must be bit-identical (0 ulp), on a uniform bf16 plan (the
specialised replay kernel) and with stored-EMA momentum (the generic kernel), and the
elements outside the share untouched. Optimizer level: the sharded step with the
exchange on a one-rank NCCL group (pushes are device-local copies) ends bit-identical
to the single-GPU step, with every pair stored and with only some.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from helpers import StepCase, step_cases

pytestmark = pytest.mark.gpu

_G, _NAMES = step_cases()
NUMELS = [5000, 2048 * 3, 8, 2048 * 9 + 8, 24, 40000]   # multiples of 8: the specialised kernels apply
N_PARAMS = len(NUMELS)


def f(x):
    return float(np.float32(x))


@pytest.fixture(scope="module")
def K():
    from zotitan_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def L():
    from zotitan_b200 import _lib
    return _lib


def flat_tables(K, layout, dtype, seed, m=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    flat = torch.zeros(layout.numel, dtype=dtype, device="cuda")
    views = layout.views(flat, [(n,) for n in NUMELS])
    for v in views:
        v.copy_(torch.randn(v.numel(), generator=g, device="cuda") * 0.02)
    mom = layout.views(torch.zeros(layout.numel, dtype=dtype, device="cuda"), [(n,) for n in NUMELS]) if m else None
    return flat, views, mom


def fill_store(K, L, layout, table, seeds, rank, world):
    """Every pair's field, generated into a noise cache by a storing pass on a scratch
    copy, pushed (this rank's share only) into a NaN-filled store with zt_copy_async."""
    from zotitan_b200.exchange import push_plan, store_elems
    lib = L.load()
    n_units = int(table.plan.n_units)
    store = torch.full((store_elems(layout, len(seeds)),), float("nan"), dtype=torch.float32, device="cuda")
    scratch = [p.clone() for p in table.params]
    st = K.ParamTable(scratch, n_params=N_PARAMS)
    zc = st.noise_cache()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for j, s in enumerate(seeds):
        st.run(K.PassCfg(zcache=zc.data_ptr()), [K.Stream(s, (f(1e-3),), z_store=True)])
        for c in push_plan(layout, n_units, j, world):
            if c.dst == rank:
                L.check(lib.zt_copy_async(store.data_ptr() + 4 * c.dst_elem, zc.data_ptr() + 4 * c.src_elem,
                                          4 * c.n_elems, stream), "zt_copy_async")
    torch.cuda.synchronize()
    return store


@pytest.mark.parametrize("momentum", [False, True])
@pytest.mark.parametrize("world,rank", [(1, 0), (2, 1), (3, 2)])
def test_replay_from_field_store_bit_identical(K, L, world, rank, momentum):
    from zotitan_b200.exchange import chunk_field
    from zotitan_b200.flat import FlatLayout
    layout = FlatLayout(NUMELS, world)
    seeds = [11, 2**63 + 7, 5, 2**40 + 3, 9]
    e, m2 = f(1e-3), f(-2e-3)
    flat_a, va, ma = flat_tables(K, layout, torch.bfloat16, 3, momentum)
    flat_b, vb, mb = flat_tables(K, layout, torch.bfloat16, 3, momentum)
    ta = K.ParamTable(va, m=ma)
    tb = K.ParamTable(vb, m=mb)
    store = fill_store(K, L, layout, tb, seeds, rank, world)
    kw = dict(ge_mode=L.ZT_GE_ACCUM, update=True, lr=f(1e-2))
    if momentum:   # stored EMA: the generic full kernel
        kw.update(momentum=L.ZT_MOM_STORED_EMA, beta1=f(0.9), one_minus_beta1=f(0.1), m_scale=f(1 / f(0.1)))
    coefs = [f(0.3), f(-0.7), f(0.05), f(1.5), f(-0.25)]
    for k, (ub, ue) in enumerate(layout.shard_ranges(rank)):
        cfg = K.PassCfg(unit_begin=ub, unit_end=ue, **kw)
        ta.run(cfg, [K.Stream(s, (e, m2, e), ge=c) for s, c in zip(seeds, coefs)])
        zf, stride = chunk_field(layout, store.data_ptr(), k)
        cfg_b = K.PassCfg(unit_begin=ub, unit_end=ue, zfield=zf, zfield_stride=stride, **kw)
        # pair 2 regenerated, the others read from the store (as when not every pair fits)
        tb.run(cfg_b, [K.Stream(s, (e, m2, e), ge=c, z_field=None if j == 2 else j)
                       for j, (s, c) in enumerate(zip(seeds, coefs))])
    torch.cuda.synchronize()
    assert torch.equal(flat_a, flat_b)
    if momentum:
        assert all(torch.equal(x, y) for x, y in zip(ma, mb))
    # the share changed and nothing outside it did
    flat0, _, _ = flat_tables(K, layout, torch.bfloat16, 3)
    U = L.ZT_UNIT_ELEMS
    mine = torch.zeros(layout.numel, dtype=torch.bool, device="cuda")
    for ub, ue in layout.shard_ranges(rank):
        mine[ub * U: ue * U] = True
    assert torch.equal(flat_b[~mine], flat0[~mine])
    assert not torch.equal(flat_b[mine], flat0[mine])


def test_field_store_argument_errors(K, L):
    lib = L.load()
    from zotitan_b200.flat import FlatLayout
    layout = FlatLayout(NUMELS, 1)
    _, v, _ = flat_tables(K, layout, torch.bfloat16, 1)
    t = K.ParamTable(v)
    store = torch.zeros(int(t.plan.n_units) * 2048 + 8, dtype=torch.float32, device="cuda")
    n_units = int(t.plan.n_units)

    def rc(streams, zfield, stride, ub=0, ue=0):
        cfg = K.PassCfg(ge_mode=L.ZT_GE_ACCUM, update=True, lr=f(1e-2), unit_begin=ub, unit_end=ue,
                        zfield=zfield, zfield_stride=stride).to_c()
        arr = K._streams_array(streams)
        return lib.zt_pass(ctypes.byref(t.plan), ctypes.byref(cfg), arr, len(streams), None)

    S = K.Stream
    full = n_units * 2048
    assert rc([S(1, (f(1e-3),), ge=f(0.5), z_field=0)], 0, full) == L.ZT_ERR_INVALID                  # no store
    assert rc([S(1, (f(1e-3),), ge=f(0.5), z_field=0)], store.data_ptr() + 4, full) == L.ZT_ERR_INVALID  # misaligned
    assert rc([S(1, (f(1e-3),), ge=f(0.5), z_field=0)], store.data_ptr(), full - 4) == L.ZT_ERR_INVALID  # stride short
    assert rc([S(1, (f(1e-3),), ge=f(0.5), z_field=0)], store.data_ptr(), full + 2) == L.ZT_ERR_INVALID  # not 16 B
    assert rc([S(1, (f(1e-3),), ge=f(0.5), z_field=0, z_load=True)], store.data_ptr(), full) == L.ZT_ERR_INVALID
    assert rc([S(1, (f(1e-3),), ge=f(0.5), z_field=70000)], store.data_ptr(), full) == L.ZT_ERR_INVALID
    # a short range needs only its own units
    assert rc([S(1, (f(1e-3),), ge=f(0.5), z_field=0)], store.data_ptr(), 2048, ub=1, ue=2) == L.ZT_OK
    torch.cuda.synchronize()


@pytest.fixture(scope="module")
def one_rank_group():
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = "29531"
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    yield
    dist.destroy_process_group()


ONE_DTYPE = ["mezo_bf16_z3", "seedwin_adam_bf16_z2", "ema_adam_f32_z2", "clip_norm_bf16", "wd_anchored_l1_bf16"]


@pytest.mark.parametrize("setting", [True, 1])
@pytest.mark.parametrize("name", ONE_DTYPE)
def test_sharded_step_with_field_exchange(one_rank_group, name, setting):
    """The sharded schedule with the field exchange on a one-rank group: the pushes are
    device-local copies into the store, and the last pass reads the stored fields
    (every pair, or only the first one: the others regenerated); the parameters equal
    the single-GPU step's."""
    from test_gpu_noise_cache import run_opt
    case = StepCase(_G, name)
    _, a1, m1, _ = run_opt(case, noise_cache=False)
    opt, aw, mw, _ = run_opt(case, sharded=True, noise_cache=True, field_exchange=setting)
    assert opt.exchange is not None and opt.layout is not None
    assert opt.exchange.n_slots == (case.cfg.z_batch if setting is True else 1)
    for a, b in zip(aw, a1):
        assert np.array_equal(a, b)
    for x, y in zip(mw, m1):
        assert x["proj_grad"] == y["proj_grad"]
    opt.exchange.close()
