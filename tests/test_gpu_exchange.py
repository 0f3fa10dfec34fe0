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


@pytest.mark.parametrize("mode", ["in_pass", "copies"])
@pytest.mark.parametrize("setting", [True, 1])
@pytest.mark.parametrize("name", ONE_DTYPE)
def test_sharded_step_with_field_exchange(one_rank_group, name, setting, mode):
    """The sharded schedule with the field exchange on a one-rank group: the pushes are
    stores of the +eps pass into the store (in_pass, when the plan takes the specialised
    kernel) or device-local copies (copies), and the last pass reads the stored fields
    (every pair, or only the first one: the others regenerated); the parameters equal
    the single-GPU step's."""
    from test_gpu_noise_cache import run_opt
    case = StepCase(_G, name)
    _, a1, m1, _ = run_opt(case, noise_cache=False)
    opt, aw, mw, _ = run_opt(case, sharded=True, noise_cache=True, field_exchange=setting, exchange_mode=mode)
    assert opt.exchange is not None and opt.layout is not None
    assert opt.exchange.n_slots == (case.cfg.z_batch if setting is True else 1)
    uniform = bool(int(opt.table.plan.props) & 1)
    assert opt.exchange.in_pass == (mode == "in_pass" and uniform)
    for a, b in zip(aw, a1):
        assert np.array_equal(a, b)
    for x, y in zip(mw, m1):
        assert x["proj_grad"] == y["proj_grad"]
    opt.exchange.close()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_in_pass_push_fills_every_rank_store(K, L, world):
    """The +eps pass with zt_pass_cfg.zpush on one GPU, `world` local stores standing for
    the ranks' stores: each store receives exactly the slices push_plan assigns to it (the
    field zt_randn gives for each tensor's key), NaN everywhere else; the pass's own
    results (live copy, noise cache) equal the same pass without the push."""
    from zotitan_b200.exchange import push_plan, store_elems
    from zotitan_b200.flat import FlatLayout
    layout = FlatLayout(NUMELS, world)
    _, va, _ = flat_tables(K, layout, torch.bfloat16, 9)
    _, vb, _ = flat_tables(K, layout, torch.bfloat16, 9)
    live_a = [torch.empty_like(v) for v in va]
    live_b = [torch.empty_like(v) for v in vb]
    ta, tb = K.ParamTable(va, live=live_a), K.ParamTable(vb, live=live_b)
    n_units = int(ta.plan.n_units)
    slots, slot, seed = 3, 2, 2**62 + 17
    stores = [torch.full((store_elems(layout, slots),), float("nan"), device="cuda") for _ in range(world)]
    za, zb = ta.noise_cache(), tb.noise_cache()
    za.fill_(float("nan"))   # a tensor's last unit is written only up to its numel
    zb.fill_(float("nan"))
    cfg_a = K.PassCfg(src=L.ZT_BUF_DATA, dst=L.ZT_BUF_LIVE, zcache=za.data_ptr())
    cfg_b = K.PassCfg(src=L.ZT_BUF_DATA, dst=L.ZT_BUF_LIVE, zcache=zb.data_ptr(),
                      zpush=tuple(t.data_ptr() for t in stores), zpush_slot=slot,
                      zpush_chunk_units=layout.per, zpush_stride=layout.chunks * layout.per * 2048)
    st = [K.Stream(seed, (f(1e-3),), z_store=True)]
    ta.run(cfg_a, st)
    tb.run(cfg_b, st)
    torch.cuda.synchronize()
    assert all(torch.equal(x, y) for x, y in zip(live_a, live_b))
    want = [torch.full_like(t, float("nan")) for t in stores]
    for c in push_plan(layout, n_units, slot, world):
        want[c.dst][c.dst_elem:c.dst_elem + c.n_elems] = za[c.src_elem:c.src_elem + c.n_elems]
    for got, w in zip(stores, want):
        assert torch.equal(torch.nan_to_num(got, nan=7.0), torch.nan_to_num(w, nan=7.0))


def test_in_pass_push_argument_errors(K, L):
    from zotitan_b200.flat import FlatLayout
    lib = L.load()
    layout = FlatLayout(NUMELS, 2)
    _, v, _ = flat_tables(K, layout, torch.bfloat16, 1)
    live = [torch.empty_like(x) for x in v]
    t = K.ParamTable(v, live=live)
    zc = t.noise_cache()
    store = torch.zeros(1 << 20, device="cuda")

    def rc(streams, **kw):
        base = dict(src=L.ZT_BUF_DATA, dst=L.ZT_BUF_LIVE, zcache=zc.data_ptr(), zpush_slot=0,
                    zpush_chunk_units=layout.per, zpush_stride=4096)
        base.update(kw)
        cfg = K.PassCfg(**base).to_c()
        arr = K._streams_array(streams)
        return lib.zt_pass(ctypes.byref(t.plan), ctypes.byref(cfg), arr, len(streams), None)

    S = K.Stream
    ok = (store.data_ptr(), store.data_ptr())
    assert rc([S(1, (f(1e-3),), z_store=True)], zpush=(store.data_ptr() + 4, store.data_ptr())) == L.ZT_ERR_INVALID
    assert rc([S(1, (f(1e-3),), z_store=True)], zpush=ok, zpush_chunk_units=0) == L.ZT_ERR_INVALID
    assert rc([S(1, (f(1e-3),))], zpush=ok) == L.ZT_ERR_INVALID                     # no storing stream
    assert rc([S(1, (f(1e-3), f(1e-3)), z_store=True)], zpush=ok) == L.ZT_ERR_INVALID   # not the +eps shape
    torch.cuda.synchronize()
