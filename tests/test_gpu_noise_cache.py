"""GPU tests of the noise cache (ZT_STREAM_Z_STORE / ZT_STREAM_Z_LOAD, zt_pass_cfg.zcache).

A pass that stores a stream's field writes exactly the Gaussians zt_randn gives for
each tensor's key, at the documented place (unit u's elements at u * 2048); a pass that
loads it gives every buffer bit-identical (0 ulp) to the same pass regenerating the
field, on uniform plans (the specialised kernels) and on a mixed-dtype, ragged,
unaligned plan (the generic kernels). A whole optimizer step with the cache on is
bit-identical to the step without it (test_gpu_step.py pins the default step, which
uses the cache, to the oracle at 0 ulp).
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import StepCase, flat, step_cases
from oracle import philox as ph

pytestmark = pytest.mark.gpu

TDT = {ph.F32: torch.float32, ph.BF16: torch.bfloat16, ph.F16: torch.float16}
MIXED = [(1, ph.BF16), (7, ph.F32), (8, ph.F16), (1023, ph.BF16), (2048, ph.F32), (2049, ph.BF16),
         (4099, ph.F16), (100003, ph.BF16), (5000, ph.F32), (777, "unaligned")]
N_PARAMS = 40
_G, _NAMES = step_cases()
GAUSSIAN = [n for n in _NAMES if "lowrank" not in n]


def f(x):
    return float(np.float32(x))


def make(specs, seed, with_ge=False):
    """Parameter tensors (and grad_est buffers) on the GPU; 'unaligned' is a bf16 view at
    a 2-byte offset, so its plan takes the generic kernels."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    keep, data, ge = [], [], []
    for n, dt in specs:
        una = dt == "unaligned"
        tdt = TDT[ph.BF16 if una else dt]
        for lst, scale in ((data, 0.02), (ge, 0.3)) if with_ge else ((data, 0.02),):
            x = (torch.randn(n + 1 if una else n, generator=g, device="cuda") * scale).to(tdt)
            if una:
                keep.append(x)
                x = x[1:]
            lst.append(x)
    return data, (ge if with_ge else None), keep


def clone_all(xs):
    return None if xs is None else [x.clone() for x in xs]


def run_pair(K, specs, passes, with_ge=False):
    """Runs the same pass sequence on two identical tables, one regenerating every field
    and one using the noise cache; compares every buffer after every pass."""
    data_a, ge_a, keep_a = make(specs, 11, with_ge)
    data_b, ge_b = clone_all(data_a), clone_all(ge_a)
    ta = K.ParamTable(data_a, n_params=N_PARAMS, ge=ge_a)
    tb = K.ParamTable(data_b, n_params=N_PARAMS, ge=ge_b)
    zc = tb.noise_cache()
    zc.fill_(float("nan"))   # nothing may read a slot no pass has written
    vals = torch.tensor([2.0137, 2.0051], dtype=torch.float32, device="cuda")
    for cfg, streams_plain, streams_cached in passes:
        if cfg.dev_inv2eps:
            cfg.dev_vals = vals.data_ptr()
        ta.run(cfg, streams_plain)
        cfg.zcache = zc.data_ptr()
        tb.run(cfg, streams_cached)
        cfg.zcache = 0
        torch.cuda.synchronize()
        for x, y in zip(data_a + (ge_a or []), data_b + (ge_b or [])):
            assert torch.equal(x, y)
    return tb, zc, keep_a


def schedule(K, L):
    """+eps (store) / -2eps (load) / restore + grad_est + next +eps (load, store) / -2eps
    (load) / two-stream restore + next (load, store) / last pass with update (load)."""
    e, m2 = f(1e-3), f(-2e-3)
    acc = dict(ge_mode=L.ZT_GE_ACCUM, ge_store=True, dev_inv2eps=f(1 / f(2e-3)), dev_invz=f(1 / f(3)),
               dev_tau=float("inf"))
    S = K.Stream
    return [
        (K.PassCfg(), [S(1, (e,))], [S(1, (e,), z_store=True)]),
        (K.PassCfg(), [S(1, (m2,))], [S(1, (m2,), z_load=True)]),
        (K.PassCfg(ge_load=False, **acc), [S(1, (e,), ge_dev=True), S(2, (e,))],
         [S(1, (e,), ge_dev=True, z_load=True), S(2, (e,), z_store=True)]),
        (K.PassCfg(), [S(2, (m2,))], [S(2, (m2,), z_load=True)]),
        (K.PassCfg(ge_load=True, **acc), [S(2, (e,), ge_dev=True), S(3, (e,))],
         [S(2, (e,), ge_dev=True, z_load=True), S(3, (e,), z_store=True)]),
        (K.PassCfg(), [S(3, (m2,))], [S(3, (m2,), z_load=True)]),
        (K.PassCfg(), [S(3, (e,)), S(4, (e,))], [S(3, (e,), z_load=True), S(4, (e,), z_store=True)]),
        (K.PassCfg(), [S(4, (m2,))], [S(4, (m2,), z_load=True)]),
        (K.PassCfg(ge_mode=L.ZT_GE_ACCUM, ge_load=True, update=True, lr=f(1e-2)),
         [S(4, (e,), ge=f(0.7)), S(9, (), ge=f(-0.2))], [S(4, (e,), ge=f(0.7), z_load=True), S(9, (), ge=f(-0.2))]),
    ]


@pytest.fixture(scope="module")
def K():
    from zotitan_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def L():
    from zotitan_b200 import _lib
    return _lib


def test_stored_field_is_the_noise_at_documented_slots(K, L):
    """After a storing +eps pass, unit u of the cache holds the Gaussians of the tensor
    owning u, element (u - first unit of the tensor) * 2048 + j at slot u * 2048 + j."""
    specs = MIXED
    tb, zc, _ = run_pair(K, specs, schedule(K, L)[:1])
    z = zc.cpu().numpy()
    u0 = 0
    for i, (n, _) in enumerate(specs):
        want = K.randn(K.param_key(1, N_PARAMS, i), n, "cuda").cpu().numpy()
        assert np.array_equal(z[u0 * 2048: u0 * 2048 + n], want), i
        u0 += (n + 2047) // 2048
    assert u0 == tb.plan.n_units


@pytest.mark.parametrize("dt", [ph.BF16, ph.F32, ph.F16])
def test_cached_schedule_uniform_plan(K, L, dt):
    """Uniform plans (specialised kernels): every pass of a cached schedule is
    bit-identical to the regenerating one."""
    specs = [(n, dt) for n in (8, 2048, 4096, 24, 100000, 2056, 16)]
    data, _, _ = make(specs, 0)
    assert K.ParamTable(data, n_params=N_PARAMS).plan.props & L.ZT_PLAN_VEC8
    run_pair(K, specs, schedule(K, L), with_ge=True)


def test_cached_schedule_mixed_plan(K, L):
    """Mixed dtypes, ragged sizes and an unaligned tensor (generic kernels)."""
    run_pair(K, MIXED, schedule(K, L), with_ge=True)


def test_noise_cache_argument_errors(K, L):
    lib = L.load()
    data, _, _ = make([(4096, ph.BF16)], 0)
    tb = K.ParamTable(data, n_params=N_PARAMS)
    zc = tb.noise_cache()
    S = K.Stream

    def rc(streams, zcache):
        cfg = K.PassCfg(zcache=zcache).to_c()
        arr = K._streams_array(streams)
        return lib.zt_pass(ctypes.byref(tb.plan), ctypes.byref(cfg), arr, len(streams), None)

    e = f(1e-3)
    assert rc([S(1, (e,), z_store=True)], 0) == L.ZT_ERR_INVALID                      # no cache
    assert rc([S(1, (e,), z_store=True)], zc.data_ptr() + 4) == L.ZT_ERR_INVALID      # misaligned
    assert rc([S(1, (e,), z_load=True, z_store=True)], zc.data_ptr()) == L.ZT_ERR_INVALID
    assert rc([S(1, (e,), z_store=True), S(2, (e,), z_load=True)], zc.data_ptr()) == L.ZT_ERR_INVALID
    assert rc([S(1, (e,), z_load=True), S(2, (e,), z_load=True)], zc.data_ptr()) == L.ZT_ERR_INVALID
    assert rc([S(1, (e,), z_store=True)], zc.data_ptr()) == L.ZT_OK
    torch.cuda.synchronize()


class ReplayScore:
    def __init__(self, values, params):
        self.it = iter(values)
        self.params = params
        self.snaps = []

    def __call__(self, model, batch):
        from zotitan_b200.objective import Score
        self.snaps.append(flat([p.detach().float().cpu().numpy() for p in self.params]))
        return Score(torch.tensor(next(self.it), device="cuda"), {})


def run_opt(case, **kw):
    from zotitan_b200.train_zo import ZOOptimizer
    ps = [torch.nn.Parameter(torch.from_numpy(p).to(TDT[d]).cuda()) for p, d in zip(case.params(), case.dtypes)]
    score = ReplayScore(case.values, ps)
    opt = ZOOptimizer(list(zip(case.names, ps)), case.cfg, score, total_steps=case.spec["total_steps"], **kw)
    afters, metrics = [], []
    for _ in range(case.spec["steps"]):
        metrics.append(opt.step(None, [None] * case.cfg.z_batch))
        afters.append(flat([p.detach().float().cpu().numpy() for p in ps]))
    return opt, afters, metrics, score.snaps


@pytest.mark.parametrize("name", GAUSSIAN)
def test_step_with_noise_cache_bit_identical(name):
    """Every golden optimizer configuration: the forwards see the same parameters and
    every step ends with the same parameters and metrics, cache on or off."""
    case = StepCase(_G, name)
    _, a0, m0, s0 = run_opt(case, noise_cache=False)
    opt, a1, m1, s1 = run_opt(case, noise_cache=True)
    assert opt.zcache is not None
    for a, b in zip(a0 + s0, a1 + s1):
        assert np.array_equal(a, b)
    for x, y in zip(m0, m1):
        for k in ("loss", "proj_grad", "proj_grad_clipped", "clip_frac", "lr"):
            assert x[k] == y[k], k


def test_noise_cache_default_follows_free_memory():
    """By default the optimizer keeps the cache when it fits in a quarter of the free
    device memory (every test model here does); noise_cache=False never allocates it."""
    case = StepCase(_G, "mezo_bf16_z3")
    opt, _, _, _ = run_opt(case)
    assert opt.zcache is not None and opt.planner.noise_cache
    assert opt.zcache.numel() == int(opt.table.plan.n_units) * 2048
    opt, _, _, _ = run_opt(case, noise_cache=False)
    assert opt.zcache is None and not opt.planner.noise_cache


def test_sharded_step_with_noise_cache():
    """The seed-sharded schedule (1-rank group) with the cache: the live copy's +eps pass
    stores, its -2eps pass loads; parameters match the cache-free single-GPU step."""
    import os
    import torch.distributed as dist
    case = StepCase(_G, "mezo_bf16_z3")
    _, a1, _, _ = run_opt(case, noise_cache=False)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = "29523"
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        opt, aw, _, _ = run_opt(case, sharded=True, noise_cache=True)
        assert opt.master is not None and opt.zcache is not None
        for a, b in zip(aw, a1):
            assert np.array_equal(a, b)
        del opt
    finally:
        dist.destroy_process_group()
