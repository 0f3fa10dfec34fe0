"""Host planner (zotitan_b200.train_zo.StepPlanner) vs the op-by-op oracle step, on CPU.

The planner decides every fused pass of a step (which seeds, which perturbation
chains, which gradient / momentum coefficients, which scalars). Executed through the
oracle's pass interpreter, that schedule must reproduce the oracle's restatement of
the reference step bit for bit, for every optimizer branch, in the single-GPU
schedule and in the seed-sharded schedule (the sharded master must end each step
bit-identical to the single-GPU result).
"""
import numpy as np
import pytest

from helpers import StepCase, flat, step_cases
from oracle import philox as ph
from oracle.pass_interp import run_pass
from oracle.zo_step import OracleZO
from zotitan_b200.train_zo import StepPlanner

_G, _NAMES = step_cases()
GAUSSIAN = [n for n in _NAMES if "lowrank" not in n]


def make_tensors(params, dtypes, planner, sharded):
    ts = []
    for i, (p, dt) in enumerate(zip(params, dtypes)):
        ts.append({"data": p, "live": p.copy() if sharded else None,
                   "m": np.zeros_like(p) if planner.needs_m else None,
                   "v": np.zeros_like(p) if planner.needs_v else None,
                   "anchor": p.copy() if planner.needs_anchor else None,
                   "ge": np.zeros_like(p) if planner.ge_onthefly else None,
                   "dtype": dt, "index": i})
    return ts


def run_planner(case, world, rank=0, noise_cache=False, field_slots=0):
    params = case.params()
    pl = StepPlanner(case.cfg, total_steps=case.spec["total_steps"], rank=rank, world=world)
    pl.noise_cache = noise_cache
    pl.field_slots = field_slots
    zc = {} if noise_cache else None
    ts = make_tensors(params, case.dtypes, pl, world > 1)
    n = len(params)
    vals_all = iter(case.values)
    afters, metrics, snaps = [], [], []
    for _ in range(case.spec["steps"]):
        local = pl.start()
        Z = case.cfg.z_batch
        vals = [next(vals_all) for _ in range(2 * Z)]
        # every rank pushes its own stored pairs: slot j holds pair j's field at the last pass
        zf = {j: pl.seeds[j] for j in range(min(field_slots, Z))}
        prev = None
        for j in local:
            run_pass(ts, n, *_spec(pl.plus_pass(j, prev)), dev_values=_dev(pl.plus_pass(j, prev), vals), zcache=zc)
            snaps.append(flat([t["live"] if world > 1 else t["data"] for t in ts]))
            run_pass(ts, n, *_spec(pl.minus_pass(j)), zcache=zc)
            snaps.append(flat([t["live"] if world > 1 else t["data"] for t in ts]))
            prev = j
        spec, m = pl.finish(vals)
        run_pass(ts, n, spec.cfg, spec.streams, zcache=zc, zfield=zf)
        afters.append(flat(params))
        if world > 1:
            assert np.array_equal(flat([t["live"] for t in ts]), afters[-1])
        metrics.append(m)
    return afters, metrics, snaps


def _spec(s):
    return s.cfg, s.streams


def _dev(s, vals):
    p = s.cfg.dev_pair
    return None if p is None else (vals[2 * p], vals[2 * p + 1])


def run_oracle(case):
    params = case.params()
    opt = OracleZO(params, case.dtypes, case.cfg, total_steps=case.spec["total_steps"], noise="c", semantics="cuda")
    opt.record_trace = True
    it = iter(case.values)
    afters, metrics = [], []
    for _ in range(case.spec["steps"]):
        metrics.append(opt.step(lambda ps, b: (next(it), {}), [None] * case.cfg.z_batch))
        afters.append(flat(params))
    return afters, metrics, [flat(t) for t in opt.trace]


@pytest.mark.parametrize("name", GAUSSIAN)
def test_single_gpu_schedule_bit_exact(name):
    case = StepCase(_G, name)
    a_pl, m_pl, s_pl = run_planner(case, world=1)
    a_or, m_or, s_or = run_oracle(case)
    for a, b in zip(a_pl, a_or):
        assert np.array_equal(a, b)
    # every forward sees exactly the reference's perturbed parameters
    assert len(s_pl) == len(s_or)
    for a, b in zip(s_pl, s_or):
        assert np.array_equal(a, b)
    for x, y in zip(m_pl, m_or):
        for k in ("loss", "proj_grad", "proj_grad_clipped", "clip_frac", "lr", "clip_tau"):
            assert x[k] == y[k], k


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("name", ["mezo_bf16_z3", "seedwin_adam_bf16_z2", "clip_norm_bf16", "es_rank_f32",
                                  "wd_anchored_l1_bf16", "ema_adam_f32_z2"])
def test_sharded_schedule_master_matches_single_gpu(name, world):
    """Seed-sharded: each rank perturbs a live copy; the final pass replays every pair's
    rounding chain on the master, so every rank ends bit-identical to one GPU."""
    case = StepCase(_G, name)
    a1, m1, _ = run_planner(case, world=1)
    for rank in range(world):
        aw, mw, snaps = run_planner(case, world=world, rank=rank)
        for a, b in zip(aw, a1):
            assert np.array_equal(a, b), rank
        for x, y in zip(mw, m1):
            assert x["proj_grad"] == y["proj_grad"]


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("name", GAUSSIAN)
def test_noise_cache_schedule_contract(name, world):
    """With the noise cache on, every pass that reads a pair's field from the cache finds
    that pair's field there (stored by the pair's +eps pass, never overwritten before its
    last use), and the schedule is otherwise unchanged: same parameters and metrics."""
    case = StepCase(_G, name)
    for rank in range(world):   # every rank, including one without pairs when z_batch < world
        a0, m0, s0 = run_planner(case, world=world, rank=rank)
        a1, m1, s1 = run_planner(case, world=world, rank=rank, noise_cache=True)   # asserts the contract
        for a, b in zip(a0 + s0, a1 + s1):
            assert np.array_equal(a, b)
        for x, y in zip(m0, m1):
            assert x["proj_grad"] == y["proj_grad"]


def test_noise_cache_contract_violations_detected():
    """The interpreter's cache model rejects a load of a field the cache does not hold and
    a store placed before the load."""
    from oracle.pass_interp import check_noise_cache
    from zotitan_b200.kernels import Stream
    zc = {}
    check_noise_cache(zc, [Stream(5, (1e-3,), z_store=True)])
    check_noise_cache(zc, [Stream(5, (-2e-3,), z_load=True)])
    with pytest.raises(AssertionError):
        check_noise_cache(zc, [Stream(6, (1e-3,), z_load=True)])
    with pytest.raises(AssertionError):
        check_noise_cache(zc, [Stream(7, (1e-3,), z_store=True), Stream(5, (1e-3,), z_load=True)])


def test_sharded_first_local_pair_sees_reference_perturbation():
    """The first pair a rank evaluates is perturbed from the step's starting parameters,
    exactly like the reference's first pair."""
    case = StepCase(_G, "mezo_bf16_z3")
    _, _, s_or = run_oracle(case)
    _, _, s_w = run_planner(case, world=2, rank=0)
    assert np.array_equal(s_w[0], s_or[0]) and np.array_equal(s_w[1], s_or[1])


def test_planner_rejects_unsupported():
    from helpers import ns
    cfg = StepCase(_G, "mezo_f32_z1").cfg_dict
    cfg["perturbation"]["distribution"] = "low_rank"
    assert StepPlanner(ns(cfg)).materialized          # one rank: supported (materialised directions)
    assert StepPlanner(ns(cfg), world=2, rank=0).sharded   # sharded: the 2-D replay runs on the master
    cfg["mom"]["momentum_method"] = "seed_window"
    with pytest.raises(AssertionError, match="seed_window momentum is incompatible"):
        StepPlanner(ns(cfg))                           # refused as the reference refuses it (train_zo.py:268-270)
    cfg["mom"]["momentum_method"] = "none"
    cfg["perturbation"]["distribution"] = "sparse"
    with pytest.raises(NotImplementedError):
        StepPlanner(ns(cfg))
    cfg["perturbation"]["distribution"] = "gaussian"
    cfg["fitness"]["strategy"] = "centered_rank"
    cfg["shared_batch"] = False
    with pytest.raises(AssertionError):
        StepPlanner(ns(cfg))


def test_planner_stream_limit():
    """Seed-window momentum regenerates every pair in the last pass: more than 256
    streams is refused. Plain MeZO accumulates on the fly and needs one stream."""
    from helpers import ns
    cfg = StepCase(_G, "seedwin_f32_z1").cfg_dict
    cfg["z_batch"] = 300
    pl = StepPlanner(ns(cfg))
    pl.start()
    with pytest.raises(ValueError, match="noise streams"):
        pl.finish([1.0, 0.5] * 300)
    cfg = StepCase(_G, "mezo_f32_z1").cfg_dict
    cfg["z_batch"] = 300
    pl = StepPlanner(ns(cfg))
    assert pl.ge_onthefly
    pl.start()
    spec, _ = pl.finish([1.0, 0.5] * 300)
    assert len(spec.streams) == 1 and spec.cfg.ge_load


def test_planner_state_dict_roundtrip():
    """Exact resume: a planner restored from state_dict continues the same seed / window."""
    case = StepCase(_G, "seedwin_adam_bf16_z2")
    pl = StepPlanner(case.cfg)
    vals = iter(case.values)
    for _ in range(2):
        pl.start()
        pl.finish([next(vals) for _ in range(4)])
    sd = pl.state_dict()
    pl2 = StepPlanner(case.cfg)
    pl2.load_state_dict(sd)
    v = [next(vals) for _ in range(4)]
    pl.start(); pl2.start()
    s1, _ = pl.finish(v)
    s2, _ = pl2.finish(v)
    assert [(s.seed, s.chain, s.ge, s.mom) for s in s1.streams] == [(s.seed, s.chain, s.ge, s.mom) for s in s2.streams]


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("slots", [1, 2, 64])
@pytest.mark.parametrize("name", ["mezo_bf16_z3", "seedwin_adam_bf16_z2", "ema_adam_f32_z2", "es_rank_f32"])
def test_field_store_schedule_contract(name, world, slots):
    """With the field exchange, the last pass reads pairs j < field_slots from slot j of
    the field store (checked against the slots' seeds) and the other pairs from the noise
    cache or regenerated; the schedule's results are unchanged."""
    case = StepCase(_G, name)
    for rank in range(world):
        a0, m0, s0 = run_planner(case, world=world, rank=rank, noise_cache=True)
        a1, m1, s1 = run_planner(case, world=world, rank=rank, noise_cache=True, field_slots=slots)
        for a, b in zip(a0 + s0, a1 + s1):
            assert np.array_equal(a, b)
        for x, y in zip(m0, m1):
            assert x["proj_grad"] == y["proj_grad"]


def test_field_store_contract_violations_detected():
    from oracle.pass_interp import check_field_store
    from zotitan_b200.kernels import Stream
    check_field_store({0: 5, 1: 6}, [Stream(5, (1e-3,), z_field=0), Stream(6, (1e-3,), z_field=1)])
    with pytest.raises(AssertionError):
        check_field_store({0: 5, 1: 6}, [Stream(6, (1e-3,), z_field=0)])
    with pytest.raises(AssertionError):
        check_field_store({0: 5}, [Stream(5, (1e-3,), z_field=0, z_load=True)])
