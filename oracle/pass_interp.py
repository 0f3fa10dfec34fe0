"""Oracle interpreter of one fused pass (test infrastructure only).

Executes the semantics that include/zotitan_b200.h documents for ``zt_pass``, one
reference op at a time through the C oracle routines, over numpy carriers with z
materialised. Used to check (a) on CPU, that the host planner's pass schedule
reproduces the op-by-op optimizer step (oracle/zo_step.py), and (b) on GPU, that the
CUDA pass computes bit-identical results given the same noise.

tensors: list of dicts with keys data, live, m, v, anchor, ge (numpy fp32 carriers or
None), dtype (oracle.philox code) and index. cfg / streams: any objects with the
attribute names of zotitan_b200.kernels.PassCfg / Stream. dev_values: the (v+, v-) pair
a ge_dev stream reads (what cfg.dev_vals points at on the device).
"""
from __future__ import annotations

import numpy as np

from . import philox as ph

GE_NONE, GE_PRODUCT, GE_ACCUM = 0, 1, 2
MOM_NONE, MOM_STORED_EMA, MOM_SEED_WINDOW = 0, 1, 2
WD_NONE, WD_STANDARD, WD_ANCHORED_L2, WD_ANCHORED_L1 = 0, 1, 2, 3
BUF_DATA, BUF_LIVE = 1, 2


def dev_coefficient(cfg, dev_values):
    """(v+ - v-) * inv2eps, clamp to +-tau, * invz, each step in fp32."""
    vp, vn = (np.float32(x) for x in dev_values)
    pg = np.float32(np.float32(vp - vn) * np.float32(cfg.dev_inv2eps))
    tau = np.float32(cfg.dev_tau)
    pg = -tau if pg < -tau else (tau if pg > tau else pg)
    return float(np.float32(pg * np.float32(cfg.dev_invz)))


UNIT = 2048


def check_noise_cache(zcache, streams):
    """The noise-cache contract of zt_pass (ZT_STREAM_Z_LOAD / ZT_STREAM_Z_STORE): at most
    one loading and one storing stream, the load first, and a loading stream's field must
    be the one the cache holds (the last stored seed). ``zcache`` is a dict standing for
    the cache's contents; the interpreter itself always regenerates z, which is what a
    correct cache would return."""
    loads = [i for i, s in enumerate(streams) if getattr(s, "z_load", False)]
    stores = [i for i, s in enumerate(streams) if getattr(s, "z_store", False)]
    assert len(loads) <= 1 and len(stores) <= 1, "one noise-cache load and one store per pass"
    assert not (loads and stores) or loads[0] < stores[0], "the noise-cache load must precede the store"
    for i in loads:
        assert zcache.get("seed") == streams[i].seed, \
            f"noise cache holds seed {zcache.get('seed')}, stream {i} loads seed {streams[i].seed}"
    for i in stores:
        zcache["seed"] = streams[i].seed


def check_field_store(zfield, streams):
    """The field-store contract of zt_pass (ZT_STREAM_Z_FIELD): a stream reading slot s
    must find its own pair's field there. ``zfield`` maps slot -> the seed whose field the
    slot holds (what the pushes of the sharded step put there); a stream may not combine
    the field store with the noise cache. The interpreter regenerates z, which is what a
    correct store returns."""
    for i, s in enumerate(streams):
        slot = getattr(s, "z_field", None)
        if slot is None:
            continue
        assert not (getattr(s, "z_load", False) or getattr(s, "z_store", False)), \
            f"stream {i} combines the field store with the noise cache"
        assert zfield.get(slot) == s.seed, f"field-store slot {slot} holds {zfield.get(slot)}, stream {i} needs {s.seed}"


def run_pass(tensors, n_params, cfg, streams, noise=ph.randn, dev_values=None, zcache=None, zfield=None):
    """A unit range (cfg.unit_begin, cfg.unit_end) restricts the pass to those 2048-element
    units of the table (numbered in table order); elements outside are left untouched.
    ``zcache``: a dict modelling the noise cache, checked with check_noise_cache;
    ``zfield``: a dict modelling the field store, checked with check_field_store."""
    if zcache is not None:
        check_noise_cache(zcache, streams)
    if zfield is not None:
        check_field_store(zfield, streams)
    elif any(getattr(s, "z_field", None) is not None for s in streams):
        raise AssertionError("a stream reads the field store but none was given")
    dev_coef = dev_coefficient(cfg, dev_values) if dev_values is not None else None
    ub, ue = getattr(cfg, "unit_begin", 0), getattr(cfg, "unit_end", 0)
    base = 0
    for t in tensors:
        units = (t["data"].size + UNIT - 1) // UNIT
        lo_u, hi_u = base, base + units
        base += units
        if ue > 0:
            a, b = max(ub, lo_u), min(ue, hi_u)
            if a >= b:
                continue
            sub = {k: (v.reshape(-1)[(a - lo_u) * UNIT: min((b - lo_u) * UNIT, v.size)]
                       if isinstance(v, np.ndarray) else v) for k, v in t.items()}
            _run_tensor(sub, n_params, cfg, streams, noise, dev_coef, ctr_offset=(a - lo_u) * UNIT)
        else:
            _run_tensor(t, n_params, cfg, streams, noise, dev_coef, ctr_offset=0)


def _run_tensor(t, n_params, cfg, streams, noise, dev_coef, ctr_offset):
    dt, n = t["dtype"], t["data"].size
    src = t["live"] if cfg.src == BUF_LIVE else t["data"]
    th = np.ascontiguousarray(src, dtype=np.float32).reshape(-1).copy()
    ge = (t["ge"].reshape(-1).astype(np.float32).copy() if getattr(cfg, "ge_load", False)
          else np.zeros(n, np.float32))
    mom = np.zeros(n, np.float32)
    for s in streams:
        key = ph.param_key(s.seed, n_params, t["index"])
        z = noise(key, n) if ctr_offset == 0 else _noise_at(noise, key, ctr_offset, n)
        for a in s.chain:
            ph.add_scaled_(dt, th, z, a)
        if s.ge is not None or getattr(s, "ge_dev", False):
            c = dev_coef if getattr(s, "ge_dev", False) else s.ge
            if cfg.ge_mode == GE_PRODUCT:
                ge = ph.mul_scalar(ph.F32, z, c)
            else:
                ph.add_scaled_(dt, ge, z, c)
        if s.mom is not None:
            ph.add_scaled_(dt, mom, z, s.mom)
    if cfg.ge_scale is not None:
        ge = ph.mul_scalar(ph.F32 if cfg.ge_mode == GE_PRODUCT else dt, ge, cfg.ge_scale)
    if getattr(cfg, "ge_store", False):
        t["ge"][...] = ge.reshape(t["ge"].shape)
    if cfg.update:
        if cfg.momentum == MOM_STORED_EMA:
            m = ph.mul_scalar(dt, t["m"].reshape(-1).astype(np.float32), cfg.beta1)
            ph.add_scaled_(dt, m, ge, cfg.one_minus_beta1)
            t["m"][...] = m.reshape(t["m"].shape)
            g = ph.mul_scalar(dt, m, cfg.m_scale)
        elif cfg.momentum == MOM_SEED_WINDOW:
            g = mom
        else:
            g = ge
        if cfg.second_moment:
            v = ph.mul_scalar(dt, t["v"].reshape(-1).astype(np.float32), cfg.beta2)
            ph.addcmul_(dt, v, ge, ge, cfg.one_minus_beta2)
            t["v"][...] = v.reshape(t["v"].shape)
            vh = ph.div_scalar(dt, v, cfg.bc2)
            ph.sqrt_add_(dt, vh, cfg.denom_eps)
            ph.addcdiv_(dt, th, g, vh, -cfg.lr)
        else:
            ph.add_scaled_(dt, th, np.ascontiguousarray(g, dtype=np.float32), -cfg.lr)
        if cfg.wd == WD_STANDARD:
            th = ph.mul_scalar(dt, th, cfg.wd_factor)
        elif cfg.wd in (WD_ANCHORED_L1, WD_ANCHORED_L2):
            ph.anchored_(dt, th, t["anchor"].reshape(-1).astype(np.float32), cfg.wd_lam, cfg.wd == WD_ANCHORED_L1)
    if cfg.dst & BUF_DATA:
        t["data"][...] = th.reshape(t["data"].shape)
    if cfg.dst & BUF_LIVE:
        t["live"][...] = th.reshape(t["live"].shape)


def _noise_at(noise, key, off0, n):
    """Gaussians at element offsets off0 .. off0+n-1 of a tensor."""
    try:
        return noise(key, n, off0)
    except TypeError:
        return noise(key, off0 + n)[off0:]
