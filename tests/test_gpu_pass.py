"""GPU parity of the fused pass (zt_pass) against the oracle's pass interpreter.

Given the same noise (the CUDA Gaussians, themselves pinned bit-exact to native
Triton by test_gpu_noise.py), every buffer the pass writes must be bit-identical to
the oracle's op-by-op evaluation: 0 ulp. One table mixes fp32/bf16/fp16 tensors of
ragged sizes (1, 7, 8, 1023, 2048, 2049, 4099, 100003) and a tensor whose storage is
not 16-byte aligned, so the unit mapping, vector and scalar paths are all covered.
A second check uses the fully independent C-oracle noise with a tolerance.
"""
import numpy as np
import pytest
import torch

from oracle import philox as ph
from oracle.pass_interp import run_pass

pytestmark = pytest.mark.gpu

TDT = {ph.F32: torch.float32, ph.BF16: torch.bfloat16, ph.F16: torch.float16}
SPECS = [(1, ph.BF16), (7, ph.F32), (8, ph.F16), (1023, ph.BF16), (2048, ph.F32), (2049, ph.BF16),
         (4099, ph.F16), (100003, ph.BF16), (5000, ph.F32), (777, "unaligned")]


@pytest.fixture(scope="module")
def K():
    from zotitan_b200 import kernels
    return kernels


def cuda_noise(K):
    cache = {}

    def noise(key, n):
        if (key, n) not in cache:
            cache[(key, n)] = K.randn(key, n, "cuda").cpu().numpy()
        return cache[(key, n)]
    return noise


def make_case(seed, with_live=False, with_m=False, with_v=False, with_anchor=False, with_ge=False, specs=SPECS):
    rng = np.random.default_rng(seed)
    host, dev, keep = [], {"data": [], "live": [], "m": [], "v": [], "anchor": [], "ge": []}, []
    for i, (n, dt) in enumerate(specs):
        unaligned = dt == "unaligned"
        dt = ph.BF16 if unaligned else dt
        def arr(scale, positive=False):
            x = rng.standard_normal(n).astype(np.float32) * scale
            return ph.rounded(dt, np.abs(x) if positive else x)
        t = {"data": arr(0.02), "dtype": dt, "index": i,
             "live": arr(0.02) if with_live else None,
             "m": arr(0.5) if with_m else None,
             "v": arr(0.01, positive=True) if with_v else None,
             "anchor": arr(0.02) if with_anchor else None,
             "ge": arr(0.3) if with_ge else None}
        host.append(t)
        for k in dev:
            if t[k] is None:
                dev[k].append(None)
                continue
            if unaligned:
                buf = torch.empty(n + 8, dtype=TDT[dt], device="cuda")
                view = buf[1:n + 1]
                view.copy_(torch.from_numpy(t[k]).to(TDT[dt]))
                keep.append(buf)
                dev[k].append(view)
            else:
                dev[k].append(torch.from_numpy(t[k]).to(TDT[dt]).cuda())
    return host, dev, keep


def table(K, dev, n_params):
    opt = {k: (dev[k] if any(x is not None for x in dev[k]) else None) for k in ("live", "m", "v", "anchor", "ge")}
    return K.ParamTable(dev["data"], n_params=n_params, **opt)


def compare(host, dev, keys=("data", "live", "m", "v", "ge")):
    for i, t in enumerate(host):
        for k in keys:
            if t[k] is None:
                continue
            got = dev[k][i].float().cpu().numpy()
            assert np.array_equal(got, t[k]), (i, k, t[k].size, t["dtype"], int(np.sum(got != t[k])))


N_PARAMS = 40  # tensors sit at indices 0..9 of a 40-long parameter list


def run_both(K, cfg, streams, dev_values=None, props=None, **case_kw):
    host, dev, keep = make_case(3, **case_kw)
    tab = table(K, dev, N_PARAMS)
    if props is not None:
        assert tab.plan.props == props
    if dev_values is not None:
        vals = torch.tensor(dev_values, dtype=torch.float32, device="cuda")
        cfg.dev_vals = vals.data_ptr()
    tab.run(cfg, streams)
    torch.cuda.synchronize()
    run_pass(host, N_PARAMS, cfg, streams, noise=cuda_noise(K), dev_values=dev_values)
    compare(host, dev)


@pytest.mark.parametrize("tau", [float("inf"), 3.0])
def test_onthefly_accumulation_with_device_coefficient(K, tau):
    """Restore pass of a pair that also accumulates its grad_est term, the coefficient
    computed on the device from the pair's two values (and clamped when clipping), then
    perturbs the next pair; and the first such pass, which starts grad_est from zero."""
    l = L()
    f = lambda x: float(np.float32(x))  # noqa: E731
    e = f(1e-3)
    for load in (True, False):
        cfg = K.PassCfg(ge_mode=l.ZT_GE_ACCUM, ge_load=load, ge_store=True, dev_inv2eps=f(1 / f(2e-3)),
                        dev_invz=f(1 / f(3)), dev_tau=f(tau) if tau != float("inf") else tau)
        streams = [K.Stream(50, (e,), ge_dev=True), K.Stream(51, (e,))]
        run_both(K, cfg, streams, dev_values=(2.0137, 2.0051), with_ge=True)
    # the last pass: loads grad_est, adds the last term with a host coefficient, updates
    cfg = K.PassCfg(ge_mode=l.ZT_GE_ACCUM, ge_load=True, update=True, lr=f(1e-2))
    run_both(K, cfg, [K.Stream(52, (e,), ge=f(0.7))], with_ge=True)


def L():
    from zotitan_b200 import _lib
    return _lib


UNIFORM_SIZES = [8, 2048, 4096, 24, 100000, 2056, 16]


@pytest.mark.parametrize("dt", [ph.BF16, ph.F32, ph.F16])
def test_uniform_plan_specialised_shapes(K, dt):
    """A plan whose tensors share one dtype and are whole, 16-byte aligned 8-element groups
    (ZT_PLAN_VEC8) runs the one-stream (+eps, -2eps, live copies), two-stream,
    restore + accumulate + perturb and replay (chains + grad_est + SGD, with and without
    weight decay) passes through kernels specialised for that dtype: every buffer they
    write is bit-identical to the oracle, including the last pass of the on-the-fly
    schedule (grad_est loaded, the last pair's term, SGD)."""
    l = L()
    f = lambda x: float(np.float32(x))  # noqa: E731
    e, m2 = f(1e-3), f(-2e-3)
    props = l.ZT_PLAN_VEC8 | {ph.BF16: l.ZT_PLAN_ALL_BF16, ph.F32: l.ZT_PLAN_ALL_F32, ph.F16: l.ZT_PLAN_ALL_F16}[dt]
    specs = [(n, dt) for n in UNIFORM_SIZES]
    live, data = l.ZT_BUF_LIVE, l.ZT_BUF_DATA
    acc = dict(ge_mode=l.ZT_GE_ACCUM, ge_store=True, dev_inv2eps=f(1 / f(2e-3)), dev_invz=f(1 / f(3)),
               dev_tau=float("inf"))
    cases = [
        (K.PassCfg(), [K.Stream(60, (e,))], None, {}),
        (K.PassCfg(), [K.Stream(61, (m2,))], None, {}),
        (K.PassCfg(src=live, dst=live), [K.Stream(62, (m2,))], None, {"with_live": True}),
        (K.PassCfg(src=data, dst=live), [K.Stream(63, (e,))], None, {"with_live": True}),
        (K.PassCfg(src=data, dst=data | live), [K.Stream(63, (e,))], None, {"with_live": True}),
        (K.PassCfg(), [K.Stream(64, (e,)), K.Stream(65, (e,))], None, {}),
        (K.PassCfg(ge_load=True, **acc), [K.Stream(66, (e,), ge_dev=True), K.Stream(67, (e,))], (2.0137, 2.0051),
         {"with_ge": True}),
        (K.PassCfg(ge_load=False, **acc), [K.Stream(68, (e,), ge_dev=True), K.Stream(69, (e,))], (1.5, 1.7),
         {"with_ge": True}),
        (K.PassCfg(ge_load=True, **{**acc, "dev_tau": f(3.0)}), [K.Stream(70, (e,), ge_dev=True), K.Stream(71, (e,))],
         (2.5, 2.0), {"with_ge": True}),
        (K.PassCfg(ge_mode=l.ZT_GE_ACCUM, ge_load=True, ge_store=True), [K.Stream(72, (e,), ge=f(0.3)),
                                                                        K.Stream(73, (e,))], None, {"with_ge": True}),
        (K.PassCfg(ge_mode=l.ZT_GE_ACCUM, ge_load=True, update=True, lr=f(1e-2)), [K.Stream(74, (e,), ge=f(0.7))],
         None, {"with_ge": True}),
        # replay shape: every stream's chain and grad_est term in registers, then SGD
        (K.PassCfg(ge_mode=l.ZT_GE_ACCUM, update=True, lr=f(1e-2)),
         [K.Stream(80 + j, (e, m2, e), ge=f(0.1 * (j - 3))) for j in range(7)], None, {}),
        (K.PassCfg(ge_mode=l.ZT_GE_ACCUM, update=True, lr=f(3e-2), wd=l.ZT_WD_STANDARD, wd_factor=f(1 - 3e-4)),
         [K.Stream(90, (), ge=f(0.4)), K.Stream(91, (e,), ge=f(-0.2)), K.Stream(92, (e, m2), ge=f(0.3)),
          K.Stream(93, (e, m2, e), ge=f(1.5))], None, {}),
        (K.PassCfg(dst=data | live, ge_mode=l.ZT_GE_ACCUM, update=True, lr=f(1e-2)),
         [K.Stream(94, (e, m2, e), ge=f(0.25)), K.Stream(95, (e, m2, e), ge=f(-0.5))], None, {"with_live": True}),
    ]
    for cfg, streams, dv, kw in cases:
        run_both(K, cfg, streams, dev_values=dv, props=props, specs=specs, **kw)


def test_perturb_and_restore_chain(K):
    e = float(np.float32(1e-3))
    run_both(K, K.PassCfg(), [K.Stream(11, (e,)), K.Stream(2**40 + 5, (e,))])
    run_both(K, K.PassCfg(), [K.Stream(11, (float(np.float32(-2e-3)),))])


def test_master_to_live_and_live_in_place(K):
    l = L()
    e = float(np.float32(1e-3))
    run_both(K, K.PassCfg(src=l.ZT_BUF_DATA, dst=l.ZT_BUF_LIVE), [K.Stream(5, (e,))], with_live=True)
    run_both(K, K.PassCfg(src=l.ZT_BUF_LIVE, dst=l.ZT_BUF_LIVE), [K.Stream(5, (-2 * e,))], with_live=True)


@pytest.mark.parametrize("variant", ["product_sgd", "accum_sgd_wd", "ema_adam", "seed_window_adam",
                                     "anchored_l1", "anchored_l2", "norm_clip_product", "norm_clip_accum",
                                     "sharded_replay"])
def test_final_pass_variants(K, variant):
    l = L()
    f = lambda x: float(np.float32(x))  # noqa: E731
    e = f(1e-3)
    base = dict(update=True, lr=f(3e-2))
    live = False
    if variant == "product_sgd":
        cfg = K.PassCfg(ge_mode=l.ZT_GE_PRODUCT, **base)
        streams = [K.Stream(9, (e,), ge=f(-1.7))]
    elif variant == "accum_sgd_wd":
        cfg = K.PassCfg(ge_mode=l.ZT_GE_ACCUM, wd=l.ZT_WD_STANDARD, wd_lam=f(0.01), wd_factor=f(1 - f(0.01)), **base)
        streams = [K.Stream(1, (), ge=f(0.3)), K.Stream(2, (), ge=f(-1.1)), K.Stream(3, (e,), ge=f(2.5))]
    elif variant == "ema_adam":
        cfg = K.PassCfg(ge_mode=l.ZT_GE_ACCUM, momentum=l.ZT_MOM_STORED_EMA, beta1=f(0.9), one_minus_beta1=f(0.1),
                        m_scale=f(1 / f(0.19)), second_moment=True, beta2=f(0.999), one_minus_beta2=f(1 - 0.999),
                        bc2=f(1 - 0.999 ** 2), denom_eps=f(1e-8), **base)
        streams = [K.Stream(4, (), ge=f(0.5)), K.Stream(5, (e,), ge=f(-0.25))]
    elif variant == "seed_window_adam":
        cfg = K.PassCfg(ge_mode=l.ZT_GE_ACCUM, momentum=l.ZT_MOM_SEED_WINDOW, second_moment=True, beta2=f(0.999),
                        one_minus_beta2=f(1 - 0.999), bc2=f(1 - 0.999 ** 3), denom_eps=f(1e-8), **base)
        streams = [K.Stream(20, (), ge=f(0.5), mom=f(0.2)), K.Stream(21, (e,), ge=f(-0.5), mom=f(0.1)),
                   K.Stream(18, (), mom=f(0.05)), K.Stream(19, (), mom=f(-0.07))]
    elif variant in ("anchored_l1", "anchored_l2"):
        code = l.ZT_WD_ANCHORED_L1 if variant.endswith("l1") else l.ZT_WD_ANCHORED_L2
        cfg = K.PassCfg(ge_mode=l.ZT_GE_PRODUCT, wd=code, wd_lam=f(0.05), wd_factor=f(0.95), **base)
        streams = [K.Stream(30, (e,), ge=f(0.9))]
    elif variant == "norm_clip_product":
        cfg = K.PassCfg(ge_mode=l.ZT_GE_PRODUCT, ge_scale=f(0.37), **base)
        streams = [K.Stream(31, (e,), ge=f(3.0))]
    elif variant == "norm_clip_accum":
        cfg = K.PassCfg(ge_mode=l.ZT_GE_ACCUM, ge_scale=f(0.37), **base)
        streams = [K.Stream(32, (), ge=f(3.0)), K.Stream(33, (e,), ge=f(-2.0))]
    else:  # sharded: replay each pair's chain on the master, write master and live
        live = True
        cfg = K.PassCfg(src=l.ZT_BUF_DATA, dst=l.ZT_BUF_DATA | l.ZT_BUF_LIVE, ge_mode=l.ZT_GE_ACCUM, **base)
        streams = [K.Stream(s, (e, f(-2e-3), e), ge=f(0.1 * s)) for s in range(40, 44)]
    need = dict(with_live=live, with_m=variant == "ema_adam", with_v="adam" in variant,
                with_anchor=variant.startswith("anchored"))
    run_both(K, cfg, streams, **need)


def test_pass_with_independent_oracle_noise(K):
    """Same pass against the C oracle's own noise (no CUDA in the checker). The two noise
    sources differ by at most 4 fp32 ulp of z (|z| < 8), so each coefficient c carries an
    absolute difference of at most 4 * 2^-21 * |c|: fp32 values within 8 ulp at scale
    plus that bound, bf16/fp16 within 1 ulp."""
    l = L()
    f = lambda x: float(np.float32(x))  # noqa: E731
    cfg = K.PassCfg(ge_mode=l.ZT_GE_ACCUM, update=True, lr=f(1e-2))
    streams = [K.Stream(7, (f(1e-3),), ge=f(0.4)), K.Stream(8, (), ge=f(-0.9))]
    host, dev, keep = make_case(5)
    tab = table(K, dev, N_PARAMS)
    before = [t["data"].copy() for t in host]
    tab.run(cfg, streams)
    torch.cuda.synchronize()
    run_pass(host, N_PARAMS, cfg, streams, noise=ph.randn)
    noise_atol = 4 * 2.0 ** -21 * (1e-3 + 1e-2 * (0.4 + 0.9))
    for i, t in enumerate(host):
        got = dev["data"][i].float().cpu().numpy()
        scale = np.maximum(np.abs(before[i]), np.abs(t["data"])) + 1e-6
        mant = 23 if t["dtype"] == ph.F32 else (7 if t["dtype"] == ph.BF16 else 10)
        ulp = np.exp2(np.floor(np.log2(scale)) - mant)
        diff = np.abs(got.astype(np.float64) - t["data"])
        if t["dtype"] == ph.F32:
            assert np.all(diff <= 8 * ulp + noise_atol), (i, float(diff.max()))
        else:
            assert np.all(diff <= ulp), (i, float((diff / ulp).max()))


def test_empty_and_large_stream_lists(K):
    l = L()
    host, dev, keep = make_case(9)
    tab = table(K, dev, N_PARAMS)
    tab.run(K.PassCfg(), [])             # no streams: copy-through
    torch.cuda.synchronize()
    compare(host, dev, keys=("data",))
    with pytest.raises(ValueError):
        tab.run(K.PassCfg(), [K.Stream(1)] * 257)
