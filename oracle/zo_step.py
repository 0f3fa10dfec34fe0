"""Oracle restatement of the reference optimizer step (test infrastructure only).

Follows ``ZOOptimizer`` in zotitan/train_zo.py op by op over fp32 carrier arrays
(values exact in each parameter's dtype), with the noise and every rounding done by
the C oracle (oracle/philox_oracle.c). It materialises z exactly like the
reference does (:295-322) and applies one torch op at a time, so it is an
independent check of the fused CUDA passes, which never materialise z.

``cfg`` is duck-typed: any object with the reference ``ZOConfig`` attribute tree
(zotitan/train_zo.py:157-197) works, so the reference's own config objects and
the product's mirror of them are both accepted.
"""
from __future__ import annotations

import collections
import math

import numpy as np

from . import philox as ph


def wsd_value(step, total_steps, lo, hi, cfg):
    """zotitan/schedule.py:51-63."""
    if total_steps == 0:
        return hi
    warmup_end = cfg.warmup_frac * total_steps
    decay_start = (1.0 - cfg.decay_frac) * total_steps
    if step < warmup_end:
        return lo + (hi - lo) * step / max(warmup_end, 1.0)
    if step < decay_start:
        return hi
    t = min((step - decay_start) / max(total_steps - decay_start, 1.0), 1.0)
    return lo + 0.5 * (hi - lo) * (1.0 + math.cos(math.pi * t))


def f32(x) -> float:
    """Round a Python float to fp32 (torch's opmath for a Scalar on fp32/bf16 math)."""
    return float(np.float32(x))


class OracleZO:
    """``ZOOptimizer`` (zotitan/train_zo.py:242-606) on numpy carriers.

    params: list of fp32 arrays (shaped like the parameters), dtypes: per-tensor
    ``oracle.philox`` dtype code. Arrays are updated in place.
    """

    def __init__(self, params, dtypes, cfg, total_steps=0, noise="c", semantics="cuda"):
        """noise: "c" (C oracle), "numpy" (Triton-interpreter evaluation) or a callable
        (key, n) -> fp32 array. semantics: how torch turns a Python scalar into the
        multiplier of a bf16/fp16 op. "cuda": fp32 opmath everywhere (torch's CUDA
        foreach and TensorIterator kernels; what the reference does on a GPU).
        "cpu": torch's CPU kernels, which convert the scalar to the tensor's reduced
        dtype for ``_foreach_mul_(list, float)`` and for ``add_(other, alpha)`` when
        both tensors share that dtype (what the reference does in the CPU goldens)."""
        self.noise = ph.randn if noise == "c" else ph.randn_numpy if noise == "numpy" else noise
        assert semantics in ("cpu", "cuda")
        self.semantics = semantics
        self.params = params
        self.dtypes = list(dtypes)
        self.cfg = cfg
        self._t = 0
        self._total_steps = total_steps
        self.has_momentum = cfg.mom.momentum_method != "none"
        self._seed_ctr = 0
        self.trace = []                      # perturbed parameter snapshots, for tests
        self.record_trace = False
        self._pg_hist = (collections.deque(maxlen=cfg.clip.window)
                         if cfg.clip.strategy != "none" and cfg.clip.clip_pct > 0 else None)
        if cfg.mom.momentum_method == "stored_ema":
            self.m = [np.zeros_like(p) for p in params]
        elif cfg.mom.momentum_method == "seed_window":
            cap = cfg.seed_window.size if cfg.seed_window.size > 0 else None
            self.seed_buf = collections.deque(maxlen=cap)
            self.proj_buf = collections.deque(maxlen=cap)
        if cfg.mom.second_moment:
            self.v = [np.zeros_like(p) for p in params]
        self._wd_enabled = cfg.weight_decay.strategy != "none" and cfg.weight_decay.lambda_ > 0
        if cfg.weight_decay.strategy == "anchored" and self._wd_enabled:
            self.theta_0 = [p.copy() for p in params]
        self.shaping = cfg.fitness.strategy != "none"

    def _alpha(self, dt_self, dt_other, a):
        """alpha of ``self.add_(other, alpha=a)``."""
        if self.semantics == "cpu":
            return ph.alpha_for(dt_self, dt_other, a)
        return f32(a)

    def _mul_scalar(self, dt, a):
        """scalar of ``torch._foreach_mul_(list, a)`` with a Python float a."""
        if self.semantics == "cpu":
            return ph.alpha_for(dt, dt, a)
        return f32(a)

    # -- noise (:287-322) -----------------------------------------------------
    def _draw_seeds(self, n):
        seeds = list(range(self._seed_ctr, self._seed_ctr + n))
        self._seed_ctr += n
        return seeds

    def sample_z(self, seed):
        n = len(self.params)
        dist = self.cfg.perturbation.distribution
        out = []
        for i, p in enumerate(self.params):
            key = ph.param_key(seed, n, i)
            z = self.noise(key, p.size).reshape(p.shape)
            if p.ndim >= 2 and dist == "low_rank":
                z = self._low_rank_z(seed, i, p)
            elif p.ndim >= 2 and dist != "gaussian":
                raise NotImplementedError(dist)
            out.append(z)
        return out

    def _low_rank_z(self, seed, i, p):
        """low_rank branch (:304-320): z = P @ Psi in the param dtype, Frobenius-normalised."""
        n = len(self.params)
        dt = self.dtypes[i]
        m, r = p.shape[0], min(self.cfg.perturbation.rank, p.shape[0])
        P = ph.rounded(dt, self.noise(ph.param_key(seed, n, i + 2 * n), m * r).reshape(m, r))
        Psi = ph.rounded(dt, self.noise(ph.param_key(seed, n, i + n), r * p.shape[1]).reshape(r, p.shape[1]))
        z = ph.rounded(dt, (P.astype(np.float64) @ Psi.astype(np.float64)).astype(np.float32))
        # z.norm() is a 0-dim tensor of z's dtype; `x + 1e-7` stays in that dtype and
        # `float / tensor` is reciprocal(tensor) * float, each rounded to the dtype.
        r1 = lambda x: float(ph.rounded(dt, np.array([x], dtype=np.float32))[0])  # noqa: E731
        norm = r1(np.float32(np.sqrt(np.sum(z.astype(np.float64) ** 2))))
        t = r1(np.float32(norm) + np.float32(1e-7))
        scale = r1(np.float32(np.float32(1.0) / np.float32(t)) * np.float32(p.size ** 0.5))
        return ph.mul_scalar(dt, np.ascontiguousarray(z), scale)

    # -- passes ---------------------------------------------------------------
    def _apply_z(self, z, scale):
        """_apply_z (:350-351): params += scale * z, one rounding per tensor op."""
        a = f32(scale)
        for p, zz, dt in zip(self.params, z, self.dtypes):
            ph.add_scaled_(dt, p.reshape(-1), zz.reshape(-1), a)

    def run_forward_passes(self, score_fn, batch, z):
        eps = self.cfg.eps
        self._apply_z(z, +eps)
        if self.record_trace:
            self.trace.append([p.copy() for p in self.params])
        pos = score_fn(self.params, batch)
        self._apply_z(z, -2 * eps)
        if self.record_trace:
            self.trace.append([p.copy() for p in self.params])
        neg = score_fn(self.params, batch)
        self._apply_z(z, +eps)
        return pos, neg

    # -- optimizer state (:324-346, :409-425) ---------------------------------
    def _reconstruct_momentum_from_seeds(self):
        beta1 = self.cfg.mom.beta1
        weights = [beta1 ** i for i in range(len(self.seed_buf))]
        total = sum(weights) + 1e-12
        mom = [np.zeros_like(p) for p in self.params]
        for step_seeds, step_pg, sw in zip(self.seed_buf, self.proj_buf, weights):
            w = sw / (len(step_seeds) * total)
            for seed, pg in zip(step_seeds, step_pg):
                a = f32(w * pg)
                for mm, zz, dt in zip(mom, self.sample_z(seed), self.dtypes):
                    ph.add_scaled_(dt, mm.reshape(-1), zz.reshape(-1), a)
        return mom

    def _get_gradient_ema(self):
        mc = self.cfg.mom
        if mc.momentum_method == "stored_ema":
            bc = 1.0 - mc.beta1 ** self._t
            s = f32(bc + mc.denom_eps)
            if self.semantics == "cuda":   # CUDA tensor / scalar multiplies by the fp32 reciprocal
                r = float(np.float32(1.0) / np.float32(s))
                return [ph.mul_scalar(dt, m, r) for m, dt in zip(self.m, self.dtypes)]
            return [ph.div_scalar(dt, m, s) for m, dt in zip(self.m, self.dtypes)]
        return self._reconstruct_momentum_from_seeds()

    def _update_optimizer_state(self, grad_est, pair_seeds, pair_grads):
        mc = self.cfg.mom
        if mc.momentum_method == "stored_ema":
            for i, dt in enumerate(self.dtypes):
                self.m[i] = ph.mul_scalar(dt, self.m[i], self._mul_scalar(dt, mc.beta1))
                a = self._alpha(dt, self._ge_dt[i], 1 - mc.beta1)
                ph.add_scaled_(dt, self.m[i].reshape(-1), grad_est[i].reshape(-1), a)
        elif mc.momentum_method == "seed_window":
            self.seed_buf.appendleft(pair_seeds)
            self.proj_buf.appendleft(pair_grads)
        if mc.second_moment:
            for i, dt in enumerate(self.dtypes):
                self.v[i] = ph.mul_scalar(dt, self.v[i], self._mul_scalar(dt, mc.beta2))
                g = np.ascontiguousarray(grad_est[i], dtype=np.float32)
                ph.addcmul_(dt, self.v[i].reshape(-1), g.reshape(-1), g.reshape(-1), f32(1 - mc.beta2))

    def _apply_update(self, grad, lr):
        """_apply_update (:376-407), eager semantics; lr is fp32 (torch.tensor(lr))."""
        mc = self.cfg.mom
        wd = self.cfg.weight_decay
        lr32 = f32(lr)
        lam = f32(f32(wd.lambda_) * lr32)
        for i, (p, dt) in enumerate(zip(self.params, self.dtypes)):
            g = np.ascontiguousarray(grad[i], dtype=np.float32).reshape(-1)
            pf = p.reshape(-1)
            if mc.second_moment:
                bc2 = 1.0 - mc.beta2 ** self._t
                vh = ph.div_scalar(dt, self.v[i].reshape(-1), f32(bc2))
                ph.sqrt_add_(dt, vh, self._mul_scalar(dt, mc.denom_eps))
                ph.addcdiv_(dt, pf, g, vh, -lr32)
            else:
                gdt = dt if self.has_momentum else self._ge_dt[i]
                ph.add_scaled_(dt, pf, g, self._alpha(dt, gdt, -lr32))
            if wd.strategy == "standard":
                p[...] = ph.mul_scalar(dt, pf, f32(1.0 - lam)).reshape(p.shape)
            elif wd.strategy == "anchored":
                ph.anchored_(dt, pf, self.theta_0[i].reshape(-1), self._alpha(dt, dt, lam),
                             wd.penalty == "l1")

    # -- clipping / shaping (:427-508) -----------------------------------------
    def _clip_threshold(self):
        cc = self.cfg.clip
        if self._pg_hist is None or not self._pg_hist:
            return float("inf")
        xs = sorted(self._pg_hist)
        return xs[min(len(xs) - 1, int((1.0 - cc.clip_pct) * len(xs)))]

    def _apply_grad_clip(self, grad_est, pg, pgc, tau):
        clip = self.cfg.clip
        z_batch = len(pg)
        clip_scale = 1.0
        if clip.strategy == "norm" and math.isfinite(tau):
            pg_norm = math.sqrt(sum(g * g for g in pg))
            clip_scale = min(1.0, tau * math.sqrt(z_batch) / (pg_norm + 1e-12))
            if clip_scale < 1.0:
                for i, dt in enumerate(self.dtypes):
                    gdt = dt if self._ge_in_param_dtype else ph.F32
                    grad_est[i] = ph.mul_scalar(gdt, np.ascontiguousarray(grad_est[i]),
                                                self._mul_scalar(gdt, clip_scale))
                pgc = [g * clip_scale for g in pgc]
        if self._pg_hist is not None:
            self._pg_hist.extend(abs(g) for g in pg)
        if clip.strategy == "per_pair" and math.isfinite(tau):
            clip_frac = sum(abs(g) > tau for g in pg) / z_batch
        elif clip.strategy == "norm":
            clip_frac = float(clip_scale < 1.0)
        else:
            clip_frac = 0.0
        return pgc, clip_frac

    @staticmethod
    def _centered_ranks(fitness):
        n = len(fitness)
        if n < 2:
            return [0.0] * n
        order = sorted(range(n), key=lambda i: fitness[i])
        ranks = [0.0] * n
        for r, i in enumerate(order):
            ranks[i] = r / (n - 1) - 0.5
        return ranks

    def _shape_fitness(self, vals):
        u = self._centered_ranks([-v for v in vals])
        return [u[2 * j + 1] - u[2 * j] for j in range(len(vals) // 2)]

    def _grpo_advantages(self, vals):
        n = len(vals)
        mean = sum(vals) / n
        adv = [mean - v for v in vals]
        if self.cfg.fitness.normalize_std:
            std = math.sqrt(sum(a * a for a in adv) / n)
            adv = [a / (std + 1e-8) for a in adv]
        return [adv[2 * j + 1] - adv[2 * j] for j in range(n // 2)]

    # -- step (:510-606) --------------------------------------------------------
    def step(self, score_fn, batches):
        """score_fn(params, batch) -> (value, metrics): value a float (fp32-exact)."""
        self._t += 1
        cfg = self.cfg
        z_batch = cfg.z_batch
        tau = self._clip_threshold()
        clip_in_loop = cfg.clip.strategy == "per_pair" and math.isfinite(tau)
        lr = wsd_value(self._t, self._total_steps, 0.0, cfg.base.lr, cfg.base.lr_wsd)
        pair_seeds = self._draw_seeds(z_batch)
        self._ge_in_param_dtype = z_batch > 1
        self._ge_dt = list(self.dtypes) if z_batch > 1 else [ph.F32] * len(self.dtypes)
        grad_est = None
        vals, pgs, pgcs, metric_dicts = [], [], [], []
        two_eps = np.float32(2 * cfg.eps)
        for j, batch in enumerate(batches):
            z = self.sample_z(pair_seeds[j])
            (vp, mp), (vn, mn) = self.run_forward_passes(score_fn, batch, z)
            vp, vn = np.float32(vp), np.float32(vn)
            if self.semantics == "cuda":
                pg = np.float32(np.float32(vp - vn) * (np.float32(1.0) / two_eps))
            else:
                pg = np.float32(np.float32(vp - vn) / two_eps)
            pgc = np.float32(min(max(pg, -tau), tau)) if clip_in_loop else pg
            if not self.shaping:
                if z_batch == 1:
                    grad_est = [ph.mul_scalar(ph.F32, np.ascontiguousarray(zz), float(pgc)) for zz in z]
                else:
                    if grad_est is None:
                        grad_est = [np.zeros_like(p) for p in self.params]
                    if self.semantics == "cuda":
                        a = float(np.float32(pgc * (np.float32(1.0) / np.float32(z_batch))))
                    else:
                        a = float(np.float32(pgc / np.float32(z_batch)))
                    for g, zz, dt in zip(grad_est, z, self.dtypes):
                        ph.add_scaled_(dt, g.reshape(-1), zz.reshape(-1), a)
            vals += [float(vp), float(vn)]
            pgs.append(float(pg))
            pgcs.append(float(pgc))
            metric_dicts += [mp, mn]
        mean_loss = sum(vals) / len(vals)
        if self.shaping:
            pgc_l = (self._grpo_advantages(vals) if cfg.fitness.strategy == "grpo"
                     else self._shape_fitness(vals))
            grad_est = [np.zeros_like(p) for p in self.params]
            self._ge_in_param_dtype = True
            self._ge_dt = list(self.dtypes)
            for j, seed in enumerate(pair_seeds):
                a = f32(pgc_l[j] / z_batch)
                for g, zz, dt in zip(grad_est, self.sample_z(seed), self.dtypes):
                    ph.add_scaled_(dt, g.reshape(-1), zz.reshape(-1), a)
            clip_frac = 0.0
        else:
            pgc_l, clip_frac = self._apply_grad_clip(grad_est, pgs, pgcs, tau)
        self._update_optimizer_state(grad_est, pair_seeds, pgc_l)
        m_t = self._get_gradient_ema() if self.has_momentum else grad_est
        self._apply_update(m_t, lr)
        metrics = {
            "loss": mean_loss,
            "proj_grad": sum(pgs) / z_batch,
            "proj_grad_clipped": sum(pgc_l) / z_batch,
            "clip_frac": clip_frac,
            "clip_tau": tau if math.isfinite(tau) else None,
            "lr": lr,
        }
        if self.shaping:
            metrics["fit_rms"] = (sum(s * s for s in pgc_l) / z_batch) ** 0.5
        agg, cnt = {}, {}
        for d in metric_dicts:
            for k, v in (d or {}).items():
                if v is None:
                    continue
                agg[k] = agg.get(k, 0.0) + float(v)
                cnt[k] = cnt.get(k, 0) + 1
        metrics.update({k: agg[k] / cnt[k] for k in agg})
        return metrics
