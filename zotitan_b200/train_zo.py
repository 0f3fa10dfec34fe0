"""Zeroth-order optimizer with the reference's API on B200-native fused passes.

Drop-in for zotitan/train_zo.py: the config tree (``ZOConfig`` and its sub-configs,
field for field, :30-197), ``ZOOptimizer(named_params, cfg, score_fn, total_steps)``
with ``.step(model, batches) -> dict`` (:242-606) and ``train_zo(...)`` (:609-675).

What changes underneath: the reference materialises fp32 noise for every tensor
with a Triton kernel and applies it with torch foreach ops (3 passes per pair plus a
grad_est buffer, momentum replay and the update). Here every pass is one
``zt_pass`` launch over all trainable tensors that generates the noise in registers
(include/zotitan_b200.h); with the noise cache (the default when it fits) a pair's
field is generated once, by the pass that applies its +eps, kept as fp32, and read back
by the pair's -2eps and restore passes:

  pair j:    [restore of pair j-1 (+eps z_{j-1}), its grad_est term] fused with
             +eps z_j ; score ; -2eps z_j ; score
  step end:  restore of the last pair + the remaining gradient-estimate terms +
             momentum replay + (m, v) update + parameter update + weight decay,
             one pass; no per-tensor z is materialised.

Arithmetic follows the reference's eager op order with the fp32 opmath scalars of
torch's CUDA kernels (tensor / Python scalar multiplies by the fp32 reciprocal),
one rounding to the parameter dtype per reference op.

Seed sharding (torch.distributed initialised with world size W > 1): rank r
evaluates pairs j = r, r+W, ...; the model reads a second ("live") copy of the
trainable tensors while the master copy stays unperturbed; one all-gather shares
the pair values; every rank then runs the same final pass over the master, which
also replays every pair's +eps/-2eps/+eps rounding chain so the result equals the
single-GPU sequence, and writes master and live.
"""
from __future__ import annotations

import collections
import math
import os
import time
from dataclasses import dataclass, field
from typing import Literal

import numpy as np
import torch

from . import _lib as L
from . import kernels as K
from .data import PrefetchLoader, get_batches
from .distributed import gather_pair_values, local_pairs, world_info
from .kernels import ParamTable, PassCfg, Stream, param_key, randn
from .schedule import BaseTrainConfig, wsd_is_constant, wsd_value


# ── configuration (zotitan/train_zo.py:30-197, field for field) ───────────────

@dataclass
class MomentumConfig:
    momentum_method: Literal["none", "stored_ema", "seed_window"] = "none"
    """none | stored_ema (full EMA buffer m) | seed_window (m rebuilt from recent seeds)."""
    beta1: float = 0.9
    beta2: float = 0.999
    second_moment: bool = False
    """Materialised EMA v of grad_est^2; the update divides by the bias-corrected sqrt(v)."""
    denom_eps: float = 1e-8


@dataclass
class SeedWindowConfig:
    size: int = 0
    """Number of past steps' seeds kept for seed_window momentum (0: unbounded)."""


@dataclass
class ClipConfig:
    strategy: Literal["none", "per_pair", "norm"] = "none"
    clip_pct: float = 0.0
    window: int = 1000


@dataclass
class PerturbationConfig:
    distribution: Literal["gaussian", "low_rank", "polar"] = "gaussian"
    rank: int = 64


@dataclass
class WeightDecayConfig:
    strategy: Literal["none", "standard", "anchored"] = "none"
    lambda_: float = 0.0
    penalty: Literal["l2", "l1"] = "l2"


@dataclass
class FitnessShapingConfig:
    strategy: Literal["none", "centered_rank", "grpo"] = "none"
    normalize_std: bool = True


@dataclass
class ZOConfig:
    base: BaseTrainConfig = field(default_factory=lambda: BaseTrainConfig(lr=1e-5, ckpt_every=5_000))
    eps: float = 1e-3
    batch_size: int = 40
    z_batch: int = 1
    shared_batch: bool = False
    mom: MomentumConfig = field(default_factory=MomentumConfig)
    seed_window: SeedWindowConfig = field(default_factory=SeedWindowConfig)
    perturbation: PerturbationConfig = field(default_factory=PerturbationConfig)
    clip: ClipConfig = field(default_factory=ClipConfig)
    fitness: FitnessShapingConfig = field(default_factory=FitnessShapingConfig)
    weight_decay: WeightDecayConfig = field(default_factory=WeightDecayConfig)


def zeropower_via_newtonschulz(G: torch.Tensor) -> torch.Tensor:
    """Polar factor of G by the hybrid Newton-Schulz iteration the reference's polar
    perturbation uses (zotitan/train_zo.py:198-222; DeepSeek-V4 section 2.4): in bf16, the
    wide orientation, X / (||X|| + 1e-7), 8 steps of aX + b(XX^T)X + c(XX^T)^2 X with
    (3.4445, -4.7750, 2.0315), then 2 with (2, -1.5, 0.5). Evaluated eagerly (the reference
    wraps it in torch.compile, whose fusion may round differently)."""
    assert G.ndim >= 2
    X = G.to(torch.bfloat16)
    transposed = X.size(0) > X.size(1)
    if transposed:
        X = X.T
    X = X / (X.norm() + 1e-7)
    for a, b, c in [(3.4445, -4.7750, 2.0315)] * 8 + [(2.0, -1.5, 0.5)] * 2:
        A = X @ X.T
        X = a * X + b * (A @ X) + c * (A @ A @ X)
    if transposed:
        X = X.T
    return X.to(G.dtype)


# ── host-side planning (no device work; unit-testable on CPU) ───────────────────

def f32(x) -> float:
    """Round a Python float to fp32, as torch's CUDA kernels take a Scalar (opmath)."""
    return float(np.float32(x))


def f32_recip(x) -> float:
    """fp32(1 / fp32(x)): the multiplier torch's CUDA division by a Python scalar uses."""
    return float(np.float32(1.0) / np.float32(x))


@dataclass
class PassSpec:
    cfg: PassCfg
    streams: list
    unit_ranges: list | None = None   # run once per [unit_begin, unit_end) range, in order


class StepPlanner:
    """Host half of ``ZOOptimizer.step``: seed counter, clip history, seed window,
    fitness shaping, the pass schedule and every scalar the passes take.

    ``world > 1`` selects the seed-sharded schedule (master/live copies); ``sharded``
    forces it on or off (a one-rank group can run the sharded schedule)."""

    def __init__(self, cfg: ZOConfig, total_steps: int = 0, rank: int = 0, world: int = 1,
                 sharded: bool | None = None):
        dist_kind = cfg.perturbation.distribution
        if dist_kind not in ("gaussian", "low_rank", "polar"):
            raise NotImplementedError(f"perturbation.distribution={dist_kind!r}")
        # low_rank / polar directions of 2-D tensors (train_zo.py:304-320) are materialised
        # per pair with the reference's own ops; 1-D tensors keep the fused Gaussian passes
        self.materialized = dist_kind != "gaussian"
        self.cfg = cfg
        self._t = 0
        self._total_steps = total_steps
        self._seed_ctr = 0
        self.rank, self.world = rank, world
        self.sharded = world > 1 if sharded is None else bool(sharded)
        # the reference refuses this combination itself (zotitan/train_zo.py:268-270)
        if dist_kind != "gaussian":
            assert cfg.mom.momentum_method != "seed_window", \
                "seed_window momentum is incompatible with non-gaussian perturbation distributions"
        # Sharded update: the step's last pass covers only this rank's unit range of a
        # flat parameter layout, followed by an all-gather of the updated master (set by
        # ZOOptimizer when the layout is in place).
        self.unit_ranges: list[tuple[int, int]] | None = None
        # Field exchange (sharded update): pairs j < field_slots have their field pushed into
        # every rank's field store, and the last pass reads it from there (slot j).
        self.field_slots = 0
        self.has_momentum = cfg.mom.momentum_method != "none"
        self._pg_hist = (collections.deque(maxlen=cfg.clip.window)
                         if cfg.clip.strategy != "none" and cfg.clip.clip_pct > 0 else None)
        if cfg.mom.momentum_method == "seed_window":
            cap = cfg.seed_window.size if cfg.seed_window.size > 0 else None
            self.seed_buf = collections.deque(maxlen=cap)
            self.proj_buf = collections.deque(maxlen=cap)
        self.shaping = cfg.fitness.strategy != "none"
        if self.shaping:
            assert cfg.shared_batch, (
                f"{cfg.fitness.strategy} fitness shaping requires shared_batch=True, because the population "
                "transform is only comparable when all z are scored on the same batch.")
            assert not (cfg.clip.strategy != "none" and cfg.clip.clip_pct > 0), \
                f"{cfg.fitness.strategy} fitness shaping is mutually exclusive with proj_grad clipping."
        wd = cfg.weight_decay
        self.wd_enabled = wd.strategy != "none" and wd.lambda_ > 0
        self.needs_m = cfg.mom.momentum_method == "stored_ema"
        self.needs_v = cfg.mom.second_moment
        self.needs_anchor = wd.strategy == "anchored" and self.wd_enabled
        # grad_est is consumed by the update itself (no momentum), the stored EMA, or v.
        self.need_ge = (not self.has_momentum) or cfg.mom.momentum_method == "stored_ema" or cfg.mom.second_moment
        # Single-GPU, several pairs, coefficients known pair by pair: each restore pass
        # also accumulates its pair into a grad_est buffer in the parameter dtype (the
        # reference's own accumulation, train_zo.py:555-556), with the coefficient computed
        # on the device from the pair's values, so the last pass needs one noise stream
        # instead of z_batch. Fitness shaping needs the whole population first and seed-
        # window momentum regenerates every seed anyway; the sharded schedule must replay
        # the pairs in order on the master.
        self.ge_onthefly = (not self.sharded and cfg.z_batch > 1 and not self.shaping and self.need_ge
                            and cfg.mom.momentum_method != "seed_window")
        # Noise cache (set by ZOOptimizer): the +eps pass of pair j also writes z_j to an
        # fp32 buffer, and the pair's -2eps and restore passes read it back instead of
        # regenerating it (one Philox/Box-Muller evaluation per element and pair instead
        # of three on one GPU, one instead of two for a rank's own pairs when sharded).
        self.noise_cache = False

    # -- reference helpers (zotitan/train_zo.py:287-293, 427-508) ----------------
    def _draw_seeds(self, n):
        seeds = list(range(self._seed_ctr, self._seed_ctr + n))
        self._seed_ctr += n
        return seeds

    def _clip_threshold(self):
        cc = self.cfg.clip
        if self._pg_hist is None or not self._pg_hist:
            return float("inf")
        xs = sorted(self._pg_hist)
        return xs[min(len(xs) - 1, int((1.0 - cc.clip_pct) * len(xs)))]

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

    # -- schedule -------------------------------------------------------------------
    def start(self) -> list[int]:
        """Begin a step; returns the pairs this rank evaluates, in order."""
        self._t += 1
        cfg = self.cfg
        self.tau = self._clip_threshold()
        self.clip_in_loop = cfg.clip.strategy == "per_pair" and math.isfinite(self.tau)
        self.lr = wsd_value(self._t, self._total_steps, lo=0.0, hi=cfg.base.lr, cfg=cfg.base.lr_wsd)
        self.seeds = self._draw_seeds(cfg.z_batch)
        self.local = local_pairs(cfg.z_batch, self.rank, self.world)
        return self.local

    def plus_pass(self, j: int, prev: int | None) -> PassSpec:
        """+eps z_j; single-GPU mode also restores the previous pair (+eps z_prev) first and,
        when accumulating on the fly, adds prev's grad_est contribution."""
        a = f32(self.cfg.eps)
        nc = self.noise_cache
        if self.sharded:
            return PassSpec(PassCfg(src=L.ZT_BUF_DATA, dst=L.ZT_BUF_LIVE), [Stream(self.seeds[j], (a,), z_store=nc)])
        if self.ge_onthefly and prev is not None:
            cfg = PassCfg(src=L.ZT_BUF_DATA, dst=L.ZT_BUF_DATA, ge_mode=L.ZT_GE_ACCUM, ge_load=prev > 0,
                          ge_store=True, dev_pair=prev, dev_inv2eps=f32_recip(2 * self.cfg.eps),
                          dev_invz=f32_recip(self.cfg.z_batch),
                          dev_tau=f32(self.tau) if self.clip_in_loop else float("inf"))
            return PassSpec(cfg, [Stream(self.seeds[prev], (a,), ge_dev=True, z_load=nc),
                                  Stream(self.seeds[j], (a,), z_store=nc)])
        streams = (([Stream(self.seeds[prev], (a,), z_load=nc)] if prev is not None else [])
                   + [Stream(self.seeds[j], (a,), z_store=nc)])
        return PassSpec(PassCfg(src=L.ZT_BUF_DATA, dst=L.ZT_BUF_DATA), streams)

    def minus_pass(self, j: int) -> PassSpec:
        """-2eps z_j (train_zo.py:369)."""
        a = f32(-2 * self.cfg.eps)
        buf = L.ZT_BUF_LIVE if self.sharded else L.ZT_BUF_DATA
        return PassSpec(PassCfg(src=buf, dst=buf), [Stream(self.seeds[j], (a,), z_load=self.noise_cache)])

    def finish(self, vals: list[float]) -> tuple[PassSpec, dict]:
        """vals = [v+_0, v-_0, v+_1, v-_1, ...] for all pairs (fp32 values). Returns the
        final pass and the scalar metrics (loss, proj_grad, ..., lr)."""
        cfg = self.cfg
        Z = cfg.z_batch
        mc = cfg.mom
        eps_inv = f32_recip(2 * cfg.eps)
        pg, pgc = [], []
        for j in range(Z):
            d = np.float32(np.float32(vals[2 * j]) - np.float32(vals[2 * j + 1]))
            g = np.float32(d * np.float32(eps_inv))  # (L+ - L-) / (2 eps) on CUDA (:544)
            pg.append(float(g))
            pgc.append(float(np.float32(min(max(float(g), -self.tau), self.tau))) if self.clip_in_loop else float(g))
        mean_loss = sum(vals) / len(vals)

        ge_mode = L.ZT_GE_NONE
        ge_coefs = [None] * Z
        ge_scale = None
        if self.shaping:  # (:568-578)
            pgc = (self._grpo_advantages(vals) if cfg.fitness.strategy == "grpo" else self._shape_fitness(vals))
            ge_mode = L.ZT_GE_ACCUM
            ge_coefs = [f32(pgc[j] / Z) for j in range(Z)]
            clip_frac = 0.0
        else:
            if Z == 1:
                ge_mode = L.ZT_GE_PRODUCT  # grad_est = z * pgc in fp32 (:552)
                ge_coefs = [f32(pgc[0])]
            else:
                ge_mode = L.ZT_GE_ACCUM    # zeros_like(p) += z * (pgc / Z) (:555-556)
                inv_z = f32_recip(Z)
                ge_coefs = [float(np.float32(np.float32(pgc[j]) * np.float32(inv_z))) for j in range(Z)]
            # norm clipping (:453-458) and the lagged history (:461-472)
            clip = cfg.clip
            clip_scale = 1.0
            if clip.strategy == "norm" and math.isfinite(self.tau):
                pg_norm = math.sqrt(sum(g * g for g in pg))
                clip_scale = min(1.0, self.tau * math.sqrt(Z) / (pg_norm + 1e-12))
                if clip_scale < 1.0:
                    ge_scale = f32(clip_scale)
                    pgc = [g * clip_scale for g in pgc]
            if self._pg_hist is not None:
                self._pg_hist.extend(abs(g) for g in pg)
            if clip.strategy == "per_pair" and math.isfinite(self.tau):
                clip_frac = sum(abs(g) > self.tau for g in pg) / Z
            elif clip.strategy == "norm":
                clip_frac = float(clip_scale < 1.0)
            else:
                clip_frac = 0.0

        if not self.need_ge:
            ge_mode = L.ZT_GE_NONE
            ge_scale = None
        # per-pair grad_est coefficients of this step (the materialised directions use them)
        self.last_ge = (ge_mode, list(ge_coefs), ge_scale)

        # seed-window state (:420-422) and replay weights (:337-345)
        mom_coefs = {}
        if mc.momentum_method == "seed_window":
            self.seed_buf.appendleft(list(self.seeds))
            self.proj_buf.appendleft(list(pgc))
            weights = [mc.beta1 ** i for i in range(len(self.seed_buf))]
            total = sum(weights) + 1e-12
            for i, (ss, pp, sw) in enumerate(zip(self.seed_buf, self.proj_buf, weights)):
                w = sw / (len(ss) * total)
                mom_coefs[i] = [f32(w * p) for p in pp]

        a_pos, a_neg = f32(cfg.eps), f32(-2 * cfg.eps)
        streams = []
        for j in range(Z):
            if self.sharded:
                chain = (a_pos, a_neg, a_pos)   # replay pair j's rounding chain on the master
            else:
                chain = (a_pos,) if j == Z - 1 else ()   # restore of the last pair (:371)
                if self.ge_onthefly and j < Z - 1:
                    continue                      # already restored and accumulated
            # the field still in the noise cache: the last pair (one GPU) or this rank's
            # last own pair (sharded replay); or pushed into the field store (slot j)
            field = self.sharded and j < self.field_slots
            cached = (bool(self.local) and j == self.local[-1]) if self.sharded else j == Z - 1
            streams.append(Stream(self.seeds[j], chain,
                                  ge_coefs[j] if ge_mode != L.ZT_GE_NONE else None,
                                  mom_coefs[0][j] if mom_coefs else None,
                                  z_load=self.noise_cache and cached and not field,
                                  z_field=j if field else None))
        for i in range(1, len(mom_coefs)):
            for s, c in zip(self.seed_buf[i], mom_coefs[i]):
                streams.append(Stream(s, (), None, c))
        if len(streams) > L.ZT_MAX_STREAMS:
            raise ValueError(f"step needs {len(streams)} noise streams > {L.ZT_MAX_STREAMS} "
                             "(reduce z_batch or seed_window.size)")

        t = self._t
        wd = cfg.weight_decay
        lr32 = f32(self.lr)
        wd_lam = f32(np.float32(wd.lambda_) * np.float32(lr32))
        wd_code = L.ZT_WD_NONE
        if wd.strategy == "standard":
            wd_code = L.ZT_WD_STANDARD
        elif wd.strategy == "anchored" and self.wd_enabled:
            wd_code = L.ZT_WD_ANCHORED_L1 if wd.penalty == "l1" else L.ZT_WD_ANCHORED_L2
        if self.sharded and self.unit_ranges is not None:
            dst = L.ZT_BUF_DATA                       # this rank's share of the master only
        elif self.sharded:
            dst = L.ZT_BUF_DATA | L.ZT_BUF_LIVE
        else:
            dst = L.ZT_BUF_DATA
        pcfg = PassCfg(
            src=L.ZT_BUF_DATA,
            dst=dst,
            ge_mode=ge_mode, ge_scale=ge_scale,
            momentum={"none": L.ZT_MOM_NONE, "stored_ema": L.ZT_MOM_STORED_EMA,
                      "seed_window": L.ZT_MOM_SEED_WINDOW}[mc.momentum_method],
            beta1=f32(mc.beta1), one_minus_beta1=f32(1 - mc.beta1),
            m_scale=f32_recip(f32((1.0 - mc.beta1 ** t) + mc.denom_eps)) if mc.momentum_method == "stored_ema" else 1.0,
            second_moment=mc.second_moment, beta2=f32(mc.beta2), one_minus_beta2=f32(1 - mc.beta2),
            bc2=f32(1.0 - mc.beta2 ** t), denom_eps=f32(mc.denom_eps),
            update=True, lr=lr32, wd=wd_code, wd_lam=wd_lam, wd_factor=f32(1.0 - wd_lam),
            ge_load=self.ge_onthefly)
        metrics = {
            "loss": mean_loss,
            "proj_grad": sum(pg) / Z,
            "proj_grad_clipped": sum(pgc) / Z,
            "clip_frac": clip_frac,
            "clip_tau": self.tau if math.isfinite(self.tau) else None,
            "lr": self.lr,
            **({"fit_rms": (sum(s * s for s in pgc) / Z) ** 0.5} if self.shaping else {}),
        }
        ranges = list(self.unit_ranges) if self.sharded and self.unit_ranges is not None else None
        return PassSpec(pcfg, streams, ranges), metrics

    # -- exact resume: the whole optimizer trajectory is seeds + scalars ---------------
    def state_dict(self) -> dict:
        sd = {"t": self._t, "seed_ctr": self._seed_ctr}
        if self._pg_hist is not None:
            sd["pg_hist"] = list(self._pg_hist)
        if self.cfg.mom.momentum_method == "seed_window":
            sd["seed_buf"] = [list(x) for x in self.seed_buf]
            sd["proj_buf"] = [list(x) for x in self.proj_buf]
        return sd

    def load_state_dict(self, sd: dict) -> None:
        self._t, self._seed_ctr = int(sd["t"]), int(sd["seed_ctr"])
        if self._pg_hist is not None:
            self._pg_hist.clear()
            self._pg_hist.extend(sd.get("pg_hist", []))
        if self.cfg.mom.momentum_method == "seed_window":
            self.seed_buf.clear(); self.proj_buf.clear()
            self.seed_buf.extend(list(x) for x in sd.get("seed_buf", []))
            self.proj_buf.extend(list(x) for x in sd.get("proj_buf", []))


def _aggregate_metrics(dicts: list[dict]) -> dict[str, float]:
    """Average each metric key over the collected score dicts (train_zo.py:228-239)."""
    total: dict[str, float] = {}
    count: dict[str, int] = {}
    for d in dicts:
        for k, v in d.items():
            if v is None:
                continue
            total[k] = total.get(k, 0.0) + (v.item() if isinstance(v, torch.Tensor) else float(v))
            count[k] = count.get(k, 0) + 1
    return {k: total[k] / count[k] for k in total}


# ── the optimizer ─────────────────────────────────────────────────────────────────

class ZOOptimizer:
    """``ZOOptimizer`` (zotitan/train_zo.py:242-606) on fused CUDA passes.

    ``process_group``: torch.distributed group to shard pairs over; default: the
    default group when it is initialised with more than one rank. ``sharded``: force the
    seed-sharded schedule on (it then needs an initialised process group) or off.
    ``shard_update`` (sharded schedule, trainable tensors of one dtype): each rank runs
    the step's last pass on 1/W of the elements and one in-place all-gather of the
    updated parameters completes them, instead of every rank regenerating every pair's
    noise over all elements. The trainable tensors are then re-homed into one flat
    buffer (the Parameters keep their identity; ``p.data`` becomes a view).
    ``noise_cache``: keep each pair's Gaussian field in an fp32 buffer (about 4 bytes per
    trainable parameter) between its +eps, -2eps and restore passes instead of
    regenerating it in each. The field is the same either way, so the step's results are
    bit-identical; the passes become cheaper because regenerating an element's noise
    (Philox4x32-10, log, cos, sqrt) costs far more than reading 4 bytes from HBM.
    None (default): on when the cache takes at most a quarter of the device's free
    memory; False keeps the noise in registers only.
    ``field_exchange`` (sharded update with the noise cache): each rank pushes the slices
    of its own pairs' fields into the field stores of the ranks that own those slices
    (copy engines over NVLink, overlapping the next pair's passes), and the last pass
    reads every stored field instead of regenerating it (zotitan_b200.exchange). The
    results are bit-identical either way. None (default): on with more than one rank,
    storing as many pairs as fit in half of the free device memory; a float sets that
    fraction and an int (not a bool) the number of stored pairs; True also runs it on a
    one-rank group; False regenerates every field. ``exchange_mode``: "copies" (copy-engine
    copies from the noise cache, overlapping the next pair's passes; the stored-pair count
    adapts step by step to the copy bandwidth) or "in_pass" (the +eps pass stores its
    field into the owners' stores over NVLink itself, when its plan takes the specialised
    kernel). ``push_order``: "rotate" (default; a pair's slices go to rank + 1, rank + 2,
    ... one after another, so every moment is a permutation of the ranks) or "all" (every
    peer at once, ``push_streams`` copy streams per peer). ``push_after``: "minus"
    (default; a pair's pushes start after its -2eps pass) or "plus" (after its +eps pass).
    ``lowrank_fused``: low_rank / polar directions of 2-D tensors recomputed on the tensor
    cores in each use (zt_lowrank_*) instead of materialised with the reference's ops."""

    def __init__(self, named_params: list, cfg: ZOConfig, score_fn, total_steps: int = 0, process_group=None,
                 sharded: bool | None = None, shard_update: bool = True, noise_cache: bool | None = None,
                 field_exchange: bool | float | None = None, exchange_mode: str = "copies",
                 lowrank_fused: bool = True, push_order: str = "rotate", push_streams: int = 1,
                 push_after: str = "minus"):
        if exchange_mode not in ("copies", "in_pass"):
            raise ValueError(f"exchange_mode must be 'copies' or 'in_pass', got {exchange_mode!r}")
        if push_after not in ("plus", "minus"):
            raise ValueError(f"push_after must be 'plus' or 'minus', got {push_after!r}")
        # copies: a pair's pushes start after its -2eps pass ("minus", default: they overlap the
        # next pair's instruction-bound passes instead of the memory-bound -2eps pass, 2.08 ->
        # 1.64 ms per -2eps pass and 142 -> 135 ms per microbench step at 4 ranks) or after
        # its +eps pass ("plus")
        self.push_after = push_after
        self.named_params = named_params
        self.params = [p.data for _, p in named_params]
        self.cfg = cfg
        self.score_fn = score_fn
        for n, p in zip([n for n, _ in named_params], self.params):
            if not p.is_cuda:
                raise ValueError(f"{n}: the zeroth-order passes run on CUDA tensors only (no CPU fallback)")
            if not p.is_contiguous():
                raise ValueError(f"{n}: trainable tensors must be contiguous")
        self.group = process_group
        rank, world = world_info(process_group)
        self.planner = StepPlanner(cfg, total_steps, rank, world, sharded=sharded)
        self.rank, self.world = rank, world
        pl = self.planner
        self.m = [torch.zeros_like(p) for p in self.params] if pl.needs_m else None
        self.v = [torch.zeros_like(p) for p in self.params] if pl.needs_v else None
        # theta_0 for anchored decay stays in HBM (the reference pins it in host
        # memory and copies it every step, train_zo.py:274, :406)
        self.theta_0 = [p.clone() for p in self.params] if pl.needs_anchor else None
        # low_rank / polar: 2-D tensors take materialised directions, 1-D ones the fused passes
        self.lr_idx = [i for i, p in enumerate(self.params) if p.dim() >= 2] if pl.materialized else []
        lr_set = set(self.lr_idx)
        # low_rank matrices, and polar ones in fp32 (the reference's QR has no 16-bit CUDA
        # kernel, so its polar branch runs only there): the direction is recomputed on the
        # tensor cores inside each use (zt_lowrank_*), never stored
        dist_kind = cfg.perturbation.distribution
        self.lr_fused = {i for i in self.lr_idx if lowrank_fused and K.lowrank_supported(self.params[i])
                         and (dist_kind == "low_rank" or self.params[i].dtype == torch.float32)}
        self.dense_idx = [i for i in range(len(self.params)) if i not in lr_set]
        # grad_est buffer of the on-the-fly accumulation (same size as the reference's
        # zeros_like grad_est for z_batch > 1; dense tensors only)
        self.ge = ([torch.zeros_like(self.params[i]) for i in self.dense_idx] if pl.ge_onthefly else None)
        dev = self.params[0].device
        self.vals_buf = torch.zeros(2 * max(1, cfg.z_batch), dtype=torch.float32, device=dev)
        self.layout = None
        one_dtype = len({p.dtype for p in self.params}) == 1
        if pl.sharded and shard_update and one_dtype and not pl.materialized:
            from .flat import FlatLayout
            self.layout = FlatLayout([p.numel() for p in self.params], world)
            dt = self.params[0].dtype
            shapes = [p.shape for p in self.params]
            self.flat_live, live = self.layout.alloc(dt, dev, like=self.params)
            for (_, p), view in zip(named_params, live):
                p.data = view                      # the model now reads the flat live copy
            self.params = live
            self.flat_master, self.master = self.layout.alloc(dt, dev, like=self.params)
            flat_view = lambda: self.layout.views(torch.zeros(self.layout.numel, dtype=dt, device=dev), shapes)  # noqa: E731
            self.m = flat_view() if pl.needs_m else None
            self.v = flat_view() if pl.needs_v else None
            self.theta_0 = self.layout.views(self.flat_master.clone(), shapes) if pl.needs_anchor else None
            self.table = ParamTable(self.master, live=self.params, m=self.m, v=self.v, anchor=self.theta_0)
            pl.unit_ranges = self.layout.shard_ranges(rank)
        elif pl.sharded and not pl.materialized:
            # model reads `live` (the parameters' own storage); `master` stays unperturbed
            self.master = [p.clone() for p in self.params]
            self.table = ParamTable(self.master, live=self.params, m=self.m, v=self.v, anchor=self.theta_0)
        elif pl.materialized:
            # sharded: the model reads `live` (the parameters); the 1-D tensors' master and the
            # 2-D tensors' master take the last pass's replay and the update
            self.master = [p.clone() for p in self.params] if pl.sharded else None
            own = self.master if pl.sharded else self.params
            n = len(self.params)
            sub = lambda lst, idx: None if lst is None else [lst[i] for i in idx]  # noqa: E731
            self.table = (ParamTable(sub(own, self.dense_idx), n_params=n, indices=self.dense_idx,
                                     live=sub(self.params, self.dense_idx) if pl.sharded else None,
                                     m=sub(self.m, self.dense_idx), v=sub(self.v, self.dense_idx),
                                     anchor=sub(self.theta_0, self.dense_idx), ge=self.ge)
                          if self.dense_idx else None)
            self.lr_ge = [torch.zeros_like(self.params[i]) for i in self.lr_idx]
            self.lr_table = (ParamTable(sub(own, self.lr_idx), n_params=n, indices=self.lr_idx,
                                        m=sub(self.m, self.lr_idx), v=sub(self.v, self.lr_idx),
                                        anchor=sub(self.theta_0, self.lr_idx), ge=self.lr_ge)
                             if self.lr_idx else None)
        else:
            self.master = None
            self.table = ParamTable(self.params, m=self.m, v=self.v, anchor=self.theta_0, ge=self.ge)
        if noise_cache is None and self.table is not None:
            free, _ = torch.cuda.mem_get_info(self.table.device)
            noise_cache = 4 * int(self.table.plan.n_units) * L.ZT_UNIT_ELEMS <= free // 4
        self.zcache = self.table.noise_cache() if noise_cache and self.table is not None else None
        pl.noise_cache = self.zcache is not None
        self._zc = self.zcache                  # the noise cache the next pass uses
        self.exchange = None
        if (self.layout is not None and self.zcache is not None and field_exchange is not False
                and (world > 1 or field_exchange is not None)):
            from .exchange import FieldExchange, slot_bytes
            # the +eps pass pushes its field itself when the plan takes the specialised kernel
            props = int(self.table.plan.props)
            cache_bytes = 4 * int(self.table.plan.n_units) * L.ZT_UNIT_ELEMS
            in_pass = bool(props & L.ZT_PLAN_VEC8) and bool(props & (L.ZT_PLAN_ALL_F32 | L.ZT_PLAN_ALL_BF16
                                                                     | L.ZT_PLAN_ALL_F16))
            in_pass = in_pass and world <= L.ZT_MAX_PUSH_RANKS and exchange_mode == "in_pass"
            # with copies, caches rotate between a rank's pairs, so a pair's pushes overlap the
            # next pairs' passes: three from 4 ranks on when memory allows (157 against 164 ms
            # per step with two at 4 ranks), two at 2 ranks, whose pushes to one peer already
            # hide under the passes (3.39 against 3.29 ZO steps/s with three)
            self.zcaches = [self.zcache]
            if not in_pass:
                n_caches = 3 if world >= 4 and 4 * cache_bytes <= torch.cuda.mem_get_info(dev)[0] else 2
                self.zcaches += [self.table.noise_cache() for _ in range(n_caches - 1)]
            if type(field_exchange) is int:
                budget = field_exchange * slot_bytes(self.layout)
            else:
                frac = field_exchange if isinstance(field_exchange, float) else 0.5
                budget = int(frac * torch.cuda.mem_get_info(dev)[0])
            self.exchange = FieldExchange(self.layout, int(self.table.plan.n_units), rank, world, cfg.z_batch, dev,
                                          budget, group=process_group, in_pass=in_pass, push_order=push_order, push_streams=push_streams)
            pl.field_slots = self.exchange.active
        self._metric_keys = None

    def close(self) -> None:
        """Release the field exchange's peer mappings (collective over the process group
        when the exchange is on); call on every rank before dropping the optimizer."""
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    # properties mirroring the reference's attributes
    @property
    def _t(self):
        return self.planner._t

    @property
    def _seed_ctr(self):
        return self.planner._seed_ctr

    @_seed_ctr.setter
    def _seed_ctr(self, v):
        self.planner._seed_ctr = int(v)

    def _run(self, spec: PassSpec) -> None:
        if spec.cfg.dev_pair is not None:
            spec.cfg.dev_vals = self.vals_buf.data_ptr() + 8 * spec.cfg.dev_pair
        if self._zc is not None and any(s.z_load or s.z_store for s in spec.streams):
            spec.cfg.zcache = self._zc.data_ptr()
        if self.table is not None:
            self.table.run(spec.cfg, spec.streams)

    # -- low_rank / polar directions of the 2-D tensors (zotitan/train_zo.py:295-322) ------
    def _lowrank_z(self, seed: int) -> list:
        """The reference's _sample_z for the 2-D tensors, one entry per tensor of lr_idx: for
        the fused ones the prepared factors (K.LowRankFactors, z never stored), for the
        others the materialised direction: P [m, r] and Psi [r, n] from the noise source
        (keys of positions i + 2n and i + n), cast to the parameter dtype,
        polar-orthogonalised for "polar", z = P @ Psi scaled to ||z||_F = sqrt(numel)."""
        return [self._lowrank_one(i, [seed]) if i in self.lr_fused else self._lowrank_dense(i, seed)
                for i in self.lr_idx]

    def _lowrank_one(self, i: int, seeds: list) -> "K.LowRankFactors":
        p = self.params[i]
        n = len(self.params)
        r = min(self.cfg.perturbation.rank, p.shape[0])
        if self.cfg.perturbation.distribution == "polar":   # factors through QR / Newton-Schulz
            Ps, Psis = zip(*(self._polar_factors(i, sd) for sd in seeds))
            return K.LowRankFactors.from_factors(p.shape, list(Ps), list(Psis), p.dtype)
        return K.LowRankFactors(p.shape, r, p.dtype, [param_key(sd, n, i + 2 * n) for sd in seeds],
                                [param_key(sd, n, i + n) for sd in seeds], p.device)

    def _polar_factors(self, i: int, seed: int):
        """P (QR of the noise factor) and Psi (Newton-Schulz polar factor) of the reference's
        polar branch (zotitan/train_zo.py:307-317), before their product."""
        pc = self.cfg.perturbation
        n = len(self.params)
        p = self.params[i]
        m, r = p.shape[0], min(pc.rank, p.shape[0])
        P = randn(param_key(seed, n, i + 2 * n), m * r, p.device).view(m, r).to(p.dtype)
        P, _ = torch.linalg.qr(P)
        Psi = randn(param_key(seed, n, i + n), r * p.shape[1], p.device).view(r, p.shape[1]).to(p.dtype)
        return P, zeropower_via_newtonschulz(Psi)

    def _lowrank_dense(self, i: int, seed: int) -> torch.Tensor:
        pc = self.cfg.perturbation
        n = len(self.params)
        p = self.params[i]
        m, r = p.shape[0], min(pc.rank, p.shape[0])
        P = randn(param_key(seed, n, i + 2 * n), m * r, p.device).view(m, r).to(p.dtype)
        if pc.distribution == "polar":
            P, _ = torch.linalg.qr(P)
        Psi = randn(param_key(seed, n, i + n), r * p.shape[1], p.device).view(r, p.shape[1]).to(p.dtype)
        if pc.distribution == "polar":
            Psi = zeropower_via_newtonschulz(Psi)
        z = P @ Psi
        return z * (p.numel() ** 0.5 / (z.norm() + 1e-7))

    def _lr_apply(self, z: list, scale: float, target=None) -> None:
        """_apply_z (:350-351) on the 2-D tensors (of `target`, default the parameters)."""
        if not self.lr_idx:
            return
        tgt = self.params if target is None else target
        dense = [(tgt[i], zz) for i, zz in zip(self.lr_idx, z) if i not in self.lr_fused]
        if dense:
            torch._foreach_add_([t for t, _ in dense], [zz for _, zz in dense], alpha=scale)
        for i, zz in zip(self.lr_idx, z):
            if i in self.lr_fused:
                zz.apply(src=tgt[i], dst=tgt[i], alphas=(scale,))

    def _lr_plus_live(self, z: list, scale: float) -> None:
        """Sharded: live = master + scale * z on the 2-D tensors, rounded once (what the
        fused +eps pass does for the others)."""
        for i, zz in zip(self.lr_idx, z):
            if i in self.lr_fused:
                zz.apply(src=self.master[i], dst=self.params[i], alphas=(scale,))
            else:
                torch.add(self.master[i], zz, alpha=scale, out=self.params[i])

    _LR_CHUNK_BYTES = 2 << 30   # factor buffers of one launch over many seeds

    def _lr_seed_chunks(self, seeds: list, i: int) -> list:
        """Seeds of one launch for tensor i: at most ZT_LOWRANK_MAX_STREAMS, and at most about
        2 GB of factor buffers ((m + n) x the padded K per seed, 9 r for fp32)."""
        p = self.params[i]
        r = min(self.cfg.perturbation.rank, p.shape[0])
        width = 9 * r if p.dtype == torch.float32 else r
        per_seed = (p.shape[0] + p.shape[1]) * 64 * ((width + 63) // 64) * 2
        M = max(1, min(L.ZT_LOWRANK_MAX_STREAMS, self._LR_CHUNK_BYTES // per_seed))
        return [seeds[c:c + M] for c in range(0, len(seeds), M)]

    def _lr_replay_master(self) -> None:
        """Sharded: every pair's +eps / -2eps / +eps rounding chain on the 2-D tensors'
        master, in pair order, as the single-GPU parameters went through them (fused
        tensors: every pair of a chunk in one launch per tensor)."""
        eps = self.cfg.eps
        seeds = self.planner.seeds
        for i in self.lr_idx:
            if i in self.lr_fused:
                for chunk in self._lr_seed_chunks(seeds, i):
                    self._lowrank_one(i, chunk).apply(src=self.master[i], dst=self.master[i],
                                                      alphas=(eps, -2 * eps, eps))
        dense = [i for i in self.lr_idx if i not in self.lr_fused]
        if dense:
            tgt = [self.master[i] for i in dense]
            for seed in seeds:
                zs = [self._lowrank_dense(i, seed) for i in dense]
                for a in (eps, -2 * eps, eps):
                    torch._foreach_add_(tgt, zs, alpha=a)

    def _lr_finish(self, spec: PassSpec) -> None:
        """grad_est of the 2-D tensors from the regenerated directions with this step's pair
        coefficients (:550-556, :575-577), then the same optimizer stages as the fused pass
        (ge read from the buffer; no noise streams)."""
        if not self.lr_idx:
            return
        import dataclasses
        pl = self.planner
        ge_mode, coefs, _ = pl.last_ge
        pos = {i: t for t, i in enumerate(self.lr_idx)}
        dense = [i for i in self.lr_idx if i not in self.lr_fused]
        dge = [self.lr_ge[pos[i]] for i in dense]
        if ge_mode == L.ZT_GE_PRODUCT:
            if dense:
                zs = [self._lowrank_dense(i, pl.seeds[0]) for i in dense]
                for g, r in zip(dge, torch._foreach_mul(zs, coefs[0])):
                    g.copy_(r)
            for i in self.lr_idx:
                if i in self.lr_fused:
                    self._lowrank_one(i, pl.seeds[:1]).apply(ge=self.lr_ge[pos[i]], coefs=[coefs[0]], ge_init=True)
        elif ge_mode == L.ZT_GE_ACCUM:
            if dense:
                torch._foreach_zero_(dge)
                for j, seed in enumerate(pl.seeds):
                    torch._foreach_add_(dge, [self._lowrank_dense(i, seed) for i in dense], alpha=coefs[j])
            for i in self.lr_idx:
                if i in self.lr_fused:
                    for c, chunk in enumerate(self._lr_seed_chunks(list(range(len(pl.seeds))), i)):
                        self._lowrank_one(i, [pl.seeds[j] for j in chunk]).apply(
                            ge=self.lr_ge[pos[i]], coefs=[coefs[j] for j in chunk], ge_init=c == 0)
        # the 2-D tensors' table has no live copy: the sharded schedule copies master -> live after
        cfg = dataclasses.replace(spec.cfg, ge_mode=L.ZT_GE_ACCUM if ge_mode != L.ZT_GE_NONE else L.ZT_GE_NONE,
                                  ge_load=ge_mode != L.ZT_GE_NONE, ge_store=False, dev_pair=None, dev_vals=0,
                                  src=L.ZT_BUF_DATA, dst=L.ZT_BUF_DATA)
        self.lr_table.run(cfg, [])

    def _acquire(self, model, batch):
        s = self.score_fn(model, batch)
        value = s.value if isinstance(s.value, torch.Tensor) else torch.tensor(float(s.value))
        return value, s.metrics

    def step(self, model, batches: list) -> dict:
        pl = self.planner
        Z = self.cfg.z_batch
        if len(batches) != Z:
            raise ValueError(f"step expects z_batch={Z} batches (entries of other ranks' pairs may be None)")
        local = pl.start()
        dev = self.params[0].device
        vals_t, metric_dicts = [], []
        prev = None
        eps = self.cfg.eps
        ex = self.exchange
        if ex is not None:
            ex.begin_step()
            pl.field_slots = ex.active      # the stored pairs of this step (pushes and last pass)
        with torch.inference_mode():
            for k, j in enumerate(local):
                z = self._lowrank_z(pl.seeds[j]) if self.lr_idx else None
                if ex is not None:
                    self._zc = self.zcaches[k % len(self.zcaches)]
                    ex.before_cache_write(self._zc)
                spec = pl.plus_pass(j, prev)
                timed = ex is not None and ex.adaptive and k == 0
                if timed:
                    t0 = torch.cuda.Event(enable_timing=True)
                    t0.record()
                if ex is not None:
                    ex.set_push(spec.cfg, j)
                self._run(spec)
                if timed:
                    t1 = torch.cuda.Event(enable_timing=True)
                    t1.record()
                    ex.note_plus(t0, t1)
                if ex is not None and self.push_after == "plus":
                    ex.push(j, self._zc)
                if pl.sharded:
                    if z is not None:
                        self._lr_plus_live(z, eps)
                else:
                    self._lr_apply(z, eps)
                vp, mp = self._acquire(model, batches[j])
                self._run(pl.minus_pass(j))
                if ex is not None and self.push_after == "minus":   # the -2eps pass only reads the cache
                    ex.push(j, self._zc)
                self._lr_apply(z, -2 * eps)
                vn, mn = self._acquire(model, batches[j])
                if not pl.sharded:
                    self._lr_apply(z, eps)
                del z
                prev = j
                vp = vp.detach().float().reshape(()).to(dev)
                vn = vn.detach().float().reshape(()).to(dev)
                if not pl.sharded:   # read by the next restore pass (device coefficient)
                    self.vals_buf[2 * j].copy_(vp)
                    self.vals_buf[2 * j + 1].copy_(vn)
                vals_t += [vp, vn]
                metric_dicts += [mp, mn]
        if ex is not None:
            ex.local_done()
            ex.finish_pushes()    # every push lands before the all-gather that ends the pair loop
        if pl.sharded:
            vals, metrics_avg = self._gather(vals_t, metric_dicts, local)
        else:
            vals = self.vals_buf[: 2 * Z].tolist()      # the step's one host sync (:564-565)
            metrics_avg = _aggregate_metrics(metric_dicts)
        spec, metrics = pl.finish(vals)
        with torch.inference_mode():
            if pl.sharded and self.lr_idx:
                self._lr_replay_master()
            self._lr_finish(spec)
            if pl.sharded and self.lr_idx:
                for i in self.lr_idx:
                    self.params[i].copy_(self.master[i])
            if self.layout is not None:
                # the last pass chunk by chunk on this rank's share; each chunk's in-place
                # all-gather starts when its pass is done and overlaps the next chunk's pass
                import torch.distributed as dist
                works = []
                for k, (ub, ue) in enumerate(spec.unit_ranges):
                    spec.cfg.unit_begin, spec.cfg.unit_end = ub, ue
                    if ex is not None:
                        spec.cfg.zfield, spec.cfg.zfield_stride = ex.chunk_field(k)
                    self._run(spec)
                    works.append(dist.all_gather_into_tensor(
                        self.layout.chunk(self.flat_master, k),
                        self.layout.shard_chunk(self.flat_master, self.rank, k), group=self.group, async_op=True))
                for k, w in enumerate(works):
                    w.wait()
                    self.layout.chunk(self.flat_live, k).copy_(self.layout.chunk(self.flat_master, k))
            else:
                self._run(spec)
        metrics.update(metrics_avg)
        return metrics

    def _gather(self, vals_t, metric_dicts, local):
        """All-gather pair values and metric scalars; returns (vals in pair order, averaged metrics)."""
        import torch.distributed as dist
        if self._metric_keys is None:
            mine = sorted({k for d in metric_dicts for k, v in d.items() if v is not None})
            allk = [None] * self.world
            dist.all_gather_object(allk, mine, group=self.group)
            self._metric_keys = sorted({k for ks in allk for k in ks})
        keys = self._metric_keys
        dev = self.params[0].device
        ex = self.exchange
        n_ex = 3 if ex is not None and ex.adaptive else 0   # the field exchange's timings ride along
        C = 2 + 2 * len(keys) + n_ex
        rows = torch.full((len(local), C), float("nan"), dtype=torch.float32, device=dev)
        if n_ex and len(local):
            rows[:, C - n_ex:] = torch.tensor(ex.stats(), dtype=torch.float32)
        for r in range(len(local)):
            rows[r, 0] = vals_t[2 * r]
            rows[r, 1] = vals_t[2 * r + 1]
            for s in range(2):
                d = metric_dicts[2 * r + s]
                for k_i, k in enumerate(keys):
                    v = d.get(k)
                    if v is not None:
                        rows[r, 2 + 2 * k_i + s] = v.detach().float() if isinstance(v, torch.Tensor) else float(v)
        allrows = gather_pair_values(rows, self.cfg.z_batch, self.rank, self.world, self.group).cpu().tolist()
        vals = [x for row in allrows for x in row[:2]]
        if n_ex:   # the same maxima on every rank, so every rank takes the same stored-pair count
            mx = [max((row[C - n_ex + i] for row in allrows if not math.isnan(row[C - n_ex + i])), default=0.0)
                  for i in range(n_ex)]
            ex.adapt(*mx, local_pairs=-(-self.cfg.z_batch // self.world))
        metrics = {}
        for k_i, k in enumerate(keys):
            xs = [x for row in allrows for x in row[2 + 2 * k_i: 4 + 2 * k_i] if not math.isnan(x)]
            if xs:
                metrics[k] = sum(xs) / len(xs)
        return vals, metrics

    # exact resume (the reference saves no optimizer state, train_zo.py:671-673)
    def state_dict(self) -> dict:
        sd = {"planner": self.planner.state_dict()}
        for name in ("m", "v", "theta_0"):
            lst = getattr(self, name)
            if lst is not None:
                sd[name] = [t.detach().cpu() for t in lst]
        return sd

    def load_state_dict(self, sd: dict) -> None:
        self.planner.load_state_dict(sd["planner"])
        for name in ("m", "v", "theta_0"):
            lst = getattr(self, name)
            if lst is not None and name in sd:
                for dst, src in zip(lst, sd[name]):
                    dst.copy_(src)
        if self.master is not None:
            for m, p in zip(self.master, self.params):
                m.copy_(p)


def train_zo(model, tokenizer, total_steps, seed, merge_fn, logger, cfg: ZOConfig | None = None, objective=None,
             profiling_cfg=None):
    """Zeroth-order training loop (zotitan/train_zo.py:609-675). Perturbs only
    params with requires_grad=True; calls merge_fn(model) after each step.
    ``profiling_cfg`` is accepted for signature parity and ignored (torch.profiler
    traces are not part of this path; kernels are profiled with ncu)."""
    if cfg is None:
        cfg = ZOConfig()
    if objective is None:
        raise ValueError("train_zo needs an objective (dataset objectives are not bundled)")
    named_params = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    n_params = sum(p.numel() for _, p in named_params)
    device = next(model.parameters()).device
    move_fn = None if getattr(objective, "flat_batches", True) else objective.to_device
    loader = PrefetchLoader(objective.train_batches(tokenizer, seed, cfg.batch_size), device, move_fn=move_fn)
    run_dir = os.environ.get("MLSWEEP_RUN_DIR", ".")
    opt = ZOOptimizer(named_params, cfg, objective.score, total_steps=total_steps)
    print(f"  ZO train: {total_steps:,} steps | {n_params:,} params")
    model.eval()
    show_lr = not wsd_is_constant(cfg.base.lr_wsd)
    overfit = cfg.base.overfit_first_batch
    fixed_batches = None
    for step in range(total_steps):
        if fixed_batches is not None:
            batches = fixed_batches
        elif cfg.shared_batch or overfit:
            one = get_batches(loader, 1)
            batches = one * cfg.z_batch if one is not None else None
        else:
            batches = get_batches(loader, cfg.z_batch)
        if batches is None:
            print("Dataloader exhausted, ending training.")
            break
        if overfit:
            fixed_batches = batches
        t0 = time.perf_counter()
        metrics = opt.step(model, batches)
        if merge_fn is not None:
            merge_fn(model)
        metrics["step_time"] = time.perf_counter() - t0
        if logger is not None:
            logger.log(metrics)
        lr_s = f" lr {metrics['lr']:.2e}" if show_lr else ""
        print(f"  step {step + 1}/{total_steps} loss {metrics['loss']:.4f} pg {metrics['proj_grad']:+.4f}{lr_s}")
        if (step + 1) % cfg.base.ckpt_every == 0:
            ckpt = os.path.join(run_dir, "checkpoint")
            if hasattr(model, "save_pretrained"):
                model.save_pretrained(ckpt)
            torch.save(opt.state_dict(), os.path.join(run_dir, "zo_optimizer.pt"))
            if logger is not None and hasattr(logger, "sync"):
                logger.sync()
    return model
