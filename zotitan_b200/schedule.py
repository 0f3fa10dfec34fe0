"""LR schedule and base training config, mirroring zotitan/schedule.py:6-63.

``maybe_torchcompile`` is intentionally absent: nothing on this path is compiled
(the hot path is the CUDA library)."""
from __future__ import annotations

import math
from dataclasses import dataclass, field


@dataclass
class WSDConfig:
    warmup_frac: float = 0.0
    """Fraction of total_steps for linear warmup (lo -> hi)."""

    decay_frac: float = 0.0
    """Fraction of total_steps for cosine decay (hi -> lo)."""


@dataclass
class BaseTrainConfig:
    lr: float = 2e-5
    """Peak learning rate."""

    lr_wsd: WSDConfig = field(default_factory=WSDConfig)
    """WSD schedule for the learning rate. Default (decay_frac=0) = constant at lr."""

    grad_clip: float = 1.0
    """Gradient clipping threshold (first-order trainer only; kept for flag parity)."""

    ckpt_every: int = 2_000
    """Save a checkpoint every N steps."""

    overfit_first_batch: bool = False
    """Debug: draw one batch up front and reuse it every step."""


def wsd_is_constant(cfg: WSDConfig) -> bool:
    """True when the schedule never changes the LR (zotitan/schedule.py:46-48)."""
    return cfg.warmup_frac == 0.0 and cfg.decay_frac == 0.0


def wsd_value(step: int, total_steps: int, lo: float, hi: float, cfg: WSDConfig) -> float:
    """Warmup-Stable-Decay schedule value at `step` (zotitan/schedule.py:51-63)."""
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
