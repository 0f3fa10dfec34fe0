"""The objective contract the zeroth-order step calls (the scorer side of the path).

Mirrors zotitan/objective.py: ``Score`` (:36-39), the ``Objective`` protocol
(:154-163), ``CrossEntropyCriterion`` (:59-95), ``RubricObjective`` (:186-217) and the
``register_objective`` registry (:170-181). Cross-entropy comes from ``losses``: the
CUDA fused scorer by default (the reference's default is its fused Liger path), or the
reference's torch path with fused=False.
Dataset-backed objectives need network datasets and are out of scope; a
synthetic-token objective stands in for them.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, Protocol

import torch

from .data import synthetic_token_batches
from .losses import get_xentropy, torch_xentropy  # noqa: F401  (torch_xentropy re-exported)

Metric = torch.Tensor | float


@dataclass
class Score:
    value: torch.Tensor | float
    metrics: dict[str, Metric]


class Objective(Protocol):
    name: str
    differentiable: bool
    flat_batches: bool
    def train_batches(self, tokenizer, seed: int, batch_size: int) -> Iterator: ...
    def to_device(self, batch, device) -> object: ...
    def score(self, model, batch) -> Score: ...


OBJECTIVES: dict[str, type] = {}


def register_objective(name: str):
    def deco(cls):
        if name in OBJECTIVES:
            raise ValueError(f"objective {name!r} is already registered to {OBJECTIVES[name]!r}")
        cls.name = name
        OBJECTIVES[name] = cls
        return cls
    return deco


class CrossEntropyCriterion:
    """value = ce + z_loss; metrics {"ce", "z_loss", "acc"} (zotitan/objective.py:59-95).
    fused=True (the reference's default) scores with the CUDA cross-entropy
    (losses.fused_xentropy); fused=False with the reference's torch path."""
    name = "ce"
    differentiable = True

    def __init__(self, compile_enabled: bool = False, compile_mode: str | None = None, z_loss_weight: float = 0.0,
                 fused: bool = True, compute_accuracy: bool = True, fn=None):
        self.compile_enabled = compile_enabled
        self.compile_mode = compile_mode
        self.z_loss_weight = z_loss_weight
        self.fused = fused
        self.compute_accuracy = compute_accuracy
        self.fn = fn or get_xentropy(fused=fused, compile_mode=compile_mode)

    def __call__(self, model, batch):
        loss, z_loss, extra = self.fn(model, batch, self.z_loss_weight, self.compute_accuracy)
        value = loss if z_loss is None else loss + z_loss
        metrics: dict[str, Metric] = {"ce": loss}
        if z_loss is not None:
            metrics["z_loss"] = z_loss
        if extra:
            metrics.update(extra)
        return value, metrics


class RubricObjective:
    """A weighted list of criteria; score = sum of weight * value (zotitan/objective.py:186-217)."""
    flat_batches = True

    def __init__(self, criteria):
        self.criteria = criteria
        self.differentiable = all(c.differentiable for c, _ in criteria)
        self._prefix = len(criteria) > 1

    def dataset_sources(self):
        return []

    def to_device(self, batch, device):
        return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in batch.items()}

    def score(self, model, batch) -> Score:
        total = None
        metrics: dict[str, Metric] = {}
        for crit, w in self.criteria:
            v, m = crit(model, batch)
            contrib = v if w == 1.0 else v * w
            total = contrib if total is None else total + contrib
            for k, mv in m.items():
                metrics[f"{crit.name}/{k}" if self._prefix else k] = mv
        assert total is not None, "objective has no criteria"
        return Score(total, metrics)


@register_objective("synthetic")
class SyntheticTokensObjective(RubricObjective):
    """Next-token CE (+ z-loss) on uniform random token ids of a fixed length."""

    def __init__(self, vocab_size: int, seq_len: int, z_loss_weight: float = 0.0, fused: bool = True):
        super().__init__([(CrossEntropyCriterion(z_loss_weight=z_loss_weight, fused=fused), 1.0)])
        self.vocab_size, self.seq_len = vocab_size, seq_len

    def train_batches(self, tokenizer, seed: int, batch_size: int):
        return synthetic_token_batches(self.vocab_size, batch_size, self.seq_len, seed)
