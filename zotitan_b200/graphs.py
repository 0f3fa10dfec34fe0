"""CUDA-graph replay of a score function (the forwards of a zeroth-order step).

A step evaluates the model 2Z times on batches of one shape, with the parameters
changed in place between evaluations by the fused passes (same storage, new values).
In eager mode each forward is thousands of kernel launches issued from Python, and for
a small model the host falls behind the GPU. ``GraphedScore`` captures
``score_fn(model, batch)`` once per batch shape into a CUDA graph and replays it: the
batch is copied into the graph's input buffers, the graph reads the current parameters
from their unchanged addresses, and the outputs are copied out so later replays do not
overwrite them.

Under stream capture transformers builds an explicit causal mask (its check for the
`is_causal` shortcut treats capture as tracing), which would move SDPA off its flash
path. For batches without an ``attention_mask`` entry every sequence is full and the
mask is purely causal, so the capture runs under ``llama_fused.assume_causal()``: the
fused attention forward then drops the mask and SDPA takes ``is_causal``. This needs
``fuse_llama(model)``; models that do not use it capture the mask as built.
"""
from __future__ import annotations

import contextlib

import torch

from . import llama_fused
from .objective import Score


def _key(model, batch: dict):
    return (id(model),) + tuple(sorted((k, tuple(v.shape), v.dtype, str(v.device))
                                       for k, v in batch.items() if isinstance(v, torch.Tensor)))


class GraphedScore:
    """score_fn(model, batch) -> Score, replayed from a CUDA graph per batch shape.

    The graph holds the model's parameter addresses: use it only while the model's
    parameters keep their storage (the zeroth-order passes update them in place).
    ``warmup`` eager calls on a side stream precede each capture."""

    def __init__(self, score_fn, warmup: int = 2):
        self.score_fn = score_fn
        self.warmup = warmup
        self._graphs: dict = {}

    def _capture(self, model, batch: dict):
        static = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in batch.items()}
        causal = "attention_mask" not in batch
        ctx = llama_fused.assume_causal() if causal else contextlib.nullcontext()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with ctx:
            with torch.cuda.stream(side):
                for _ in range(self.warmup):
                    self.score_fn(model, static)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = self.score_fn(model, static)
        value = out.value if isinstance(out.value, torch.Tensor) else torch.tensor(float(out.value))
        return static, graph, value, dict(out.metrics)

    def __call__(self, model, batch: dict) -> Score:
        key = _key(model, batch)
        entry = self._graphs.get(key)
        if entry is None:
            entry = self._graphs[key] = self._capture(model, batch)
        static, graph, value, metrics = entry
        for k, v in batch.items():
            if isinstance(v, torch.Tensor):
                static[k].copy_(v, non_blocking=True)
        graph.replay()
        return Score(value.clone(), {k: (m.clone() if isinstance(m, torch.Tensor) else m) for k, m in metrics.items()})

    def reset(self) -> None:
        """Drop every captured graph (after the model's parameters were re-homed)."""
        self._graphs.clear()
