"""Flat parameter layout for the sharded update.

Tensors of one dtype are laid back to back in one buffer, each padded to a whole
number of ZT_UNIT_ELEMS-element work units, and the unit count is padded to a
multiple of the world size. Unit u then covers elements [u*2048, (u+1)*2048) of the
buffer, and rank r's share of the step's last pass, units
[r*U/W, (r+1)*U/W), is one contiguous slice: after the pass one in-place all-gather
of that slice completes every rank's copy.
"""
from __future__ import annotations

import torch

from . import _lib as L


class FlatLayout:
    def __init__(self, numels: list[int], world: int):
        u = L.ZT_UNIT_ELEMS
        self.offsets = []
        units = 0
        for n in numels:
            self.offsets.append(units * u)
            units += (n + u - 1) // u
        self.units = units
        self.world = world
        self.padded_units = ((units + world - 1) // world) * world
        self.numel = self.padded_units * u
        self.numels = list(numels)

    def shard_units(self, rank: int) -> tuple[int, int]:
        per = self.padded_units // self.world
        return rank * per, (rank + 1) * per

    def shard_slice(self, flat: torch.Tensor, rank: int) -> torch.Tensor:
        ub, ue = self.shard_units(rank)
        return flat[ub * L.ZT_UNIT_ELEMS: ue * L.ZT_UNIT_ELEMS]

    def views(self, flat: torch.Tensor, shapes) -> list[torch.Tensor]:
        return [flat[o: o + n].view(shape) for o, n, shape in zip(self.offsets, self.numels, shapes)]

    def alloc(self, dtype, device, like: list[torch.Tensor] | None = None) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """A zeroed flat buffer and its per-tensor views (filled from `like` if given)."""
        flat = torch.zeros(self.numel, dtype=dtype, device=device)
        shapes = [t.shape for t in like] if like is not None else [(n,) for n in self.numels]
        views = self.views(flat, shapes)
        if like is not None:
            for v, t in zip(views, like):
                v.copy_(t)
        return flat, views
