"""Flat parameter layout for the sharded update.

Tensors of one dtype are laid back to back in one buffer, each padded to a whole
number of ZT_UNIT_ELEMS-element work units. The unit count is padded to a multiple of
world * chunks, and the buffer is cut into `chunks` equal chunks of world * C units:
in chunk k, rank r owns units [k*W*C + r*C, k*W*C + (r+1)*C). Unit u covers elements
[u*2048, (u+1)*2048) of the buffer. The step's last pass then runs chunk by chunk on
each rank's share, and the in-place all-gather of chunk k (contiguous, rank-major) can
cross NVLink while the pass works on chunk k+1.
"""
from __future__ import annotations

import torch

from . import _lib as L


class FlatLayout:
    def __init__(self, numels: list[int], world: int, chunks: int = 4):
        u = L.ZT_UNIT_ELEMS
        self.offsets = []
        units = 0
        for n in numels:
            self.offsets.append(units * u)
            units += (n + u - 1) // u
        self.units = units
        self.world = world
        self.chunks = chunks
        grain = world * chunks
        self.padded_units = ((units + grain - 1) // grain) * grain
        self.per = self.padded_units // grain          # units of one rank in one chunk
        self.numel = self.padded_units * u
        self.numels = list(numels)

    def shard_ranges(self, rank: int) -> list[tuple[int, int]]:
        """This rank's unit ranges, one per chunk, in chunk order."""
        w, c = self.world, self.per
        return [(k * w * c + rank * c, k * w * c + (rank + 1) * c) for k in range(self.chunks)]

    def chunk(self, flat: torch.Tensor, k: int) -> torch.Tensor:
        """Chunk k of a flat buffer (every rank's share of it, rank-major)."""
        n = self.world * self.per * L.ZT_UNIT_ELEMS
        return flat[k * n: (k + 1) * n]

    def shard_chunk(self, flat: torch.Tensor, rank: int, k: int) -> torch.Tensor:
        """This rank's share of chunk k (a slice of chunk(flat, k): in-place all-gather)."""
        ub, ue = self.shard_ranges(rank)[k]
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
