"""Geometry of the flat parameter layout of the sharded update (zotitan_b200.flat), on CPU.

Every work unit belongs to exactly one rank's range; each chunk is one contiguous slice
holding every rank's share in rank order, so a rank's share of a chunk is the slice that
an in-place all-gather of that chunk expects from it; the tensors' views sit at
unit-aligned offsets and never overlap.
"""
import pytest
import torch

from zotitan_b200 import _lib as L
from zotitan_b200.flat import FlatLayout

U = L.ZT_UNIT_ELEMS


@pytest.mark.parametrize("world,chunks", [(1, 4), (2, 4), (3, 3), (8, 4), (8, 1)])
@pytest.mark.parametrize("numels", [[1], [7, 2048, 2049, 5000], [100003, 1, 4096 * 3 + 5] * 3])
def test_ranges_cover_every_unit_once(numels, world, chunks):
    lay = FlatLayout(numels, world, chunks=chunks)
    assert lay.padded_units % (world * chunks) == 0 and lay.padded_units >= lay.units
    seen = []
    for r in range(world):
        ranges = lay.shard_ranges(r)
        assert len(ranges) == chunks
        for ub, ue in ranges:
            assert ue - ub == lay.per
            seen.extend(range(ub, ue))
    assert sorted(seen) == list(range(lay.padded_units))


@pytest.mark.parametrize("world,chunks", [(2, 4), (4, 3)])
def test_chunk_slices_match_an_in_place_all_gather(world, chunks):
    lay = FlatLayout([3 * U + 11, 17, 5 * U], world, chunks=chunks)
    flat = torch.arange(lay.numel, dtype=torch.float64)
    for k in range(chunks):
        chunk = lay.chunk(flat, k)
        assert chunk.is_contiguous() and chunk.numel() == world * lay.per * U
        parts = [lay.shard_chunk(flat, r, k) for r in range(world)]
        # rank r's share of chunk k is the r-th equal piece of the chunk (in-place all-gather)
        assert torch.equal(torch.cat(parts), chunk)
        for r, part in enumerate(parts):
            ub, _ = lay.shard_ranges(r)[k]
            assert part.data_ptr() == flat.data_ptr() + ub * U * flat.element_size()


def test_views_are_unit_aligned_and_disjoint():
    numels = [7, 2048, 2049, 1, 4097]
    lay = FlatLayout(numels, 2)
    flat = torch.zeros(lay.numel)
    views = lay.views(flat, [(n,) for n in numels])
    end = 0
    for o, n, v in zip(lay.offsets, numels, views):
        assert o % U == 0 and o >= end and v.numel() == n
        end = o + n
    assert end <= lay.units * U <= lay.numel
