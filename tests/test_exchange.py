"""Field-exchange geometry (zotitan_b200.exchange), on CPU.

W ranks are emulated in one process with numpy: each rank's noise cache holds its own
pairs' fields (indexed by plan unit), every rank applies its push plan into every rank's
store, and each store slot must then hold, at the offsets the last pass reads for unit u
of chunk k (zfield = store + k*C*2048, slot*stride + (u - unit_begin)*2048), exactly
field_j[u*2048 ...] -- for every rank, chunk, unit of its share and stored pair.
"""
import numpy as np
import pytest

from zotitan_b200.exchange import chunk_field, push_plan, slots_that_fit, store_elems
from zotitan_b200.flat import FlatLayout

U = 2048


def field(j, n_units):
    """A field whose every element names its pair and position."""
    return (np.arange(n_units * U, dtype=np.float64) + 1e9 * (j + 1)).astype(np.float64)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("numels", [[5000, 3, 2048 * 7 + 1], [2048 * 64], [1, 1, 1, 1, 1]])
def test_push_plan_fills_every_share_exactly(world, numels):
    layout = FlatLayout(numels, world)
    n_units = layout.units
    Z = 2 * world + 1
    pairs_of = {r: list(range(r, Z, world)) for r in range(world)}
    n_slots = Z - 1                       # the last pair is not stored
    stores = [np.full(store_elems(layout, n_slots), np.nan) for _ in range(world)]
    written = [np.zeros(store_elems(layout, n_slots), dtype=int) for _ in range(world)]
    for src in range(world):
        for j in pairs_of[src]:
            if j >= n_slots:
                continue
            f = field(j, n_units)
            for c in push_plan(layout, n_units, j, world):
                assert 0 <= c.src_elem and c.src_elem + c.n_elems <= f.size
                assert 0 <= c.dst_elem and c.dst_elem + c.n_elems <= stores[c.dst].size
                stores[c.dst][c.dst_elem:c.dst_elem + c.n_elems] = f[c.src_elem:c.src_elem + c.n_elems]
                written[c.dst][c.dst_elem:c.dst_elem + c.n_elems] += 1
    for r in range(world):
        assert written[r].max() <= 1                       # no element written twice
        for k, (ub, ue) in enumerate(layout.shard_ranges(r)):
            ue = min(ue, n_units)                           # the pass clamps to the plan's units
            zf, stride = chunk_field(layout, 0, k)
            base = zf // 4
            for j in range(n_slots):
                f = field(j, n_units)
                for u in range(ub, ue):
                    off = base + j * stride + (u - ub) * U
                    assert np.array_equal(stores[r][off:off + U], f[u * U:(u + 1) * U]), (r, k, j, u)


def test_slots_that_fit():
    layout = FlatLayout([2048 * 100], 2)
    slot_bytes = 4 * layout.chunks * layout.per * U
    assert slots_that_fit(layout, 64, 0) == 0
    assert slots_that_fit(layout, 64, 3 * slot_bytes + 5) == 3
    assert slots_that_fit(layout, 4, 100 * slot_bytes) == 4
