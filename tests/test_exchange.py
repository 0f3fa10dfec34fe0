"""Field-exchange geometry (zotitan_b200.exchange), on CPU.

W ranks are emulated in one process with numpy: each rank's noise cache holds its own
pairs' fields (indexed by plan unit), every rank applies its push plan into every rank's
store, and each store slot must then hold, at the offsets the last pass reads for unit u
of chunk k (zfield = store + k*C*2048, slot*stride + (u - unit_begin)*2048), exactly
field_j[u*2048 ...] -- for every rank, chunk, unit of its share and stored pair.
"""
import numpy as np
import pytest

from zotitan_b200.exchange import chunk_field, push_plan, rotating_peers, slots_that_fit, store_elems
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


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_in_pass_destination_formula_matches_push_plan(world):
    """The +eps pass kernel's push (zt_pass_cfg.zpush) puts unit u of the flat layout at
    zpush[p][slot * stride + (kc * C + o) * 2048] with kc = u / (W C), p = (u mod W C) / C,
    o = u mod C; the copy path's push_plan puts the same unit at the same place."""
    layout = FlatLayout([5000, 2048 * 3, 8, 2048 * 9 + 8, 24, 40000, 2048 * 70], world)
    n_units, C, W = layout.units, layout.per, world
    stride = layout.chunks * C * U
    slot = 3
    want = {}
    for c in push_plan(layout, n_units, slot, world):
        first_unit = c.src_elem // U
        for i in range(c.n_elems // U):
            want[first_unit + i] = (c.dst, c.dst_elem + i * U)
    got = {}
    for u in range(n_units):
        kc, within = divmod(u, W * C)
        p, o = divmod(within, C)
        got[u] = (p, slot * stride + (kc * C + o) * U)
    assert got == want


def _bare_exchange(s_max, world=4):
    from zotitan_b200.exchange import FieldExchange
    ex = object.__new__(FieldExchange)
    ex.world, ex.in_pass, ex.adaptive = world, False, True
    ex.s_max = ex.s = s_max
    return ex


def test_adapt_stores_fewer_pairs_while_pushes_lag_and_cost_more_than_regeneration():
    ex = _bare_exchange(8)
    assert ex.active == 32 and ex.stored(31) and not ex.stored(32)
    ex.adapt(lag=10.0, push=2.0, plus=1.5, local_pairs=8)     # 4 pushes too many -> drop 4
    assert ex.s == 4 and ex.active == 16
    ex.adapt(lag=1.5, push=2.0, plus=1.5, local_pairs=8)      # within one push: hold
    assert ex.s == 4
    ex.adapt(lag=0.5, push=2.0, plus=1.5, local_pairs=8)      # ends early: one more
    assert ex.s == 5
    ex.adapt(lag=10.0, push=1.0, plus=1.5, local_pairs=8)     # pushes cheaper than regenerating: hold
    assert ex.s == 5
    ex.adapt(lag=100.0, push=2.0, plus=1.5, local_pairs=8)    # never below zero
    assert ex.s == 0
    ex.adapt(lag=0.0, push=0.0, plus=0.0, local_pairs=8)      # nothing measured: hold
    assert ex.s == 0


def test_adapt_caps_at_slots_and_local_pairs():
    ex = _bare_exchange(3)
    ex.s = 2
    ex.adapt(lag=0.0, push=2.0, plus=1.0, local_pairs=2)
    assert ex.s == 2
    ex.adapt(lag=0.0, push=2.0, plus=1.0, local_pairs=8)
    assert ex.s == 3
    ex.adapt(lag=0.0, push=2.0, plus=1.0, local_pairs=8)
    assert ex.s == 3
    ex.adaptive = False
    ex.adapt(lag=50.0, push=2.0, plus=1.0, local_pairs=8)
    assert ex.s == 3


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_rotating_pushes_are_permutations_at_every_step(world):
    """Push k of every rank goes to rank + k: each step is a permutation (no receiver gets
    two senders at once), every rank reaches every peer exactly once, never itself."""
    orders = [rotating_peers(r, world) for r in range(world)]
    for r, o in enumerate(orders):
        assert sorted(o) == [p for p in range(world) if p != r]
    for k in range(world - 1):
        assert sorted(o[k] for o in orders) == list(range(world))
