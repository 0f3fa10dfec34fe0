"""Field exchange of the seed-sharded step: every pair's noise field reaches the ranks
that replay it, instead of being regenerated there.

In the sharded schedule (one process per GPU, parameters in a ``FlatLayout``) rank r
generates the Gaussian field of each of its own pairs over every parameter in the
pair's +eps pass (the forward needs all of them perturbed), and the step's last pass on
rank r replays every pair's rounding chain on r's share of the parameters. Regenerating
those fields there doubles the noise work of the step (the passes are bound by
instruction issue, one Philox4x32-10 + log/cos per element). Here the +eps pass keeps its
field in a noise cache, and copy-engine copies push the slice of it that falls on each
rank's share into that rank's *field store* (``zt_pass_cfg.zfield``). The copies run on
the copy engines over NVLink (peer mappings through CUDA IPC) and overlap the next pair's
passes; the last pass then reads every stored field from HBM.

Store layout on each rank: ``n_slots`` slots (pairs j < n_slots are stored, the same on
every rank), each holding the rank's share in chunk order: chunk k's C units at
``slot * stride + k * C * 2048`` (fp32), ``stride = chunks * C * 2048``. The last pass's
launch over chunk k then passes ``zfield = store + k * C * 2048`` and reads unit u at
``(u - unit_begin) * 2048`` of a slot, as zt_pass documents.

Ordering (no kernel waits on another rank; the collectives order the copies):
- a pair's pushes start after its +eps pass (event on the compute stream) and the noise
  cache they read is reused two pairs later only after they finished (two caches
  alternate);
- every push of a step finishes before this rank's all-gather of the pair values starts
  (the compute stream waits for the push streams), so a rank whose all-gather completed
  knows every rank's pushes into its store have landed;
- pushes of the next step start after this rank's parameter all-gather completed, which
  needs every rank's contribution, sent only after that rank's last pass had read its
  store.

The reference runs one process per GPU with no communication (sweeps/runall.py:5), so
this module has no counterpart there.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L

U = L.ZT_UNIT_ELEMS


@dataclass(frozen=True)
class Copy:
    """One push: n_elems fp32 from the source cache at src_elem to slot storage of
    rank dst at dst_elem (element offsets into the cache / the destination store)."""
    dst: int
    dst_elem: int
    src_elem: int
    n_elems: int


def push_plan(layout, n_units: int, slot: int, world: int) -> list[Copy]:
    """The copies that move one pair's field (noise cache indexed by plan unit, n_units
    units) into slot `slot` of every rank's store, for a FlatLayout of `world` ranks."""
    C, chunks = layout.per, layout.chunks
    stride = chunks * C * U
    out = []
    for p in range(world):
        for k in range(chunks):
            start = k * world * C + p * C
            n = max(0, min(C, n_units - start))
            if n:
                out.append(Copy(p, slot * stride + k * C * U, start * U, n * U))
    return out


def store_elems(layout, n_slots: int) -> int:
    return n_slots * layout.chunks * layout.per * U


def chunk_field(layout, store_ptr: int, k: int) -> tuple[int, int]:
    """(zfield address, zfield_stride) of the last pass's launch over chunk k."""
    return store_ptr + 4 * k * layout.per * U, layout.chunks * layout.per * U


def slot_bytes(layout) -> int:
    """Bytes of one slot of a rank's field store: its share of one field, fp32."""
    return 4 * layout.chunks * layout.per * U


def slots_that_fit(layout, z_batch: int, budget_bytes: int) -> int:
    sb = slot_bytes(layout)
    return max(0, min(z_batch, budget_bytes // sb)) if sb else 0


class FieldExchange:
    """Field stores of one rank plus the peer mappings and copy streams that fill them.

    Collective: every rank of `group` constructs it with the same arguments except its
    budget; the slot count is the smallest any rank can hold."""

    def __init__(self, layout, n_units: int, rank: int, world: int, z_batch: int, device, budget_bytes: int,
                 group=None):
        import torch.distributed as dist
        self.layout, self.n_units, self.rank, self.world = layout, n_units, rank, world
        self.device = torch.device(device)
        mine = torch.tensor([slots_that_fit(layout, z_batch, budget_bytes)], dtype=torch.int64,
                            device=self.device if dist.get_backend(group) == "nccl" else "cpu")
        dist.all_reduce(mine, op=dist.ReduceOp.MIN, group=group)
        self.n_slots = int(mine.item())
        self.store = torch.empty(max(1, store_elems(layout, self.n_slots)), dtype=torch.float32, device=self.device)
        lib = L.load()
        self._opened = []
        ptrs = [0] * world
        ptrs[rank] = self.store.data_ptr()
        if world > 1:
            h = (ctypes.c_ubyte * L.ZT_IPC_HANDLE_BYTES)()
            off = ctypes.c_uint64()
            with torch.cuda.device(self.device):
                L.check(lib.zt_ipc_export(self.store.data_ptr(), h, ctypes.byref(off)), "zt_ipc_export")
            handles = [None] * world
            dist.all_gather_object(handles, (bytes(h), off.value), group=group)
            for p, (hb, o) in enumerate(handles):
                if p == rank:
                    continue
                base = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    L.check(lib.zt_ipc_open((ctypes.c_ubyte * L.ZT_IPC_HANDLE_BYTES).from_buffer_copy(hb),
                                            ctypes.byref(base)), "zt_ipc_open")
                self._opened.append(base.value)
                ptrs[p] = base.value + o
        self.peer_store = ptrs
        self.group = group
        self.plans = [push_plan(layout, n_units, j, world) for j in range(self.n_slots)]
        # one copy stream per destination: the copies to different peers run side by side
        self.streams = [torch.cuda.Stream(self.device) for _ in range(world)]
        self._last = [None] * world          # last push event per destination
        self._by_cache = {}                  # cache address -> push events that read it

    def stored(self, j: int) -> bool:
        return j < self.n_slots

    def chunk_field(self, k: int) -> tuple[int, int]:
        return chunk_field(self.layout, self.store.data_ptr(), k)

    def before_cache_write(self, cache: torch.Tensor) -> None:
        """The compute stream waits until the pushes reading `cache` are done."""
        cur = torch.cuda.current_stream(self.device)
        for ev in self._by_cache.pop(cache.data_ptr(), []):
            cur.wait_event(ev)

    def push(self, j: int, cache: torch.Tensor) -> None:
        """Push pair j's field (in `cache`, written by work already on the compute stream)
        to every rank's store."""
        if not self.stored(j):
            return
        lib = L.load()
        cur = torch.cuda.current_stream(self.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        src = cache.data_ptr()
        evs = []
        by_dst: dict[int, list[Copy]] = {}
        for c in self.plans[j]:
            by_dst.setdefault(c.dst, []).append(c)
        for p, copies in by_dst.items():
            s = self.streams[p]
            s.wait_event(ready)
            for c in copies:
                L.check(lib.zt_copy_async(self.peer_store[p] + 4 * c.dst_elem, src + 4 * c.src_elem, 4 * c.n_elems,
                                          ctypes.c_void_p(s.cuda_stream)), "zt_copy_async")
            ev = torch.cuda.Event()
            ev.record(s)
            self._last[p] = ev
            evs.append(ev)
        self._by_cache.setdefault(src, []).extend(evs)

    def finish_pushes(self) -> None:
        """The compute stream waits for every push issued so far (before the step's
        all-gather of pair values)."""
        cur = torch.cuda.current_stream(self.device)
        for ev in self._last:
            if ev is not None:
                cur.wait_event(ev)
        self._last = [None] * self.world
        self._by_cache.clear()

    def close(self, barrier: bool = True) -> None:
        """Unmap the peers' stores. With `barrier` (collective over the group) every rank
        has unmapped before any rank returns, so none frees a store another still maps."""
        lib = L.load()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for base in self._opened:
                lib.zt_ipc_close(ctypes.c_void_p(base))
        self._opened = []
        if barrier and self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def __del__(self):
        try:
            if self._opened:
                self.close(barrier=False)
        except Exception:
            pass
