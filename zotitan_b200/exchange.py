"""Field exchange of the seed-sharded step: every pair's noise field reaches the ranks
that replay it, instead of being regenerated there.

In the sharded schedule (one process per GPU, parameters in a ``FlatLayout``) rank r
generates the Gaussian field of each of its own pairs over every parameter in the
pair's +eps pass (the forward needs all of them perturbed), and the step's last pass on
rank r replays every pair's rounding chain on r's share of the parameters. Regenerating
those fields there doubles the noise work of the step (the passes are bound by
instruction issue, one Philox4x32-10 + log/cos per element). Instead every pair's field
lands in the *field stores* (``zt_pass_cfg.zfield``) of the ranks that replay it, and the
last pass reads every stored field from HBM. Two ways of getting it there:

- by copies (the default): the +eps pass keeps its field in a noise cache and copy-engine
  copies (``zt_copy_async``) push the slices into the stores, overlapping the next pairs'
  passes; two or three caches rotate between a rank's pairs. The slices of a pair go to
  rank + 1, rank + 2, ... one after another on one link stream (``push_order="rotate"``):
  the ranks push in step, so every moment is a permutation of the ranks (762 GB/s per GPU
  measured at 4 ranks). Every rank pushing to its peers in the same order (lowest rank
  first) puts all first copies on one receiver: 391 GB/s;
- in the pass (``in_pass``, when the plan takes the specialised +eps kernel and there are
  at most ZT_MAX_PUSH_RANKS ranks): the +eps pass that generates the field also stores
  each unit of it straight into the owning rank's store over NVLink (``zt_pass_cfg.zpush``,
  peer mappings through CUDA IPC), then fences at system scope. Measured at 4 ranks it
  made the +eps pass the bottleneck (193 against 157 ms per step by copies in rank order):
  every rank's kernel walks the units in the same order, so all ranks store to the same
  owner at once (the hot spot of copies issued in rank order, ~390 GB/s per GPU), and the
  remote stores hold the pass's warps.

The push rate bounds what the copies can carry. So the number of stored pairs adapts (``adapt``):
each rank times how long its pushes ran past its local passes in the previous step, the
timings ride on the pair-value all-gather, and every rank applies the same rule to the
same maxima, so the count changes between steps and identically everywhere.

Store layout on each rank: ``n_slots`` slots (pairs j < n_slots are stored, the same on
every rank), each holding the rank's share in chunk order: chunk k's C units at
``slot * stride + k * C * 2048`` (fp32), ``stride = chunks * C * 2048``. The last pass's
launch over chunk k then passes ``zfield = store + k * C * 2048`` and reads unit u at
``(u - unit_begin) * 2048`` of a slot, as zt_pass documents.

Ordering (no kernel waits on another rank; the collectives order the pushes):
- copies: a pair's pushes start after its +eps pass (event on the compute stream) and the
  noise cache they read is reused two pairs later only after they finished;
- every push of a step finishes before this rank's all-gather of the pair values starts
  (in the pass: the +eps kernels precede it on the compute stream and end with a
  system-scope fence; copies: the compute stream waits for the copy streams), so a rank
  whose all-gather completed knows every rank's pushes into its store have landed;
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


def rotating_peers(rank: int, world: int) -> list[int]:
    """The peers rank `rank` pushes a pair's slices to, in order: rank + 1, rank + 2, ...
    (mod world). The k-th push of every rank goes to rank + k, so when the ranks push in
    step each of the world - 1 steps is a permutation: every rank sends to one peer and
    receives from one."""
    return [(rank + k) % world for k in range(1, world)]


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
                 group=None, in_pass: bool = False, push_streams: int = 1, push_order: str = "rotate"):
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
        self.in_pass = bool(in_pass) and world <= L.ZT_MAX_PUSH_RANKS
        self.plans = [push_plan(layout, n_units, j, world) for j in range(self.n_slots)]
        # Push order. "rotate" (default): one link stream sends a pair's slices to rank + 1,
        # rank + 2, ... in turn, so while the ranks push in step every moment is a permutation
        # (each GPU sends to one peer and receives from one); the rank's own slice goes on a
        # second stream. "all": copy streams per destination (`push_streams` each), issued in
        # rank order, every peer at once. Measured at 4 ranks (bench.py --profile-case
        # push-rates): rotating 762 GB/s per GPU; every peer at once 713-759 GB/s when each
        # rank starts at its next peer, 391 GB/s when all ranks start at the same peer.
        if push_order not in ("rotate", "all"):
            raise ValueError(f"push_order must be 'rotate' or 'all', got {push_order!r}")
        self.push_order = push_order
        self.push_streams = max(1, int(push_streams))
        if push_order == "rotate":
            self.streams = [[torch.cuda.Stream(self.device)], [torch.cuda.Stream(self.device)]]   # link, local
        else:
            self.streams = [[torch.cuda.Stream(self.device) for _ in range(self.push_streams)] for _ in range(world)]
        self._n_streams = sum(len(x) for x in self.streams)
        self._last = [None] * self._n_streams   # last push event per copy stream
        self._by_cache = {}                  # cache address -> push events that read it
        # Stored pairs in use: pairs j < active = s * world, i.e. the first s own pairs of
        # every rank (pairs go round-robin: pair j is rank j % W's (j // W)-th). Every rank
        # updates s with the same rule from the same all-gathered timings (adapt).
        self.s_max = self.n_slots // world
        self.s = self.s_max
        self.adaptive = not self.in_pass
        self._cur = self._prev = None

    @property
    def active(self) -> int:
        return self.s * self.world

    def stored(self, j: int) -> bool:
        return j < self.active

    # -- timing of the copies against the local passes, for the stored-pair count --------
    def begin_step(self) -> None:
        """Start the step's timing record (the previous step's is kept for stats())."""
        self._prev, self._cur = self._cur, {"push_start": None, "push_end": [], "plus": None, "local_done": None,
                                            "pushed": 0}
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(self.device))
        self._cur["start"] = ev

    def note_plus(self, before, after) -> None:
        """Events around one +eps pass of the step (its duration is the cost of
        regenerating one pair's worth of noise)."""
        if self._cur is not None and self._cur["plus"] is None:
            self._cur["plus"] = (before, after)

    def local_done(self) -> None:
        if self._cur is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self._cur["local_done"] = ev

    def stats(self) -> tuple[float, float, float]:
        """(lag, push, plus) in ms from the previous step: how long its pushes ran past the
        end of its local passes, the copy time of one pair's push at the rate it sustained,
        and one +eps pass. Zeros when there is nothing to report."""
        t = self._prev
        if not self.adaptive or t is None or t["push_start"] is None or not t["push_end"] or t["plus"] is None \
                or t["local_done"] is None or t["pushed"] == 0:
            return 0.0, 0.0, 0.0
        evs = [t["push_start"], t["local_done"], *t["push_end"], *t["plus"]]
        if not all(e.query() for e in evs):
            return 0.0, 0.0, 0.0
        end = max(t["push_start"].elapsed_time(e) for e in t["push_end"])      # first push start -> last end
        lag = max(0.0, end - t["push_start"].elapsed_time(t["local_done"]))
        push = end / t["pushed"]
        plus = t["plus"][0].elapsed_time(t["plus"][1])
        return lag, push, plus

    def adapt(self, lag: float, push: float, plus: float, local_pairs: int) -> None:
        """Update the stored own-pair count s from the all-gathered maxima of stats(): while
        the pushes run more than one pair's push past the local passes and a pair's push
        costs more than regenerating its noise in the last pass (about one +eps pass), store
        fewer pairs; when they end within half a push, store one more."""
        if not self.adaptive or push <= 0.0:
            return
        s_cap = min(self.s_max, local_pairs)
        if lag > push and push > plus and self.s > 0:
            self.s = max(0, self.s - max(1, int((lag - push) / push + 0.999)))
        elif lag < 0.5 * push and self.s < s_cap:
            self.s += 1

    def set_push(self, cfg, j: int) -> None:
        """In-pass mode: point the +eps pass of pair j (a kernels.PassCfg) at slot j of every
        rank's store, if pair j is stored."""
        if self.in_pass and self.stored(j):
            cfg.zpush = tuple(self.peer_store)
            cfg.zpush_slot = j
            cfg.zpush_chunk_units = self.layout.per
            cfg.zpush_stride = self.layout.chunks * self.layout.per * U

    def chunk_field(self, k: int) -> tuple[int, int]:
        return chunk_field(self.layout, self.store.data_ptr(), k)

    def before_cache_write(self, cache: torch.Tensor) -> None:
        """The compute stream waits until the pushes reading `cache` are done."""
        if self.in_pass:
            return
        cur = torch.cuda.current_stream(self.device)
        for ev in self._by_cache.pop(cache.data_ptr(), []):
            cur.wait_event(ev)

    def push(self, j: int, cache: torch.Tensor) -> None:
        """Push pair j's field (in `cache`, written by work already on the compute stream)
        to every rank's store (copies; in-pass mode pushes from the +eps pass itself)."""
        if self.in_pass or not self.stored(j):
            return
        lib = L.load()
        cur = torch.cuda.current_stream(self.device)
        timing = self.adaptive and self._cur is not None
        ready = torch.cuda.Event(enable_timing=timing)
        ready.record(cur)
        if timing:
            if self._cur["push_start"] is None:
                self._cur["push_start"] = ready
            self._cur["pushed"] += 1
        src = cache.data_ptr()
        evs = []
        by_dst: dict[int, list[Copy]] = {}
        for c in self.plans[j]:
            by_dst.setdefault(c.dst, []).append(c)
        if self.push_order == "rotate":
            work = [(0, self.streams[0][0], rotating_peers(self.rank, self.world)),
                    (1, self.streams[1][0], [self.rank])]
        else:
            work = []
            for p in by_dst:
                k = min(self.push_streams, len(by_dst[p]))
                for q in range(k):
                    work.append((p * self.push_streams + q, self.streams[p][q], [(p, q, k)]))
        for slot, s, dsts in work:
            s.wait_event(ready)
            for d in dsts:
                if self.push_order == "rotate":
                    p, copies = d, by_dst.get(d, [])
                else:
                    p, q, k = d
                    copies = by_dst[p][q::k]
                for c in copies:
                    L.check(lib.zt_copy_async(self.peer_store[p] + 4 * c.dst_elem, src + 4 * c.src_elem,
                                              4 * c.n_elems, ctypes.c_void_p(s.cuda_stream)), "zt_copy_async")
            ev = torch.cuda.Event(enable_timing=timing)
            ev.record(s)
            self._last[slot] = ev
            evs.append(ev)
        self._by_cache.setdefault(src, []).extend(evs)
        if timing:
            self._cur["push_end"] = [e for e in self._last if e is not None]

    def finish_pushes(self) -> None:
        """The compute stream waits for every push issued so far (before the step's
        all-gather of pair values)."""
        cur = torch.cuda.current_stream(self.device)
        for ev in self._last:
            if ev is not None:
                cur.wait_event(ev)
        self._last = [None] * self._n_streams
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
