"""Batch prefetch and synthetic token batches.

``PrefetchLoader`` / ``get_batches`` keep the contract of zotitan/data.py:104-177:
batches are fetched ahead of the consumer by a background thread and copied to the
device on a side CUDA stream, an exception raised by the source surfaces in the
consumer's ``next()``, and ``get_batches`` returns None once the source runs dry.
``synthetic_token_batches`` is the seeded per-(step, pair) token source the
benchmarks and sharded runs use, so every rank derives its own batches without
exchanging data.
"""
from __future__ import annotations

import queue
import threading

import torch


class _End:
    """Queue item that ends the stream: the source's StopIteration or its error."""

    def __init__(self, exc: BaseException):
        self.exc = exc


class PrefetchLoader:
    """Iterate `iterator` with `depth` batches fetched and moved to `device` ahead.

    One worker thread pulls from the source. It holds a credit per batch it may have
    outstanding (a semaphore of `depth` credits, one returned per batch consumed), so
    it never runs further ahead than `depth` batches (the reference keeps one). On CUDA
    the worker moves each batch on its own stream (pinned host copy, non-blocking
    device copy, or `move_fn(batch, device)`) and records an event; the consumer's
    current stream waits on that event, and every tensor of the batch is marked as used
    by the consumer's stream so the caching allocator cannot hand its memory out early.
    """

    def __init__(self, iterator, device, move_fn=None, depth: int = 1):
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self._src = iter(iterator)
        self.device = torch.device(device)
        self._move_fn = move_fn
        self._cuda = self.device.type == "cuda"
        self._side = torch.cuda.Stream(self.device) if self._cuda else None
        self._credits = threading.Semaphore(depth)
        self._out: queue.Queue = queue.Queue()
        self._closed = threading.Event()
        self._done = None
        self._worker = threading.Thread(target=self._work, name="PrefetchLoader", daemon=True)
        self._worker.start()

    def _to_device(self, batch):
        if self._move_fn is not None:
            return self._move_fn(batch, self.device)
        if not self._cuda:
            return {k: v.to(self.device) for k, v in batch.items()}
        return {k: v.pin_memory().to(self.device, non_blocking=True) for k, v in batch.items()}

    def _work(self):
        while True:
            self._credits.acquire()
            if self._closed.is_set():
                return
            try:
                batch = next(self._src)
                if self._cuda:
                    with torch.cuda.stream(self._side):
                        batch = self._to_device(batch)
                        ready = torch.cuda.Event()
                        ready.record(self._side)
                else:
                    batch, ready = self._to_device(batch), None
            except BaseException as e:  # StopIteration or an error of the source
                self._out.put(_End(e))
                return
            self._out.put((batch, ready))

    def __iter__(self):
        return self

    def __next__(self):
        if self._done is not None:
            raise self._done
        item = self._out.get()
        if isinstance(item, _End):
            self._done = StopIteration() if isinstance(item.exc, StopIteration) else item.exc
            raise item.exc
        batch, ready = item
        if ready is not None:
            consumer = torch.cuda.current_stream(self.device)
            consumer.wait_event(ready)
            for v in (batch.values() if isinstance(batch, dict) else ()):
                if isinstance(v, torch.Tensor) and v.is_cuda:
                    v.record_stream(consumer)
        self._credits.release()
        return batch

    def close(self):
        """Stop the worker after the batch it is fetching (if any)."""
        self._closed.set()
        self._credits.release()


def get_batches(loader, n: int):
    """The next n batches of `loader` as a list, or None if it runs dry first
    (zotitan/data.py:168-177)."""
    out = []
    while len(out) < n:
        batch = next(loader, None)
        if batch is None:
            return None
        out.append(batch)
    return out


def synthetic_token_batch(vocab: int, batch: int, seq: int, seed: int, device="cpu",
                          pin: bool = False) -> dict:
    """Uniform random token ids from torch.Generator(seed); labels = input ids (next-token CE)."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq), generator=g)
    if pin:
        ids = ids.pin_memory()
    ids = ids.to(device, non_blocking=pin)
    return {"input_ids": ids, "labels": ids}


def synthetic_token_batches(vocab: int, batch: int, seq: int, seed: int = 0):
    """Endless iterator of synthetic batches; batch k uses seed (seed, k)."""
    k = 0
    while True:
        yield synthetic_token_batch(vocab, batch, seq, seed * 1_000_003 + k)
        k += 1
