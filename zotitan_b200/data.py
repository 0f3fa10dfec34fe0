"""Batch prefetch and synthetic token batches.

``PrefetchLoader`` / ``get_batches`` keep the contract of zotitan/data.py:104-177:
one batch of look-ahead fetched by a background thread and copied to the device on
a side CUDA stream; loader exceptions are re-raised in the consumer.
``synthetic_token_batches`` is the seeded per-(step, pair) token source the
benchmarks and sharded runs use, so every rank derives its own batches without
exchanging data.
"""
from __future__ import annotations

import threading

import torch


class PrefetchLoader:
    def __init__(self, iterator, device, move_fn=None):
        self._it = iter(iterator)
        self.device = torch.device(device)
        self._stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self._move = move_fn
        self._ready = None
        self._thread = None
        self._prefetch()

    def _move_batch(self, batch):
        if self._move is not None:
            return self._move(batch, self.device)
        return {k: v.pin_memory().to(self.device, non_blocking=True) for k, v in batch.items()}

    def _prefetch(self):
        def _task():
            try:
                batch = next(self._it)
            except BaseException as e:  # StopIteration or a loader error, surfaced in __next__
                self._ready = e
                return
            if self._stream is not None:
                with torch.cuda.stream(self._stream):
                    batch = self._move_batch(batch)
            elif self._move is not None:
                batch = self._move(batch, self.device)
            else:
                batch = {k: v.to(self.device) for k, v in batch.items()}
            self._ready = batch

        self._thread = threading.Thread(target=_task, daemon=True)
        self._thread.start()

    def __iter__(self):
        return self

    def __next__(self):
        assert self._thread is not None, "PrefetchLoader not properly initialized"
        self._thread.join()
        item, self._ready = self._ready, None
        if isinstance(item, BaseException):
            raise item
        if self._stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._stream)
        self._prefetch()
        return item


def get_batches(loader, n: int):
    """Pull n batches; None if the loader runs dry first (zotitan/data.py:168-177)."""
    batches = []
    for _ in range(n):
        batch = next(loader, None)
        if batch is None:
            return None
        batches.append(batch)
    return batches


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
