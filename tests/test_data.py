"""Batch plumbing of the training loop (zotitan_b200.data), on CPU.

PrefetchLoader keeps the contract of the reference's loader (zotitan/data.py:104-177):
batches arrive in order with one of look-ahead fetched by a background thread, an error
raised by the source surfaces in the consumer's next(), and get_batches returns None
once the source runs dry. The synthetic token source is a pure function of its seed.
"""
import pytest
import torch

from zotitan_b200.data import PrefetchLoader, get_batches, synthetic_token_batch, synthetic_token_batches


def _source(n):
    for i in range(n):
        yield {"input_ids": torch.full((2, 3), i), "labels": torch.full((2, 3), i)}


def test_prefetch_loader_order_and_exhaustion():
    loader = PrefetchLoader(_source(5), "cpu")
    got = get_batches(loader, 3)
    assert [int(b["input_ids"][0, 0]) for b in got] == [0, 1, 2]
    assert get_batches(loader, 3) is None          # only 2 left: the reference returns None
    assert get_batches(loader, 1) is None          # and keeps returning None once dry


def test_prefetch_loader_reraises_source_errors():
    def bad():
        yield {"input_ids": torch.zeros(1)}
        raise RuntimeError("broken shard")
    loader = PrefetchLoader(bad(), "cpu")
    next(loader)
    with pytest.raises(RuntimeError, match="broken shard"):
        next(loader)


def test_prefetch_loader_move_fn():
    seen = []

    def move(batch, device):
        seen.append(device)
        return {k: v + 100 for k, v in batch.items()}
    loader = PrefetchLoader(_source(2), "cpu", move_fn=move)
    assert int(next(loader)["labels"][0, 0]) == 100
    assert seen and all(d == torch.device("cpu") for d in seen)


def test_synthetic_batches_are_seeded():
    a = synthetic_token_batch(50, 2, 8, seed=7)
    b = synthetic_token_batch(50, 2, 8, seed=7)
    c = synthetic_token_batch(50, 2, 8, seed=8)
    assert torch.equal(a["input_ids"], b["input_ids"]) and not torch.equal(a["input_ids"], c["input_ids"])
    assert torch.equal(a["input_ids"], a["labels"])
    assert int(a["input_ids"].max()) < 50 and int(a["input_ids"].min()) >= 0
    it1, it2 = synthetic_token_batches(50, 2, 8, seed=3), synthetic_token_batches(50, 2, 8, seed=3)
    for _ in range(3):
        assert torch.equal(next(it1)["input_ids"], next(it2)["input_ids"])


def test_prefetch_loader_keeps_exactly_depth_batches_ahead():
    import time
    pulled = []

    def counting():
        for i in range(10):
            pulled.append(i)
            yield {"input_ids": torch.full((1,), i)}

    for depth in (1, 3):
        pulled.clear()
        loader = PrefetchLoader(counting(), "cpu", depth=depth)
        time.sleep(0.2)
        assert len(pulled) == depth            # fetched ahead, no further
        next(loader)
        time.sleep(0.2)
        assert len(pulled) == depth + 1
        loader.close()
