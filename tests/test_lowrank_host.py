"""Host-side arithmetic of the fused low-rank path (no GPU): how a step's seeds are split
into launches of the low-rank kernels, and the exact three-way bf16 split of fp32 factors."""
import torch

from zotitan_b200 import _lib as L


def _bare_optimizer(shape, dtype, rank):
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer
    opt = object.__new__(ZOOptimizer)
    opt.params = [torch.zeros(shape, dtype=dtype)]
    opt.cfg = ZOConfig()
    opt.cfg.perturbation.rank = rank
    return opt


def test_seed_chunks_respect_stream_limit_and_buffer_budget():
    seeds = list(range(300))
    small = _bare_optimizer((256, 512), torch.bfloat16, 64)         # 98 KB of factors per seed
    chunks = small._lr_seed_chunks(seeds, 0)
    assert [len(c) for c in chunks] == [L.ZT_LOWRANK_MAX_STREAMS] * 2 + [300 - 2 * L.ZT_LOWRANK_MAX_STREAMS]
    assert sum(chunks, []) == seeds                                  # every seed once, in order
    big = _bare_optimizer((128256, 2048), torch.float32, 64)        # fp32: K = 9 r = 576, 150 MB per seed
    per_seed = (128256 + 2048) * 576 * 2
    chunks = big._lr_seed_chunks(seeds, 0)
    assert max(len(c) for c in chunks) == (2 << 30) // per_seed
    assert sum(chunks, []) == seeds


def test_split3_is_exact():
    from zotitan_b200.kernels import _split3
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4096, generator=g) * torch.logspace(-30, 30, 4096)
    parts = _split3(x)
    assert all(p.dtype == torch.bfloat16 for p in parts)
    assert torch.equal(parts[0].double() + parts[1].double() + parts[2].double(), x.double())
