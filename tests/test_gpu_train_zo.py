"""The public training entry point train_zo (zotitan/train_zo.py:609-675), on a GPU.

train_zo is what `./train.py --optimizer zo` calls. On a toy bf16 Llama with the
synthetic-token objective it must: log one metrics dict per step with the reference's
keys, call merge_fn after every step, save the model and the optimizer state at
ckpt_every, and leave the model exactly where a hand-written loop of ZOOptimizer.step
over the same batches leaves it (the loader and the loop add no arithmetic).
"""
import os

import pytest
import torch

from toy_models import TOY, build_llama

pytestmark = pytest.mark.gpu


class ListLogger:
    def __init__(self):
        self.rows = []

    def log(self, metrics):
        self.rows.append(dict(metrics))


def _cfg(shared_batch=False):
    from zotitan_b200.train_zo import ZOConfig
    cfg = ZOConfig()
    cfg.z_batch, cfg.batch_size, cfg.eps, cfg.shared_batch = 2, 2, 1e-3, shared_batch
    cfg.base.lr, cfg.base.ckpt_every = 1e-2, 2
    return cfg


@pytest.mark.parametrize("shared_batch", [False, True])
def test_train_zo_matches_manual_loop(tmp_path, monkeypatch, shared_batch):
    from zotitan_b200.data import get_batches
    from zotitan_b200.objective import SyntheticTokensObjective
    from zotitan_b200.train_zo import ZOOptimizer, train_zo
    monkeypatch.setenv("MLSWEEP_RUN_DIR", str(tmp_path))
    steps, seed = 3, 5
    objective = SyntheticTokensObjective(TOY["vocab_size"], 16, z_loss_weight=1e-4)
    model = build_llama(TOY, dtype=torch.bfloat16, device="cuda")
    ref = build_llama(TOY, dtype=torch.bfloat16, device="cuda")
    merges = []
    logger = ListLogger()
    out = train_zo(model, None, steps, seed, lambda m: merges.append(m), logger, cfg=_cfg(shared_batch),
                   objective=objective)
    assert out is model and len(merges) == steps and len(logger.rows) == steps
    for row in logger.rows:
        for k in ("loss", "proj_grad", "proj_grad_clipped", "clip_frac", "clip_tau", "lr", "step_time", "ce"):
            assert k in row, k
        assert torch.isfinite(torch.tensor(row["loss"]))
    assert os.path.exists(tmp_path / "zo_optimizer.pt") and os.path.isdir(tmp_path / "checkpoint")
    sd = torch.load(tmp_path / "zo_optimizer.pt", weights_only=False)
    assert sd["planner"]["t"] == 2         # saved after step 2 (ckpt_every = 2)

    # the same steps by hand: the loader's batches in order, then ZOOptimizer.step
    cfg = _cfg(shared_batch)
    named = [(n, p) for n, p in ref.named_parameters() if p.requires_grad]
    opt = ZOOptimizer(named, cfg, objective.score, total_steps=steps)
    it = iter(objective.train_batches(None, seed, cfg.batch_size))
    to_dev = lambda b: {k: v.cuda() for k, v in b.items()}  # noqa: E731
    for _ in range(steps):
        if shared_batch:
            batches = [to_dev(next(it))] * cfg.z_batch
        else:
            batches = [to_dev(b) for b in get_batches(it, cfg.z_batch)]
        m = opt.step(ref, batches)
    assert m["loss"] == logger.rows[-1]["loss"]
    for (n, a), (_, b) in zip(model.named_parameters(), ref.named_parameters()):
        assert torch.equal(a, b), n
