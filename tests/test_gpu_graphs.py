"""CUDA-graph replay of the score function (zotitan_b200.graphs.GraphedScore), on a GPU.

On a toy bf16 Llama with the fused forward, the replayed score equals the eager score
exactly (value and metrics) for new batches and after the parameters change in place,
and a zeroth-order run scored through the graphs ends with the same parameters as one
scored eagerly.
"""
import pytest
import torch

from toy_models import build_llama

pytestmark = pytest.mark.gpu

# head_dim 16 and 256-row tiles, so the fused attention, RoPE and gated-GEMM paths run
SHAPE = dict(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, max_position_embeddings=64, tie_word_embeddings=False)
B, S = 4, 64


def _setup():
    from zotitan_b200.llama_fused import fuse_llama
    from zotitan_b200.objective import SyntheticTokensObjective
    model = build_llama(SHAPE, dtype=torch.bfloat16, device="cuda")
    assert fuse_llama(model) > 0
    return model, SyntheticTokensObjective(SHAPE["vocab_size"], S, z_loss_weight=1e-4)


def test_graphed_score_equals_eager():
    from zotitan_b200.data import synthetic_token_batch
    from zotitan_b200.graphs import GraphedScore
    model, obj = _setup()
    graphed = GraphedScore(obj.score)
    w = model.model.layers[0].mlp.gate_proj.weight
    with torch.inference_mode():
        for seed in range(4):
            batch = synthetic_token_batch(SHAPE["vocab_size"], B, S, seed, device="cuda")
            a, b = obj.score(model, batch), graphed(model, batch)
            assert torch.equal(a.value, b.value), seed
            assert set(a.metrics) == set(b.metrics)
            for k in a.metrics:
                assert torch.equal(torch.as_tensor(a.metrics[k]), torch.as_tensor(b.metrics[k])), k
            w.add_(1e-3)   # in place, as the zeroth-order passes change the parameters
    assert len(graphed._graphs) == 1   # one batch shape, one capture


def test_zo_steps_with_graphed_score_match_eager():
    from zotitan_b200.data import synthetic_token_batch
    from zotitan_b200.graphs import GraphedScore
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer
    runs = []
    for use_graphs in (False, True):
        model, obj = _setup()
        cfg = ZOConfig()
        cfg.z_batch, cfg.eps, cfg.base.lr = 2, 1e-3, 1e-2
        score = GraphedScore(obj.score) if use_graphs else obj.score
        opt = ZOOptimizer([(n, p) for n, p in model.named_parameters()], cfg, score, total_steps=3)
        losses = []
        for t in range(3):
            batches = [synthetic_token_batch(SHAPE["vocab_size"], B, S, 10 * t + j, device="cuda") for j in range(2)]
            losses.append(opt.step(model, batches)["loss"])
        runs.append((losses, [p.detach().clone() for p in model.parameters()]))
    assert runs[0][0] == runs[1][0]
    for a, b in zip(runs[0][1], runs[1][1]):
        assert torch.equal(a, b)
