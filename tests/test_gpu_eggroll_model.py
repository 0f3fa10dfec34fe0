"""EGGROLL population forward vs member-by-member evaluation with materialised weights.

The oracle side perturbs a plain HF Llama with the reference's low_rank branch restated
op by op (oracle.zo_step.OracleZO.sample_z, distribution "low_rank", rank 4, C-oracle
noise) as theta + sign*sigma*z and runs one forward per member. The population side runs
all members in one forward through zotitan_b200.eggroll (tcgen05 GEMMs with the rank-4
term in the epilogue, perturbed norms and embedding rows). Bar: per-member cross-entropy
within 1e-3 relative.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPE = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=4, max_position_embeddings=128, tie_word_embeddings=False)
SIGMA = 2e-2


def _cfg(rank=4):
    from types import SimpleNamespace as NS
    return NS(mom=NS(momentum_method="none", second_moment=False), clip=NS(strategy="none", clip_pct=0.0, window=1),
              weight_decay=NS(strategy="none", lambda_=0.0), fitness=NS(strategy="none"),
              perturbation=NS(distribution="low_rank", rank=rank), seed_window=NS(size=0))


def _member_losses_materialised(tokens, pair_seeds):
    from oracle import philox as ph
    from oracle.zo_step import OracleZO
    from toy_models import build_llama
    base = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    named = [(n, p) for n, p in base.named_parameters()]
    host = [p.detach().float().cpu().numpy() for _, p in named]
    oz = OracleZO([h.copy() for h in host], [ph.BF16] * len(host), _cfg(), noise="c", semantics="cuda")
    losses = []
    for s in pair_seeds:
        z = oz.sample_z(s)
        for sign in (1.0, -1.0):
            with torch.no_grad():
                for (_, p), h, zz in zip(named, host, z):
                    pert = torch.from_numpy(h).cuda() + sign * SIGMA * torch.from_numpy(np.ascontiguousarray(zz)).cuda()
                    p.copy_(pert.to(torch.bfloat16))
                out = base(input_ids=tokens, labels=tokens)
            losses.append(float(out.loss))
    return losses


@pytest.mark.parametrize("batch", [2, 4])
def test_population_forward_matches_materialised_members(batch):
    """batch 2 (128 rows per member): the rank-4 terms in fp32 epilogues; batch 4 (256 rows
    per member): the rank-4 terms as tensor-core K-slabs. Both run the gated MLP GEMM."""
    from toy_models import build_llama
    from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
    g = torch.Generator().manual_seed(5)
    tokens = torch.randint(0, SHAPE["vocab_size"], (batch, 64), generator=g).cuda()
    pair_seeds = [3, 11]
    model = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    pop = EggrollPopulation(model, EggrollConfig(sigma=SIGMA))
    got = pop.evaluate(tokens, pair_seeds).cpu().numpy()
    from zotitan_b200 import kernels as K
    assert K.eggroll_take_error() == 0
    want = _member_losses_materialised(tokens, pair_seeds)
    np.testing.assert_allclose(got, want, rtol=1e-3)
    # antithetic members really differ, and differ from the unperturbed model
    base = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    with torch.no_grad():
        l0 = float(base(input_ids=tokens, labels=tokens).loss)
    assert abs(got[0] - got[1]) > 1e-4 and abs(got[0] - l0) > 1e-5
