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


@pytest.mark.parametrize("n_pairs", [4, 8])
def test_es_update_matches_sum_of_materialised_directions(n_pairs):
    """EggrollPopulation.apply_update (rank-4*pairs GEMM for 2-D tensors, dense Gaussian
    sum for 1-D) against theta - lr * sum_j coef_j z_j with every z_j materialised by the
    oracle's restatement of the reference's low_rank branch. The oracle rounds each z_j to
    bf16 twice (product, then the scaled product) and takes the norm of the rounded product,
    as the reference does; the factors normalise the exact product, whose bf16-rounded norm
    can sit one step away. So the bar is one bf16 step of theta plus 2^-6 of
    lr * sum_j |coef_j z_j| (the terms' rounding does not cancel where the terms do)."""
    from oracle.zo_step import OracleZO
    from toy_models import build_llama
    from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
    model = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    named = [(n, p) for n, p in model.named_parameters()]
    host = [p.detach().float().cpu().numpy() for _, p in named]
    pop = EggrollPopulation(model, EggrollConfig(sigma=SIGMA))
    # 4 pairs: inner dimension 32, the update through torch's addmm; 8 pairs: 64, zt_gemm_addto
    seeds = [3, 11, 17, 23, 29, 31, 37, 41][:n_pairs]
    coefs = [0.25, -0.5, 0.125, 0.75, -0.375, 0.0625, 0.5, -0.25][:n_pairs]
    lr = 1e-2
    from zotitan_b200 import kernels as K
    calls = {"n": 0}
    orig = K.gemm_addto

    def counting(*a, **kw):
        calls["n"] += 1
        return orig(*a, **kw)

    K.gemm_addto = counting
    try:
        pop.apply_update(seeds, coefs, lr)
    finally:
        K.gemm_addto = orig
    assert (calls["n"] > 0) == (n_pairs == 8)
    oz = OracleZO([h.copy() for h in host], [__import__("oracle.philox", fromlist=["x"]).BF16] * len(host), _cfg(),
                  noise="c", semantics="cuda")
    delta = [np.zeros_like(h, dtype=np.float64) for h in host]
    mag = [np.zeros_like(h, dtype=np.float64) for h in host]
    for s, c in zip(seeds, coefs):
        for d, m_, z in zip(delta, mag, oz.sample_z(s)):
            d += c * z.astype(np.float64)
            m_ += abs(c) * np.abs(z.astype(np.float64))
    for (name, p), h, d, m_ in zip(named, host, delta, mag):
        got = p.detach().float().cpu().numpy()
        want = h - lr * d
        ulp = np.ldexp(1.0, np.frexp(np.maximum(np.abs(want), 2.0 ** -126))[1] - 8)
        err = np.abs(got - want)
        bound = ulp + 2.0 ** -6 * lr * m_ + 1e-12
        assert (err <= bound).all(), (name, float((err / bound).max()))
        assert not np.array_equal(got, h), name


def test_es_step_single_rank():
    from toy_models import build_llama
    from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
    g = torch.Generator().manual_seed(9)
    tokens = torch.randint(0, SHAPE["vocab_size"], (4, 64), generator=g).cuda()
    model = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    pop = EggrollPopulation(model, EggrollConfig(sigma=SIGMA))
    before = [p.detach().clone() for _, p in pop.named]
    m = pop.step(tokens, [1, 2, 3, 4, 5, 6], lr=1e-3, strategy="centered_rank", chunk_pairs=4)
    assert m["members"] == 12 and np.isfinite(m["loss"]) and m["fit_rms"] > 0
    assert any(not torch.equal(b, p) for b, (_, p) in zip(before, pop.named))
    from zotitan_b200 import kernels as K
    assert K.eggroll_take_error() == 0


def test_cuda_graph_replay_matches_eager():
    """cuda_graphs: the first chunk of a shape is captured, later chunks replay it with new
    pair seeds (device memory) and new tokens. Every replayed result is bit-identical to
    the eager forward of the same chunk (same kernels, same order)."""
    from toy_models import build_llama
    from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
    g = torch.Generator().manual_seed(9)
    toks = [torch.randint(0, SHAPE["vocab_size"], (4, 64), generator=g).cuda() for _ in range(3)]
    seeds = [[3, 11], [5, 2**63 + 7], [2**64 - 1, 0]]
    model = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    graphed = EggrollPopulation(model, EggrollConfig(sigma=SIGMA, cuda_graphs=True))
    got = [graphed.evaluate(t, s).clone() for t, s in zip(toks, seeds)]
    assert len(graphed._graphs) == 1
    model2 = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    eager = EggrollPopulation(model2, EggrollConfig(sigma=SIGMA, cuda_graphs=False))
    want = [eager.evaluate(t, s) for t, s in zip(toks, seeds)]
    for a, b in zip(got, want):
        assert torch.equal(a, b), (a, b)
    assert not torch.equal(got[0], got[1])


def test_device_seed_keys_match_host_keys():
    """zt_eggroll_factors / zt_eggroll_rmsnorm with keys derived on the device from pair
    seeds equal the calls given the host-computed keys."""
    from zotitan_b200 import kernels as K
    from zotitan_b200.eggroll import _key
    n_params, idx = 291, 17
    seeds_list = [1, 2**40 + 3, 2**64 - 5]
    seeds = torch.tensor([s - 2**64 if s >= 2**63 else s for s in seeds_list], dtype=torch.int64, device="cuda")
    ka = [_key(s, n_params, idx + 2 * n_params) for s in seeds_list]
    kb = [_key(s, n_params, idx + n_params) for s in seeds_list]
    host = K.eggroll_factors(ka, kb, 384, 256, 1e-3, "cuda", ext_slot=0)
    dev = K.eggroll_factors(None, None, 384, 256, 1e-3, "cuda", ext_slot=0,
                            dev_seeds=(seeds, n_params, idx + 2 * n_params, idx + n_params))
    for h, d in zip(host, dev):
        assert torch.equal(h, d)
    x = torch.randn(6 * 128, 256, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(256, device="cuda")).bfloat16()
    yh = K.eggroll_rmsnorm(x, w, [_key(s, n_params, idx) for s in seeds_list], 1e-2, 1e-5, 128)
    yd = K.eggroll_rmsnorm(x, w, None, 1e-2, 1e-5, 128, dev_seeds=(seeds, n_params, idx))
    assert torch.equal(yh, yd)
