"""GPU parity of the EGGROLL population companions, through the C ABI.

- zt_eggroll_factors: A and B bit-exact with the noise source rounded to bf16 (the
  reference's `_philox_randn(...).view(...).to(p.dtype)`, zotitan/train_zo.py:308-314),
  duplicated for both members of a pair; the scale within one bf16 step of the low_rank
  normalisation evaluated on the rounded product (oracle restatement of :318-319).
- zt_eggroll_rmsnorm: transformers' LlamaRMSNorm applied member by member with weights
  w + sign*sigma*z; bar: >= 99% of outputs bit-exact, all within two bf16 steps (the row
  sum of squares is reduced in a different order, so the normalised row can differ by one
  bf16 step before the weight product, which is rounded again).
- zt_eggroll_rope: bit-exact with transformers' apply_rotary_pos_emb on bf16 tensors.
- zt_eggroll_swiglu: F.silu(g) * u on bf16 tensors; bar: >= 99.9% bit-exact, all within
  one bf16 step.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from zotitan_b200 import kernels as K  # noqa: E402


def _bf16_steps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of b's bf16 spacing."""
    a, b = a.float(), b.float()
    e = torch.frexp(b.abs().clamp_min(2.0**-126))[1].float()
    return (a - b).abs() / torch.ldexp(torch.ones_like(e), (e - 8).int())


@pytest.mark.parametrize("n,k,pairs", [(256, 512, 1), (1024, 256, 3), (4096, 14336, 8), (128256, 256, 2)])
def test_factors_match_noise_and_normalisation(n, k, pairs):
    seeds = [7 + 13 * j for j in range(pairs)]
    n_params, idx = 291, 17
    ka = [K.param_key(s, n_params, idx + 2 * n_params) for s in seeds]
    kb = [K.param_key(s, n_params, idx + n_params) for s in seeds]
    sigma = 1e-3
    a, b, scale = K.eggroll_factors(ka, kb, n, k, sigma, "cuda")
    torch.cuda.synchronize()
    P = K.randn_keys(ka, n * 4, "cuda").view(pairs, n, 4).bfloat16().float()
    Psi = K.randn_keys(kb, 4 * k, "cuda").view(pairs, 4, k).bfloat16().float()
    assert torch.equal(a[0::2], P) and torch.equal(a[1::2], P)
    Bt = Psi.transpose(1, 2).contiguous()
    assert torch.equal(b[0::2], Bt) and torch.equal(b[1::2], Bt)
    sc = scale.cpu().numpy()
    np.testing.assert_array_equal(sc[0::2], -sc[1::2])
    for j in range(pairs):
        z = (P[j].double() @ Psi[j].double()).float().bfloat16().double()
        r1 = lambda x: float(torch.tensor([x], dtype=torch.float32).bfloat16().float())  # noqa: E731
        norm = r1(float(np.float32(np.sqrt(float((z ** 2).sum())))))
        t = r1(float(np.float32(norm) + np.float32(1e-7)))
        c = r1(float(np.float32(np.float32(1.0) / np.float32(t)) * np.float32((n * k) ** 0.5)))
        want = np.float32(sigma) * np.float32(c)
        assert abs(sc[2 * j] - want) <= abs(want) * 2.0**-7, (j, sc[2 * j], want)


def test_factors_unnormalised_scale_is_sigma():
    a, b, scale = K.eggroll_factors([5, 6], [7, 8], 256, 128, 0.25, "cuda", normalize=False)
    assert scale.cpu().tolist() == [0.25, -0.25, 0.25, -0.25]


@pytest.mark.parametrize("d,pairs,rows_per_member", [(256, 1, 128), (4096, 3, 256), (2048, 2, 384)])
def test_rmsnorm_matches_llama_rmsnorm_per_member(d, pairs, rows_per_member):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm
    g = torch.Generator(device="cuda").manual_seed(d + pairs)
    x = (torch.randn(2 * pairs * rows_per_member, d, device="cuda", generator=g) * 3).bfloat16()
    w = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    keys = [K.param_key(s, 50, 3) for s in range(11, 11 + pairs)]
    sigma, eps = 0.05, 1e-5
    y = K.eggroll_rmsnorm(x, w, keys, sigma, eps, rows_per_member)
    norm = LlamaRMSNorm(d, eps=eps).cuda().bfloat16()
    want = torch.empty_like(x)
    z = K.randn_keys(keys, d, "cuda").double()
    for m in range(2 * pairs):
        sgn = 1.0 if m % 2 == 0 else -1.0
        wm = (w.double() + (sgn * np.float32(sigma)) * z[m // 2]).float().bfloat16()
        with torch.no_grad():
            norm.weight.copy_(wm)
            rows = slice(m * rows_per_member, (m + 1) * rows_per_member)
            want[rows] = norm(x[rows])
    steps = _bf16_steps(y, want)
    assert float(steps.max()) <= 2.0
    assert float((steps == 0).float().mean()) >= 0.99


@pytest.mark.parametrize("hq,hk,hd,seq,batch", [(32, 8, 128, 256, 3), (4, 4, 64, 64, 2), (8, 2, 16, 48, 1)])
def test_rope_matches_transformers(hq, hk, hd, seq, batch):
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    g = torch.Generator(device="cuda").manual_seed(hq * hd + seq)
    q = torch.randn(batch, seq, hq * hd, device="cuda", generator=g).bfloat16()
    k = torch.randn(batch, seq, hk * hd, device="cuda", generator=g).bfloat16()
    inv = 1.0 / (10000 ** (torch.arange(0, hd, 2, device="cuda").float() / hd))
    f = torch.arange(seq, device="cuda").float()[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    cos, sin = emb.cos().bfloat16(), emb.sin().bfloat16()
    qh = q.view(batch, seq, hq, hd).transpose(1, 2)
    kh = k.view(batch, seq, hk, hd).transpose(1, 2)
    want_q, want_k = apply_rotary_pos_emb(qh, kh, cos[None], sin[None])
    q2, k2 = q.clone(), k.clone()
    K.eggroll_rope_(q2, k2, cos.contiguous(), sin.contiguous(), seq, hd)
    assert torch.equal(q2.view(batch, seq, hq, hd).transpose(1, 2), want_q)
    assert torch.equal(k2.view(batch, seq, hk, hd).transpose(1, 2), want_k)


@pytest.mark.parametrize("shape", [(8,), (1000, 56), (4096, 14336)])
def test_swiglu_matches_torch(shape):
    g = torch.Generator(device="cuda").manual_seed(len(shape))
    gate = (torch.randn(*shape, device="cuda", generator=g) * 4).bfloat16()
    up = torch.randn(*shape, device="cuda", generator=g).bfloat16()
    y = K.eggroll_swiglu(gate, up)
    want = torch.nn.functional.silu(gate) * up
    steps = _bf16_steps(y, want)
    assert float(steps.max()) <= 1.0
    assert float((steps == 0).float().mean()) >= 0.999
