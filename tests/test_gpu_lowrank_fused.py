"""Fused low-rank directions (zt_lowrank_prepare / zt_lowrank_apply) against the
reference's materialised ops (zotitan/train_zo.py:304-320).

The reference builds z = P @ Psi with a library GEMM and scales it by torch scalar ops.
The fused kernels recompute z on the tensor cores inside every use. Two facts are
checked separately:
- the direction: equal to the reference's materialised z except where the fp32 sum of
  the r products lies on a rounding boundary of the dtype (one unit in the last place,
  in a small fraction of elements), and the scale equal to torch's;
- the uses: given the kernel's own direction (read back with `directions()`), the
  chained parameter updates and the grad-estimate sums equal torch's foreach ops on it
  bit for bit (same roundings in the same order).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def torch_direction(m, n, r, dtype, kp, kpsi):
    """The reference's _sample_z for one 2-D tensor (:308-320), materialised."""
    from zotitan_b200.kernels import randn
    P = randn(kp, m * r, "cuda").view(m, r).to(dtype)
    Psi = randn(kpsi, r * n, "cuda").view(r, n).to(dtype)
    z = P @ Psi
    return z * ((m * n) ** 0.5 / (z.norm() + 1e-7)), P, Psi


def ulp_diff(a, b, dtype):
    """|a - b| in units of the dtype's last place at max(|a|, |b|)."""
    a64, b64 = a.double(), b.double()
    mag = torch.maximum(a64.abs(), b64.abs()).clamp_min(torch.finfo(dtype).tiny)
    ulp = torch.pow(2.0, torch.floor(torch.log2(mag)) - (7 if dtype == torch.bfloat16 else 10))
    return ((a64 - b64).abs() / ulp)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("m,n,r", [(256, 512, 64), (300, 520, 64), (1000, 2048, 8), (130, 96, 100), (48, 80, 4)])
def test_direction_matches_reference_ops(dt, m, n, r):
    from zotitan_b200 import kernels as K
    dtype = DT[dt]
    keys_p, keys_psi = [12345, 777, 99], [4242, 31, 2**31 - 5]
    f = K.LowRankFactors((m, n), r, dtype, keys_p, keys_psi, "cuda")
    got = f.directions()
    ref_scales = []
    for s in range(3):
        z_ref, P, Psi = torch_direction(m, n, r, dtype, keys_p[s], keys_psi[s])
        # the factors are the reference's, zero-padded in K
        assert torch.equal(f.p[s * m:(s + 1) * m, :r], P)
        assert torch.equal(f.psi_t[s * n:(s + 1) * n, :r], Psi.T)
        assert not f.p[s * m:(s + 1) * m, r:].any() and not f.psi_t[s * n:(s + 1) * n, r:].any()
        # the scale: torch's op sequence on the reference's product
        zr = (P @ Psi)
        scale_t = (m * n) ** 0.5 / (zr.norm() + 1e-7)
        ref_scales.append(float(scale_t))
        u = ulp_diff(got[s], z_ref, dtype)
        frac_exact = float((u == 0).double().mean())
        assert float(u.max()) <= 1.0, (s, float(u.max()))
        assert frac_exact >= 0.995, frac_exact
    sc = f.scale.cpu().tolist()
    for a, b in zip(sc, ref_scales):
        assert abs(a - b) <= abs(b) * (2 ** -7 if dtype == torch.bfloat16 else 2 ** -10), (a, b)
    torch.cuda.synchronize()
    assert K.lowrank_take_error() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("m,n", [(512, 768), (300, 520)])
def test_parameter_chain_and_grad_estimate_match_torch_ops(dt, m, n):
    """Three streams: theta <- round(theta + a z_s) for a in (eps, -2 eps, eps), stream by
    stream, and ge = round(c0 z0), ge <- round(ge + c_s z_s), equal to torch's foreach ops
    on the kernel's own directions; src != dst reads src once then dst."""
    from zotitan_b200 import kernels as K
    dtype = DT[dt]
    g = torch.Generator(device="cuda").manual_seed(5)
    theta = (torch.randn(m, n, device="cuda", generator=g) * 0.05).to(dtype)
    f = K.LowRankFactors((m, n), 64, dtype, [11, 12, 13], [21, 22, 23], "cuda")
    z = f.directions()
    eps = 1e-3
    coefs = [0.75, -1.25, 2.5e-3]
    ref = theta.clone()
    for s in range(3):
        for a in (eps, -2 * eps, eps):
            torch._foreach_add_([ref], [z[s]], alpha=a)
    ge_ref = torch.zeros_like(theta)
    for s in range(3):
        torch._foreach_add_([ge_ref], [z[s]], alpha=coefs[s])
    out = torch.empty_like(theta)
    ge = torch.full_like(theta, float("nan"))
    f.apply(src=theta, dst=out, alphas=(eps, -2 * eps, eps), ge=ge, coefs=coefs, ge_init=True)
    assert torch.equal(out, ref)
    assert torch.equal(ge, ge_ref)
    # in place, and accumulating into an existing estimate
    t2 = theta.clone()
    f.apply(src=t2, dst=t2, alphas=(eps,))
    ref2 = theta.clone()
    for s in range(3):
        torch._foreach_add_([ref2], [z[s]], alpha=eps)
    assert torch.equal(t2, ref2)
    f.apply(ge=ge, coefs=coefs)
    for s in range(3):
        torch._foreach_add_([ge_ref], [z[s]], alpha=coefs[s])
    assert torch.equal(ge, ge_ref)
    torch.cuda.synchronize()
    assert K.lowrank_take_error() == 0


def test_optimizer_low_rank_fused_against_materialised():
    """A MeZO step with low_rank directions through the fused kernels against the
    materialised path (the reference's ops), with the same pair values: the parameters
    equal up to the product's boundary roundings (rare, one or two bf16 units)."""
    from zotitan_b200.objective import Score
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer

    def run(fused, steps=2):
        g = torch.Generator(device="cuda").manual_seed(8)
        ps = [torch.nn.Parameter((torch.randn(256, 512, device="cuda", generator=g) * 0.02).bfloat16()),
              torch.nn.Parameter(torch.ones(512, device="cuda").bfloat16()),
              torch.nn.Parameter((torch.randn(384, 256, device="cuda", generator=g) * 0.02).bfloat16())]
        cfg = ZOConfig()
        cfg.eps, cfg.z_batch, cfg.base.lr = 1e-3, 3, 5e-2
        cfg.perturbation.distribution, cfg.perturbation.rank = "low_rank", 64
        vals = iter([2.0, 1.9, 2.1, 2.15, 1.8, 1.75, 2.2, 2.3, 2.05, 1.95, 2.0, 2.12])
        opt = ZOOptimizer([(f"p{i}", p) for i, p in enumerate(ps)], cfg,
                          lambda m, b: Score(torch.tensor(next(vals), device="cuda"), {}), lowrank_fused=fused)
        assert opt.lr_fused == ({0, 2} if fused else set())
        for _ in range(steps):
            opt.step(None, [None] * 3)
        torch.cuda.synchronize()
        return [p.detach().clone() for p in ps]

    a_f = run(True)
    a_m = run(False)
    for x, y in zip(a_f, a_m):
        u = ulp_diff(x, y, torch.bfloat16)
        assert float(u.max()) <= 2.0
        assert float((u == 0).double().mean()) >= 0.99


def test_fp32_low_rank_direction_close_to_reference_ops():
    """fp32 parameters: P and Psi split exactly into three bf16 parts each, the nine
    cross products summed on the tensor cores in fp32 (every product exact), so z is the
    fp32 product up to summation order; the scale in fp32 as torch computes it."""
    from zotitan_b200 import kernels as K
    m, n, r = 300, 520, 64
    keys_p, keys_psi = [12345, 777], [4242, 31]
    f = K.LowRankFactors((m, n), r, torch.float32, keys_p, keys_psi, "cuda")
    got = f.directions()
    for s in range(2):
        z_ref, _, _ = torch_direction(m, n, r, torch.float32, keys_p[s], keys_psi[s])
        torch.testing.assert_close(got[s], z_ref, rtol=2e-6, atol=2e-6)
    torch.cuda.synchronize()
    assert K.lowrank_take_error() == 0


def test_polar_fp32_direction_from_given_factors():
    """polar: the factors go through the reference's QR and Newton-Schulz (torch ops on the
    small m x r and r x n matrices); the product and its uses run fused. P is split into
    three bf16 parts, Psi (the bf16 iteration's output) is exact in bf16."""
    from zotitan_b200 import kernels as K
    from zotitan_b200.kernels import randn
    from zotitan_b200.train_zo import zeropower_via_newtonschulz
    m, n, r = 256, 384, 16
    P = randn(99, m * r, "cuda").view(m, r)
    P, _ = torch.linalg.qr(P)
    Psi = zeropower_via_newtonschulz(randn(98, r * n, "cuda").view(r, n))
    z = P @ Psi
    z_ref = z * ((m * n) ** 0.5 / (z.norm() + 1e-7))
    f = K.LowRankFactors.from_factors((m, n), [P], [Psi], torch.float32)
    got = f.directions()[0]
    torch.testing.assert_close(got, z_ref, rtol=2e-6, atol=2e-6)
    theta = torch.randn(m, n, device="cuda") * 0.02
    ref = theta.clone()
    for a in (1e-3, -2e-3, 1e-3):
        torch._foreach_add_([ref], [got], alpha=a)
    f.apply(src=theta, dst=theta, alphas=(1e-3, -2e-3, 1e-3))
    assert torch.equal(theta, ref)


@pytest.mark.parametrize("dist_kind", ["low_rank", "polar"])
def test_optimizer_fp32_fused_against_materialised(dist_kind):
    """fp32 low_rank and polar MeZO steps through the fused kernels against the reference's
    materialised ops with the same pair values. The tensor cores accumulate the split
    products in fp32 in their own order, so z differs from the library's fp32 GEMM by up to
    ~2e-6 of its scale (direction tests above). Here proj_grad is 50 and the update moves
    the parameters by O(1), so the bar is 1e-5 relative plus 4e-6 absolute."""
    from zotitan_b200.objective import Score
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer

    def run(fused):
        g = torch.Generator(device="cuda").manual_seed(8)
        ps = [torch.nn.Parameter(torch.randn(256, 512, device="cuda", generator=g) * 0.02),
              torch.nn.Parameter(torch.ones(512, device="cuda")),
              torch.nn.Parameter(torch.randn(384, 256, device="cuda", generator=g) * 0.02)]
        cfg = ZOConfig()
        cfg.eps, cfg.z_batch, cfg.base.lr = 1e-3, 3, 5e-2
        cfg.perturbation.distribution, cfg.perturbation.rank = dist_kind, 16
        vals = iter([2.0, 1.9, 2.1, 2.15, 1.8, 1.75, 2.2, 2.3, 2.05, 1.95, 2.0, 2.12])
        opt = ZOOptimizer([(f"p{i}", p) for i, p in enumerate(ps)], cfg,
                          lambda m, b: Score(torch.tensor(next(vals), device="cuda"), {}), lowrank_fused=fused)
        assert opt.lr_fused == ({0, 2} if fused else set())
        for _ in range(2):
            opt.step(None, [None] * 3)
        torch.cuda.synchronize()
        return [p.detach().clone() for p in ps]

    for x, y in zip(run(True), run(False)):
        torch.testing.assert_close(x, y, rtol=1e-5, atol=4e-6)
