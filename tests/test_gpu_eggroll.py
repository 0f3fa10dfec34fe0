"""EGGROLL population linear layer (tcgen05 GEMM + rank-4 epilogue) vs a torch fp32
reference of the same formula: Y = X W^T + sigma_i (X B_i) A_i^T per member.

Tolerance: the output is bf16 (8 significant bits), so |Y - ref| <= 8e-3 |ref| plus
1e-3 of the largest |ref| for entries near zero; accumulation-order differences
between the tensor cores and the fp32 reference are far below that.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def reference(x, w, a, b, sigma, T):
    xf, wf = x.float(), w.float()
    y = xf @ wf.T
    members = x.shape[0] // T
    for i in range(members):
        r = slice(i * T, (i + 1) * T)
        y[r] += sigma[i] * ((xf[r] @ b[i]) @ a[i].T)
    return y


@pytest.mark.parametrize("M,N,K,T", [(256, 512, 128, 128), (2048, 4096, 512, 512), (512, 256, 4096, 256), (384, 512, 256, 128),
                                     (1024, 1024, 1024, 1024)])
def test_eggroll_linear_matches_reference(M, N, K, T):
    from zotitan_b200 import kernels as K_
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    members = M // T
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    a = torch.randn(members, N, 4, device="cuda", generator=g)
    b = torch.randn(members, K, 4, device="cuda", generator=g)
    sigma = torch.randn(members, device="cuda", generator=g) * 1e-2
    y = K_.eggroll_linear(x, w, a, b, sigma, T)
    torch.cuda.synchronize()
    assert K_.eggroll_take_error() == 0
    ref = reference(x, w, a, b, sigma, T)
    err = (y.float() - ref).abs()
    bound = 8e-3 * ref.abs() + 1e-3 * ref.abs().max()
    assert bool((err <= bound).all()), float((err / (ref.abs() + 1e-6)).max())
    # the rank-4 term is really applied: a zero sigma gives the plain GEMM
    y0 = K_.eggroll_linear(x, w, a, b, torch.zeros_like(sigma), T)
    ref0 = x.float() @ w.float().T
    assert bool(((y0.float() - ref0).abs() <= 8e-3 * ref0.abs() + 1e-3 * ref0.abs().max()).all())
    assert not torch.equal(y0, y)


def test_eggroll_rejects_bad_shapes():
    from zotitan_b200 import _lib as L
    from zotitan_b200 import kernels as K_
    x = torch.zeros(128, 100, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(256, 100, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(L.ZtError, match="K % 64"):
        K_.eggroll_linear(x, w, torch.zeros(1, 256, 4, device="cuda"), torch.zeros(1, 100, 4, device="cuda"),
                          torch.zeros(1, device="cuda"), 128)


@pytest.mark.parametrize("M,K,T,nseg", [(256, 4096, 128, 3), (1024, 14336, 512, 1), (512, 4100, 256, 2),
                                        (128, 64, 64, 3)])
def test_shared_xb_matches_reference_and_single_set(M, K, T, nseg):
    """zt_eggroll_xb: X B_s for several factor sets in one read of X, within fp32
    accumulation-order error of the fp64 product; each set's result is bit-identical to the
    single-set pass that zt_eggroll_linear runs internally (same per-set accumulation order)."""
    from zotitan_b200 import kernels as K_
    g = torch.Generator(device="cuda").manual_seed(M + K + nseg)
    members = M // T
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    bs = [torch.randn(members, K, 4, device="cuda", generator=g) for _ in range(nseg)]
    xbs = K_.eggroll_xb(x, bs, T)
    for b, xb in zip(bs, xbs):
        ref = torch.cat([x[i * T:(i + 1) * T].double() @ b[i].double() for i in range(members)])
        scale = (x.double().abs() @ b.abs().double().amax(0)).amax()
        assert float((xb.double() - ref).abs().max()) <= 1e-5 * float(scale)
        single = K_.eggroll_xb(x, [b], T)[0]
        assert torch.equal(single, xb)


def test_linear_with_precomputed_xb_is_identical():
    from zotitan_b200 import kernels as K_
    M, N, K, T = 512, 1024, 2048, 256
    g = torch.Generator(device="cuda").manual_seed(11)
    members = M // T
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    ws = [(torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16() for _ in range(3)]
    as_ = [torch.randn(members, N, 4, device="cuda", generator=g) for _ in range(3)]
    bs = [torch.randn(members, K, 4, device="cuda", generator=g) for _ in range(3)]
    sigma = torch.randn(members, device="cuda", generator=g) * 1e-2
    xbs = K_.eggroll_xb(x, bs, T)
    for w, a, b, xb in zip(ws, as_, bs, xbs):
        y_shared = K_.eggroll_linear(x, w, a, None, sigma, T, xb=xb, xb_ready=True)
        y_own = K_.eggroll_linear(x, w, a, b, sigma, T)
        assert torch.equal(y_shared, y_own)
    torch.cuda.synchronize()
    assert K_.eggroll_take_error() == 0


@pytest.mark.parametrize("M,N,K,T", [(512, 256, 512, 256), (1024, 1408, 1024, 512)])
def test_gated_pair_matches_unfused_path(M, N, K, T):
    """zt_eggroll_gated (gate and up in one pair GEMM, SwiGLU in the epilogue) against two
    EGGROLL linears and zt_eggroll_swiglu: the same rounding steps, so outputs agree to the
    bit except where the two GEMMs' accumulation orders differ (at most one bf16 step)."""
    from zotitan_b200 import kernels as K_
    g = torch.Generator(device="cuda").manual_seed(M + N)
    members = M // T
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    wu = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    fg = (torch.randn(members, N, 4, device="cuda", generator=g), torch.randn(members, K, 4, device="cuda", generator=g),
          torch.randn(members, device="cuda", generator=g) * 1e-2)
    fu = (torch.randn(members, N, 4, device="cuda", generator=g), torch.randn(members, K, 4, device="cuda", generator=g),
          torch.randn(members, device="cuda", generator=g) * 1e-2)
    xbg, xbu = K_.eggroll_xb(x, [fg[1], fu[1]], T)
    y = K_.eggroll_gated(x, wg, wu, fg, fu, xbg, xbu, T)
    if N % 256 == 0:
        gate = K_.eggroll_linear(x, wg, fg[0], None, fg[2], T, xb=xbg, xb_ready=True)
        up = K_.eggroll_linear(x, wu, fu[0], None, fu[2], T, xb=xbu, xb_ready=True)
        want = K_.eggroll_swiglu(gate, up)
    else:  # torch evaluation of the same rounding chain
        def lin(w, f, xb):
            y_ = x.float() @ w.float().T
            for i in range(members):
                r = slice(i * T, (i + 1) * T)
                y_[r] += f[2][i] * (xb[r] @ f[0][i].T)
            return y_.bfloat16()
        want = K_.eggroll_swiglu(lin(wg, fg, xbg), lin(wu, fu, xbu))
    torch.cuda.synchronize()
    assert K_.eggroll_take_error() == 0
    d = (y.float() - want.float()).abs()
    tol = 2 ** -7 * want.float().abs() + 1e-6 if N % 256 == 0 else 2 ** -6 * want.float().abs() + 1e-3
    assert bool((d <= tol).all()), float(d.max())
    if N % 256 == 0:
        assert float((d == 0).float().mean()) >= 0.999
