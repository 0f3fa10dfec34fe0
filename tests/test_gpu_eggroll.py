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


def _steps(a, b):
    a, b = a.float(), b.float()
    e = torch.frexp(b.abs().clamp_min(2.0 ** -126))[1].float()
    return (a - b).abs() / torch.ldexp(torch.ones_like(e), (e - 8).int())


def test_ksliced_factor_and_xb_rows():
    """A_ext rows are the bf16 factors in the documented slots; X_ext rows hold
    hi + lo = sigma_i X B_i to ~2^-16 relative."""
    from zotitan_b200 import kernels as K_
    n, k, T = 512, 1024, 256
    keys_a, keys_b = [11, 12], [21, 22]
    a, b, sc, ae0 = K_.eggroll_factors(keys_a, keys_b, n, k, 1e-3, "cuda", ext_slot=0)
    _, _, _, ae1 = K_.eggroll_factors(keys_a, keys_b, n, k, 1e-3, "cuda", ext_slot=1)
    ab = a.bfloat16()
    assert torch.equal(ae0[..., 0:4], ab) and torch.equal(ae0[..., 4:8], ab) and not ae0[..., 8:].any()
    assert torch.equal(ae1[..., 8:12], ab) and torch.equal(ae1[..., 12:16], ab) and not ae1[..., :8].any()
    x = torch.randn(4 * T, k, device="cuda").bfloat16()
    xb = K_.eggroll_xb(x, [b], T)[0]
    xe = K_.eggroll_xb_ext(x, [b], [sc], [0], T)[0]
    want = xb * sc.repeat_interleave(T)[:, None]
    got = xe[:, 0:4].float() + xe[:, 4:8].float()
    assert float(((got - want).abs() / want.abs().clamp_min(1e-30)).max()) < 2 ** -15
    assert not xe[:, 8:].any()
    g1, g2 = K_.eggroll_xb_ext(x, [b, b], [sc, sc], [1, 2], T)
    assert g1.data_ptr() == g2.data_ptr() and torch.equal(g1[:, 0:8], xe[:, 0:8]) and torch.equal(g1[:, 8:], xe[:, 0:8])


@pytest.mark.parametrize("M,N,K,T,sigma", [(512, 1024, 1024, 256, 1e-3), (2048, 4096, 4096, 1024, 1e-3),
                                           (512, 1024, 1024, 256, 5e-2)])
def test_ksliced_linear_matches_fp32_epilogue(M, N, K, T, sigma):
    """The rank-4 term as a tensor-core K-slab against the fp32 epilogue. The slab carries
    sigma X B as hi + lo bf16 (~2^-16 relative), so the outputs agree within one bf16 step
    plus 2^-14 of the term's magnitude sum_r |sigma X B_r| |A_r| (absolute: where the term
    cancels the base product the output is small and the bound is loose in bf16 steps)."""
    from zotitan_b200 import kernels as K_
    g = torch.Generator(device="cuda").manual_seed(M + K)
    members = M // T
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    a, b, sc, ae = K_.eggroll_factors(list(range(1, members // 2 + 1)), list(range(50, 50 + members // 2)), N, K,
                                      sigma, "cuda", ext_slot=0)
    y32 = K_.eggroll_linear(x, w, a, b, sc, T)
    xe = K_.eggroll_xb_ext(x, [b], [sc], [0], T)[0]
    yk = K_.eggroll_linear(x, w, a, None, sc, T, x_ext=xe, w_ext=ae)
    xb = K_.eggroll_xb(x, [b], T)[0]
    torch.cuda.synchronize()
    assert K_.eggroll_take_error() == 0
    sxb = (xb * sc.repeat_interleave(T)[:, None]).abs()
    term = torch.cat([sxb[i * T:(i + 1) * T] @ a[i].abs().T for i in range(members)])
    ulp = torch.ldexp(torch.ones_like(y32.float()), (torch.frexp(y32.float().abs().clamp_min(2.0 ** -126))[1] - 8).int())
    d = (yk.float() - y32.float()).abs()
    assert bool((d <= ulp + 2.0 ** -14 * term).all()), float((d - ulp - 2.0 ** -14 * term).max())
    if sigma <= 1e-3:
        assert float((d == 0).float().mean()) >= 0.99
    assert not torch.equal(y32, (x.float() @ w.float().T).bfloat16())   # the term is applied


def test_ksliced_gated_matches_fp32_epilogue():
    from zotitan_b200 import kernels as K_
    M, N, K, T = 1024, 1408, 1024, 512
    g = torch.Generator(device="cuda").manual_seed(77)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    wu = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    fg = K_.eggroll_factors([3], [4], N, K, 1e-3, "cuda", ext_slot=0)
    fu = K_.eggroll_factors([5], [6], N, K, 1e-3, "cuda", ext_slot=1)
    xbg, xbu = K_.eggroll_xb(x, [fg[1], fu[1]], T)
    y32 = K_.eggroll_gated(x, wg, wu, fg, fu, xbg, xbu, T)
    xe = K_.eggroll_xb_ext(x, [fg[1], fu[1]], [fg[2], fu[2]], [1, 2], T)[0]
    yk = K_.eggroll_gated(x, wg, wu, fg, fu, None, None, T, x_ext=xe)
    torch.cuda.synchronize()
    assert K_.eggroll_take_error() == 0
    d = (yk.float() - y32.float()).abs()
    assert bool((d <= 2.0 ** -7 * y32.float().abs() + 1e-3 * y32.float().abs().max()).all())
    assert float((d == 0).float().mean()) >= 0.98


@pytest.mark.parametrize("M,K,T,nseg", [(512, 1024, 256, 3), (2048, 4096, 1024, 2), (256, 128, 128, 1)])
def test_tensor_core_xb_matches_cuda_core_xb(M, K, T, nseg):
    """X B on the tensor cores (B^T in bf16 from the factor kernel) against the CUDA-core pass:
    fp32 accumulations of the same exact products in different orders (relative 1e-5 of
    sum |x||b|); the K-slab rows it writes agree to ~2^-15."""
    from zotitan_b200 import kernels as K_
    members = M // T
    bt = torch.zeros((members, 16, K), dtype=torch.bfloat16, device="cuda")
    facs = [K_.eggroll_factors(list(range(s * 10 + 1, s * 10 + 1 + members // 2)),
                               list(range(s * 10 + 50, s * 10 + 50 + members // 2)), 256, K, 1e-3, "cuda",
                               ext_slot=0, b_ext=bt, b_ext_row=4 * s) for s in range(nseg)]
    for s, f in enumerate(facs):
        assert torch.equal(bt[:, 4 * s:4 * s + 4, :].float(), f[1].transpose(1, 2))
    assert not bt[:, 4 * nseg:, :].any()
    x = torch.randn(M, K, device="cuda").bfloat16()
    ref = K_.eggroll_xb(x, [f[1] for f in facs], T)
    xes_cc = K_.eggroll_xb_ext(x, [f[1] for f in facs], [f[2] for f in facs], [0] * nseg, T)
    xes_tc = K_.eggroll_xb_ext(x, [f[1] for f in facs], [f[2] for f in facs], [0] * nseg, T, bt=bt)
    torch.cuda.synchronize()
    assert K_.eggroll_take_error() == 0
    for f, r, a_, b_ in zip(facs, ref, xes_cc, xes_tc):
        scale = float((x.float().abs() @ f[1].abs().amax(0)).amax())
        v_cc = a_[:, 0:4].float() + a_[:, 4:8].float()
        v_tc = b_[:, 0:4].float() + b_[:, 4:8].float()
        sig = f[2].repeat_interleave(T)[:, None].abs()
        assert float((v_tc - v_cc).abs().max()) <= 1e-5 * scale * float(sig.max()) + 2 ** -14 * float(v_cc.abs().max())
        assert not b_[:, 8:].any()


@pytest.mark.parametrize("M,N,K", [(256, 128, 64), (512, 384, 256), (2048, 1408, 1024), (8192, 8192, 2048)])
def test_gemm_swiglu_matches_torch(M, N, K):
    """zt_gemm_swiglu (the plain pair GEMM, no rank-4 term, SwiGLU in the epilogue) against
    torch's gate / up GEMMs and F.silu(g) * u on bf16: the same rounding points, so the
    outputs differ only where the two GEMMs' fp32 accumulation orders put g or u on
    different sides of a bf16 rounding boundary (>= 99% identical, within 2^-6 relative
    plus 1e-3 absolute)."""
    from zotitan_b200 import kernels as K_
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(N, K, device="cuda", generator=g) * K ** -0.5).bfloat16()
    wu = (torch.randn(N, K, device="cuda", generator=g) * K ** -0.5).bfloat16()
    y = K_.gemm_swiglu(x, wg, wu)
    want = torch.nn.functional.silu(x @ wg.T) * (x @ wu.T)
    torch.cuda.synchronize()
    assert K_.eggroll_take_error() == 0
    d = (y.float() - want.float()).abs()
    assert bool((d <= 2 ** -6 * want.float().abs() + 1e-3).all()), float(d.max())
    assert float((d == 0).float().mean()) >= 0.99


def test_gemm_swiglu_rejects_bad_shapes():
    from zotitan_b200 import kernels as K_
    from zotitan_b200._lib import ZtError
    x = torch.zeros(200, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(128, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ZtError):
        K_.gemm_swiglu(x, w, w)   # 200 rows: not whole 256-row tiles


@pytest.mark.parametrize("m,n,k", [(512, 256, 128), (1000, 96, 64), (1024, 4096, 4096), (4096, 4096, 512)])
def test_gemm_addto_matches_fp32_reference(m, n, k):
    """zt_gemm_addto: w <- bf16(w + alpha a b^T) against the fp32 product added to w and
    rounded once in torch: equal, or one bf16 step apart where the fp32 sums of the two
    accumulation orders straddle a rounding boundary (rare)."""
    from zotitan_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    w = (torch.randn(m, n, device="cuda", generator=g) * 0.02).bfloat16()
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    b = torch.randn(n, k, device="cuda", generator=g).bfloat16()
    alpha = -1e-3
    exact = w.double() + alpha * (a.double() @ b.double().T)
    want = exact.float().bfloat16()
    got = K.gemm_addto(w.clone(), a, b, alpha)
    torch.cuda.synchronize()
    assert K.gemm_take_error() == 0
    diff = (got.double() - exact).abs()
    # one bf16 step of the result, plus the fp32 accumulation error of the product term
    # (where w and the term nearly cancel the result's own step is smaller than that)
    step = torch.ldexp(torch.ones_like(diff), torch.frexp(exact.abs().clamp_min(2.0 ** -126))[1] - 8)
    bound = step + abs(alpha) * 2.0 ** -20 * (a.double().abs() @ b.double().abs().T)
    assert bool((diff <= bound).all()), float((diff / bound).max())
    assert float((got != want).float().mean()) < 0.01
    assert not torch.equal(got, w)


def test_gemm_addto_rejects_bad_shapes():
    from zotitan_b200 import _lib as L
    lib = L.load()
    w = torch.zeros(256, 96, dtype=torch.bfloat16, device="cuda")
    a = torch.zeros(256, 64, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(96, 64, dtype=torch.bfloat16, device="cuda")
    assert lib.zt_gemm_addto(w.data_ptr(), 96, a.data_ptr(), b.data_ptr(), 1.0, 256, 96, 48, None) == L.ZT_ERR_INVALID
    assert lib.zt_gemm_addto(w.data_ptr(), 96, a.data_ptr(), b.data_ptr(), 1.0, 256, 80, 64, None) == L.ZT_ERR_INVALID
    assert lib.zt_gemm_addto(w.data_ptr(), 90, a.data_ptr(), b.data_ptr(), 1.0, 256, 96, 64, None) == L.ZT_ERR_INVALID
