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


@pytest.mark.parametrize("M,N,K,T", [(256, 512, 128, 128), (2048, 4096, 512, 512), (512, 256, 4096, 256),
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
