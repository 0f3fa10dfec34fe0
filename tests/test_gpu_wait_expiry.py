"""The bounded-wait abort path of the tcgen05 GEMMs, exercised without a fault.

Every mbarrier wait in the fused cross-entropy GEMM (zt_linear_xent) and the EGGROLL GEMMs
(zt_eggroll_linear) gives up after a clock deadline: the kernel then records an error
code, raises both CTAs' abort flags, drains its own copies and MMAs, frees its tensor
memory and returns. The same holds for the fused low-rank GEMM (zt_lowrank_apply). The test hook
`test_stall_loads` makes the loader issue no copies, so
the first wait for a loaded stage expires with no copy and no MMA in flight (nothing to
drain). The tests check that the call reports the expiry through the take-error entry
point, that the context stays usable, and that the next normal call is correct.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def test_linear_xent_wait_expiry_reported_and_context_usable():
    from zotitan_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(512, 256, device="cuda", generator=g).bfloat16()
    w = (torch.randn(1024, 256, device="cuda", generator=g) * 0.02).bfloat16()
    t = torch.randint(0, 1024, (512,), device="cuda", generator=g)
    assert K.linear_xent_take_error() == 0
    K.linear_xent(x, w, t, test_stall_loads=True, test_wait_cycles=2_000_000)   # ~1 ms per wait
    torch.cuda.synchronize()
    code = K.linear_xent_take_error()
    assert code in (3, 4)          # the MMA issuer's wait for a loaded stage, or the epilogue's
    assert K.linear_xent_take_error() == 0                                     # cleared
    loss, lse, correct = K.linear_xent(x, w, t)
    logits = F.linear(x, w).float()
    ref = torch.logsumexp(logits, -1) - logits.gather(1, t[:, None])[:, 0]
    torch.cuda.synchronize()
    assert K.linear_xent_take_error() == 0
    torch.testing.assert_close(loss, ref, rtol=1e-3, atol=1e-3)


def test_eggroll_gemm_wait_expiry_reported_and_context_usable():
    """The CTA-pair EGGROLL GEMM (rows a multiple of 256) with the default ~2 s bound."""
    from zotitan_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(4)
    M, N, Kd, T = 256, 256, 128, 256
    x = torch.randn(M, Kd, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, Kd, device="cuda", generator=g) * 0.02).bfloat16()
    a = torch.randn(1, N, 4, device="cuda", generator=g)
    b = torch.randn(1, Kd, 4, device="cuda", generator=g)
    sigma = torch.full((1,), 1e-3, device="cuda")
    assert K.eggroll_take_error() == 0
    K.eggroll_linear(x, w, a, b, sigma, T, test_stall_loads=True)
    torch.cuda.synchronize()
    assert K.eggroll_take_error() in (3, 4)
    y = K.eggroll_linear(x, w, a, b, sigma, T)
    ref = x.float() @ w.float().T + 1e-3 * ((x.float() @ b[0]) @ a[0].T)
    torch.cuda.synchronize()
    assert K.eggroll_take_error() == 0
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


def test_lowrank_gemm_wait_expiry_reported_and_context_usable():
    from zotitan_b200 import kernels as K
    f = K.LowRankFactors((512, 512), 64, torch.bfloat16, [3], [4], "cuda")
    theta = torch.zeros(512, 512, device="cuda", dtype=torch.bfloat16)
    assert K.lowrank_take_error() == 0
    f.apply(src=theta, dst=theta, alphas=(1.0,), test_stall_loads=True, test_wait_cycles=2_000_000)
    torch.cuda.synchronize()
    assert K.lowrank_take_error() in (1, 3, 4)   # a wait of the stage pipeline
    # the ragged-row kernel (rows not whole 16-byte groups) takes the same hook
    g = K.LowRankFactors((300, 300), 64, torch.bfloat16, [3], [4], "cuda")
    t3 = torch.zeros(300, 300, device="cuda", dtype=torch.bfloat16)
    g.apply(src=t3, dst=t3, alphas=(1.0,), test_stall_loads=True, test_wait_cycles=2_000_000)
    torch.cuda.synchronize()
    assert K.lowrank_take_error() in (1, 3, 4)
    assert K.lowrank_take_error() == 0
    z = f.directions()
    torch.cuda.synchronize()
    assert K.lowrank_take_error() == 0
    assert abs(float(z.float().norm()) - 512.0) <= 4.0     # ||z||_F = sqrt(m n)
