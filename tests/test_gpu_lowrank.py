"""low_rank and polar MeZO perturbations (zotitan/train_zo.py:304-320) on the GPU.

2-D tensors take directions materialised with the reference's own ops (P, Psi from the
noise source, cast to the parameter dtype, z = P @ Psi scaled to ||z||_F = sqrt(numel));
1-D tensors keep the fused Gaussian passes; the fused pass then applies the optimizer
stages to the accumulated estimate. Checked against the reference's recorded low_rank run
(golden `lowrank_f32_z2`, rank 2, z_batch 2, fp32) with the fp32 bars of the Gaussian
golden test (8 ulp at scale or 2e-8 absolute: the reference ran its noise under Triton's
CPU interpreter, up to 4 ulp from the device, and its matmul on the CPU).
"""
import numpy as np
import pytest
import torch

from helpers import StepCase, scale_ulps, step_cases
from oracle import philox as ph
from test_gpu_step import run_gpu

pytestmark = pytest.mark.gpu
_G, _ = step_cases()


def test_low_rank_step_vs_reference_golden():
    case = StepCase(_G, "lowrank_f32_z2")
    a_gpu, metrics, snaps = run_gpu(case)
    dts = np.concatenate([[d] * n for d, n in zip(case.dtypes, case.numels)])
    assert not (dts == ph.BF16).any()
    for got, ref in ((snaps[0], case.snap_pos), (snaps[1], case.snap_neg)):
        u = scale_ulps(got, ref, case.init, dts)
        assert np.all((u <= 8) | (np.abs(got.astype(np.float64) - ref) <= 2e-8)), float(u.max())
    u = scale_ulps(a_gpu[0], case.after[0], case.init, dts)
    absd = np.abs(a_gpu[0].astype(np.float64) - case.after[0])
    assert np.all((u <= 8) | (absd <= 2e-8)), float(absd.max())
    assert abs(metrics[0]["loss"] - case.metrics[0]["loss"]) <= 1e-6 * abs(case.metrics[0]["loss"])
    assert not np.array_equal(a_gpu[0], case.init)


def test_polar_direction_is_orthogonal_and_normalised():
    """polar: P from QR (orthonormal columns), Psi from the Newton-Schulz polar iteration
    (rows near-orthonormal), z scaled to ||z||_F = sqrt(numel); a step with it runs."""
    from zotitan_b200.objective import Score
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer, zeropower_via_newtonschulz
    g = torch.Generator(device="cuda").manual_seed(3)
    G = torch.randn(8, 256, device="cuda", generator=g)
    X = zeropower_via_newtonschulz(G).float()
    sv = torch.linalg.svdvals(X)
    assert float(sv.min()) > 0.5 and float(sv.max()) < 1.5          # polar factor, bf16 iteration
    ps = [torch.nn.Parameter(torch.randn(64, 96, device="cuda", generator=g) * 0.02),
          torch.nn.Parameter(torch.ones(64, device="cuda"))]
    cfg = ZOConfig()
    cfg.eps, cfg.z_batch, cfg.base.lr = 1e-3, 2, 1e-2
    cfg.perturbation.distribution, cfg.perturbation.rank = "polar", 4
    vals = iter([1.0, 0.5, 0.25, 0.75])
    opt = ZOOptimizer([("w", ps[0]), ("n", ps[1])], cfg, lambda m, b: Score(torch.tensor(next(vals), device="cuda"), {}))
    z = opt._lowrank_z(7)[0]
    z = z.directions()[0] if hasattr(z, "directions") else z     # fused (fp32 polar) or materialised
    assert abs(float(z.norm()) - (64 * 96) ** 0.5) <= 1e-3 * (64 * 96) ** 0.5
    w0, n0 = ps[0].detach().clone(), ps[1].detach().clone()
    m = opt.step(None, [None, None])
    assert np.isfinite(m["loss"]) and not torch.equal(w0, ps[0]) and not torch.equal(n0, ps[1])


@pytest.mark.parametrize("dist_kind", ["low_rank", "polar"])
def test_sharded_low_rank_matches_single_gpu(dist_kind):
    """The seed-sharded schedule with materialised directions (one-rank NCCL group): each
    own pair perturbs the live copy from the master, the last pass replays every pair's
    +eps / -2eps / +eps chain on the master (the 2-D tensors with the reference's ops, the
    1-D ones in the fused pass) and updates it; the parameters equal the single-GPU run's
    exactly, and the forwards see master + eps z."""
    import os

    import torch.distributed as dist
    from zotitan_b200.objective import Score
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer

    # bf16 for low_rank; fp32 for polar, whose QR (torch.linalg.qr) has no bf16 CUDA kernel,
    # so the reference's own polar branch runs only on fp32 parameters on a GPU
    dt = torch.bfloat16 if dist_kind == "low_rank" else torch.float32

    def run(sharded):
        g = torch.Generator(device="cuda").manual_seed(11)
        ps = [torch.nn.Parameter((torch.randn(48, 80, device="cuda", generator=g) * 0.02).to(dt)),
              torch.nn.Parameter(torch.ones(48, device="cuda").to(dt)),
              torch.nn.Parameter((torch.randn(80, 48, device="cuda", generator=g) * 0.02).to(dt))]
        cfg = ZOConfig()
        cfg.eps, cfg.z_batch, cfg.base.lr = 1e-3, 3, 5e-2
        cfg.perturbation.distribution, cfg.perturbation.rank = dist_kind, 4
        vals = iter([2.0, 1.9, 2.1, 2.15, 1.8, 1.75, 2.2, 2.3, 2.05, 1.95, 2.0, 2.12])
        opt = ZOOptimizer([(f"p{i}", p) for i, p in enumerate(ps)], cfg,
                          lambda m, b: Score(torch.tensor(next(vals), device="cuda"), {}), sharded=sharded)
        for _ in range(2):
            opt.step(None, [None] * 3)
        torch.cuda.synchronize()
        return [p.detach().float().cpu().numpy() for p in ps], opt

    a1, _ = run(False)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = "29541"
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        aw, opt = run(True)
        assert opt.planner.sharded and opt.lr_idx == [0, 2] and opt.master is not None
        for x, y in zip(a1, aw):
            assert np.array_equal(x, y)
        for m, p in zip(opt.master, opt.params):
            assert torch.equal(m, p)
    finally:
        dist.destroy_process_group()
