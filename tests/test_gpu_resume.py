"""Exact resume (zotitan_b200.ZOOptimizer.state_dict / load_state_dict).

The reference loses its optimizer state at every checkpoint (zotitan/train_zo.py:671-673:
only the model is saved). Here a run interrupted after k steps, saved, and resumed in a
fresh optimizer over fresh parameter tensors ends bit-identical to the uninterrupted run:
the state is the seed counter, the step index, the seed window with its proj_grad history,
the clip history and the m / v / theta_0 buffers.
"""
import numpy as np
import pytest
import torch

from helpers import StepCase, flat, step_cases
from test_gpu_step import TDT, ReplayScore, run_gpu

pytestmark = pytest.mark.gpu
_G, _ = step_cases()


@pytest.mark.parametrize("name,k", [("seedwin_adam_bf16_z2", 2), ("ema_adam_f32_z2", 1), ("clip_norm_bf16", 2),
                                    ("wd_anchored_l1_bf16", 1)])
def test_resume_matches_uninterrupted_run(name, k):
    from zotitan_b200.train_zo import ZOOptimizer
    case = StepCase(_G, name)
    full, _, _ = run_gpu(case)
    Z, steps = case.cfg.z_batch, case.spec["steps"]
    ps = [torch.nn.Parameter(torch.from_numpy(p).to(TDT[d]).cuda()) for p, d in zip(case.params(), case.dtypes)]
    opt = ZOOptimizer(list(zip(case.names, ps)), case.cfg, ReplayScore(case.values, ps),
                      total_steps=case.spec["total_steps"])
    for _ in range(k):
        opt.step(None, [None] * Z)
    sd = opt.state_dict()
    saved = [p.detach().cpu().clone() for p in ps]
    del opt
    ps2 = [torch.nn.Parameter(t.cuda()) for t in saved]
    opt2 = ZOOptimizer(list(zip(case.names, ps2)), case.cfg, ReplayScore(case.values[2 * Z * k:], ps2),
                       total_steps=case.spec["total_steps"])
    opt2.load_state_dict(sd)
    for _ in range(steps - k):
        opt2.step(None, [None] * Z)
    got = flat([p.detach().float().cpu().numpy() for p in ps2])
    assert np.array_equal(got, full[-1])
