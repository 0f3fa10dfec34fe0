"""Seed-sharded ZOOptimizer on 2 GPUs over NCCL (skipped with fewer GPUs).

Two ranks, one process per GPU, replay the reference's recorded pair values: rank r
scores pairs r, r+2, ...; one all-gather shares the values; both ranks run the last
pass over their master copy. Both must end bit-identical to the single-GPU
ZOOptimizer, and the live copy the model reads must equal the master.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, out_dir):
    sys.path[:0] = [os.path.dirname(HERE), HERE]
    from datetime import timedelta

    import torch.distributed as dist
    from helpers import StepCase, flat, step_cases
    from test_gpu_step import TDT, ReplayScore
    from zotitan_b200.train_zo import ZOOptimizer
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    G, _ = step_cases()
    case = StepCase(G, name)
    ps = [torch.nn.Parameter(torch.from_numpy(p).to(TDT[d]).cuda()) for p, d in zip(case.params(), case.dtypes)]
    Z = case.cfg.z_batch
    # this rank's score_fn sees only its own pairs: feed it their recorded values in order
    vals = []
    for s in range(case.spec["steps"]):
        step_vals = case.values[2 * Z * s: 2 * Z * (s + 1)]
        for j in range(rank, Z, world):
            vals += step_vals[2 * j: 2 * j + 2]
    opt = ZOOptimizer(list(zip(case.names, ps)), case.cfg, ReplayScore(vals, ps))
    assert opt.planner.sharded
    for _ in range(case.spec["steps"]):
        opt.step(None, [None] * Z)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), flat([p.detach().float().cpu().numpy() for p in ps]))
    np.save(os.path.join(out_dir, f"master{rank}.npy"), flat([m.float().cpu().numpy() for m in opt.master]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["mezo_bf16_z3", "seedwin_adam_bf16_z2"])
def test_two_gpu_sharded_matches_single_gpu(name, tmp_path):
    from helpers import StepCase, step_cases
    from test_gpu_step import run_gpu
    G, _ = step_cases()
    a1, _, _ = run_gpu(StepCase(G, name))
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for r in range(2):
        live = np.load(tmp_path / f"rank{r}.npy")
        assert np.array_equal(live, a1[-1]), r
        assert np.array_equal(np.load(tmp_path / f"master{r}.npy"), live)
