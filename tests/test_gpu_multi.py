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


def _worker(rank, world, port, name, out_dir, exchange=True):
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
    opt = ZOOptimizer(list(zip(case.names, ps)), case.cfg, ReplayScore(vals, ps),
                      field_exchange=None if exchange else False)
    assert opt.planner.sharded
    assert (opt.exchange is not None) == exchange   # peer stores mapped over CUDA IPC
    for _ in range(case.spec["steps"]):
        opt.step(None, [None] * Z)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), flat([p.detach().float().cpu().numpy() for p in ps]))
    np.save(os.path.join(out_dir, f"master{rank}.npy"), flat([m.float().cpu().numpy() for m in opt.master]))
    dist.barrier()
    if opt.exchange is not None:
        opt.exchange.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", [True, False])
@pytest.mark.parametrize("name", ["mezo_bf16_z3", "seedwin_adam_bf16_z2"])
def test_two_gpu_sharded_matches_single_gpu(name, exchange, tmp_path):
    from helpers import StepCase, step_cases
    from test_gpu_step import run_gpu
    G, _ = step_cases()
    a1, _, _ = run_gpu(StepCase(G, name))
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, str(tmp_path), exchange)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for r in range(2):
        live = np.load(tmp_path / f"rank{r}.npy")
        assert np.array_equal(live, a1[-1]), r
        assert np.array_equal(np.load(tmp_path / f"master{r}.npy"), live)


def _egg_worker(rank, world, port, out_dir):
    sys.path[:0] = [os.path.dirname(HERE), HERE]
    from datetime import timedelta

    import torch.distributed as dist
    from test_gpu_eggroll_model import SHAPE
    from toy_models import build_llama
    from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    tokens = torch.randint(0, SHAPE["vocab_size"], (4, 64), generator=torch.Generator().manual_seed(9)).cuda()
    model = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    pop = EggrollPopulation(model, EggrollConfig(sigma=2e-2))
    m = pop.step(tokens, [1, 2, 3, 4, 5, 6], lr=1e-3, strategy="centered_rank", chunk_pairs=2)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"egg{rank}.npy"), np.concatenate([p.detach().float().cpu().numpy().ravel()
                                                                     for _, p in pop.named]))
    np.save(os.path.join(out_dir, f"eggloss{rank}.npy"), np.array([m["loss"]]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_eggroll_step_matches_single_gpu(tmp_path):
    """EGGROLL ES step with the pairs sharded over 2 GPUs (rank r scores pairs r, r+2, ...;
    one all-gather of the member losses; the same update on both ranks) ends bit-identical
    to the one-GPU step: a member's loss does not depend on which members share its chunk."""
    from test_gpu_eggroll_model import SHAPE
    from toy_models import build_llama
    from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
    tokens = torch.randint(0, SHAPE["vocab_size"], (4, 64), generator=torch.Generator().manual_seed(9)).cuda()
    model = build_llama(SHAPE, dtype=torch.bfloat16, seed=0, device="cuda")
    pop = EggrollPopulation(model, EggrollConfig(sigma=2e-2))
    m1 = pop.step(tokens, [1, 2, 3, 4, 5, 6], lr=1e-3, strategy="centered_rank", chunk_pairs=4)
    one = np.concatenate([p.detach().float().cpu().numpy().ravel() for _, p in pop.named])
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_egg_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"egg{r}.npy"), one), r
        assert float(np.load(tmp_path / f"eggloss{r}.npy")[0]) == m1["loss"]
