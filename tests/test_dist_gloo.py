"""Seed-sharded population over torch.distributed, on CPU (gloo, world size 2).

Each rank evaluates its pairs (j = rank, rank + W, ...) through the host planner and
the oracle's pass interpreter, shares the pair values with the real
gather_pair_values all-gather, and runs the last pass. Every rank must end
bit-identical to the single-GPU op-by-op oracle. A second test makes one rank fail
before the collective and checks that the other rank's all-gather ends with an
error within the process-group timeout instead of hanging.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    from datetime import timedelta

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    return dist


def _sharded_worker(rank, world, port, name, out_dir, shard_update=False):
    sys.path[:0] = [os.path.dirname(HERE), HERE]
    import torch
    from helpers import StepCase, flat, step_cases
    from oracle.pass_interp import run_pass
    from zotitan_b200.distributed import gather_pair_values
    from zotitan_b200.train_zo import StepPlanner
    dist = _init(rank, world, port, 60)
    G, _ = step_cases()
    case = StepCase(G, name)
    params = case.params()
    pl = StepPlanner(case.cfg, total_steps=case.spec["total_steps"], rank=rank, world=world)
    assert pl.sharded
    layout = None
    if shard_update:   # last pass on this rank's unit range, then all-gather the flat master
        from zotitan_b200.flat import FlatLayout
        layout = FlatLayout([p.size for p in params], world, chunks=3)
        pl.unit_ranges = layout.shard_ranges(rank)
    ts = [{"data": p, "live": p.copy(), "m": np.zeros_like(p) if pl.needs_m else None,
           "v": np.zeros_like(p) if pl.needs_v else None, "anchor": p.copy() if pl.needs_anchor else None,
           "ge": None, "dtype": dt, "index": i} for i, (p, dt) in enumerate(zip(params, case.dtypes))]
    it = iter(case.values)
    Z = case.cfg.z_batch
    for _ in range(case.spec["steps"]):
        vals_all = [next(it) for _ in range(2 * Z)]
        local = pl.start()
        rows = []
        for j in local:
            spec = pl.plus_pass(j, None)
            run_pass(ts, len(ts), spec.cfg, spec.streams)
            spec = pl.minus_pass(j)
            run_pass(ts, len(ts), spec.cfg, spec.streams)
            rows.append([vals_all[2 * j], vals_all[2 * j + 1]])   # this rank's "forwards"
        local_t = torch.tensor(rows, dtype=torch.float32).reshape(len(local), 2)
        gathered = gather_pair_values(local_t, Z, rank, world).tolist()
        vals = [x for row in gathered for x in row]
        spec, _ = pl.finish(vals)
        for ub, ue in (spec.unit_ranges or [(0, 0)]):   # chunk by chunk, as ZOOptimizer runs it
            spec.cfg.unit_begin, spec.cfg.unit_end = ub, ue
            run_pass(ts, len(ts), spec.cfg, spec.streams)
        if layout is not None:
            buf = np.zeros(layout.numel, np.float32)
            for o, p in zip(layout.offsets, params):
                buf[o:o + p.size] = p.reshape(-1)
            full = torch.from_numpy(buf)
            for k in range(layout.chunks):   # in-place all-gather of each chunk
                dist.all_gather_into_tensor(layout.chunk(full, k), layout.shard_chunk(full, rank, k).clone())
            full = full.numpy()
            for o, p, t in zip(layout.offsets, params, ts):
                p.reshape(-1)[:] = full[o:o + p.size]
                t["live"].reshape(-1)[:] = full[o:o + p.size]
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), flat(params))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("shard_update", [False, True])
@pytest.mark.parametrize("name", ["mezo_bf16_z3", "seedwin_adam_bf16_z2", "es_rank_f32"])
def test_sharded_gloo_ranks_match_single_gpu(name, shard_update, tmp_path):
    """Both the replicated last pass and the sharded update (each rank updates its unit
    range, one all-gather completes the parameters) end bit-identical to one GPU."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, name, str(tmp_path), shard_update))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    from helpers import StepCase, flat, step_cases
    from oracle.zo_step import OracleZO
    G, _ = step_cases()
    case = StepCase(G, name)
    params = case.params()
    opt = OracleZO(params, case.dtypes, case.cfg, total_steps=case.spec["total_steps"], noise="c", semantics="cuda")
    it = iter(case.values)
    for _ in range(case.spec["steps"]):
        opt.step(lambda ps, b: (next(it), {}), [None] * case.cfg.z_batch)
    want = flat(params)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"rank{r}.npy"), want), r


def _failing_worker(rank, world, port, out_dir):
    sys.path[:0] = [os.path.dirname(HERE), HERE]
    import torch
    from zotitan_b200.distributed import gather_pair_values
    dist = _init(rank, world, port, 5)
    if rank == 1:
        os._exit(3)                      # dies between steps, before the collective
    try:
        gather_pair_values(torch.zeros(1, 2), 2, rank, world)
        status = "returned"
    except Exception as e:               # the collective must fail, not hang
        status = "error:" + type(e).__name__
    open(os.path.join(out_dir, "rank0.txt"), "w").write(status)
    os._exit(0)


def test_dead_rank_ends_collective_with_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    assert (tmp_path / "rank0.txt").read_text().startswith("error:")


def test_local_pairs_cover_every_pair_once():
    from zotitan_b200.distributed import local_pairs
    for Z in (1, 2, 7, 8, 64):
        for W in (1, 2, 3, 8):
            got = sorted(j for r in range(W) for j in local_pairs(Z, r, W))
            assert got == list(range(Z))
