"""Seed-sharded population: pair assignment and the one collective of a step.

Pairs (perturbation seeds) are independent, so rank r evaluates pairs
j = r, r + W, r + 2W, ... of a step's Z pairs, with parameters replicated. The
only exchange is an all-gather of every pair's two scalar values (and the
score's metric scalars): ``gather_pair_values``. After it every rank holds the
same numbers and rebuilds the same update from seeds.

The reference runs one process per GPU with no communication
(sweeps/runall.py:5 ``GPUS_PER_RUN = 1``); this module is new.
"""
from __future__ import annotations

import math
from datetime import timedelta

import torch
import torch.distributed as dist


def world_info(group=None) -> tuple[int, int]:
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def local_pairs(z_batch: int, rank: int, world: int) -> list[int]:
    """Pairs of a step evaluated by `rank` (round-robin over ranks)."""
    return list(range(rank, z_batch, world))


def gather_pair_values(local: torch.Tensor, z_batch: int, rank: int, world: int, group=None) -> torch.Tensor:
    """All-gather per-pair rows.

    local: [len(local_pairs(z_batch, rank, world)), C] float32 rows in local pair order.
    Returns [z_batch, C] float32 on local's device, rows in global pair order.
    """
    n_max = math.ceil(z_batch / world) if z_batch else 0
    C = local.shape[1]
    backend = dist.get_backend(group)
    dev = local.device if backend == "nccl" else torch.device("cpu")
    buf = torch.full((n_max, C), float("nan"), dtype=torch.float32, device=dev)
    if local.shape[0]:
        buf[: local.shape[0]] = local.to(dev, torch.float32)
    out = torch.empty((world * n_max, C), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(out, buf, group=group)
    # row k of rank r holds pair r + k*world
    res = torch.empty((z_batch, C), dtype=torch.float32, device=dev)
    for r in range(world):
        js = local_pairs(z_batch, r, world)
        if js:
            res[js] = out[r * n_max: r * n_max + len(js)]
    return res.to(local.device)


def init_process_group_from_env(backend: str | None = None, timeout_s: float = 120.0):
    """torchrun-style init (RANK/WORLD_SIZE/MASTER_ADDR/MASTER_PORT) with a short
    timeout so that a rank that never arrives ends the others' collective with an error."""
    if dist.is_initialized():
        return
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kw = {}
    if backend == "nccl" and torch.cuda.is_available():
        import os
        kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_s), **kw)
