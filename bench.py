#!/usr/bin/env python
"""Benchmark of the zeroth-order hot path (one JSON line on rank 0).

Workload (N=1 default): the kernel microbench on the full parameter set of a
Llama-3.2-1B-shaped model (146 bf16 tensors, 1,235,814,400 params, N(0,0.02)),
64 seeds per step drawn from a seeded uint64 stream, eps = 1e-3. One step = for each
seed: +eps (fused with the previous seed's restore and its grad_est term), -2eps; then
the last restore, the last grad_est term and the update in one pass: 129 fused passes,
no forward (synthetic pair values). ``value`` = ZO steps/s over all ranks (seeds sharded
round-robin over ranks, one all-gather of the pair values, replicated final pass).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "ZO steps/s + perturb-pass HBM GB/s (Llama-1B); EGGROLL member-evals/s (8B)"
UNIT = "ZO steps/s"
N_SEEDS = 64
EPS = 1e-3
LR = 1e-6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seeds", type=int, default=N_SEEDS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-eggroll", action="store_true", help="skip the EGGROLL population measurement")
    ap.add_argument("--no-mezo", action="store_true", help="skip the MeZO full fine-tune step measurement")
    ap.add_argument("--no-lora", action="store_true", help="skip the MeZO-Adam LoRA step measurement")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own step on the GPU (baseline/reference_steps.py)")
    ap.add_argument("--field-exchange", type=float, default=0.8,
                    help="sharded runs: fraction of free device memory for the field stores (0: regenerate)")
    ap.add_argument("--exchange-mode", choices=["copies", "in_pass"], default="copies",
                    help="sharded runs: push the fields by copy-engine copies or from the +eps pass")
    ap.add_argument("--push-order", choices=["rotate", "all"], default="rotate",
                    help="sharded runs: field pushes to one peer at a time in rotating order, or to all at once")
    ap.add_argument("--push-after", choices=["plus", "minus"], default=None,
                    help="sharded runs: start a pair's field pushes after its +eps or its -2eps pass")
    ap.add_argument("--push-streams", type=int, default=1,
                    help="sharded runs with --push-order all: copy streams per destination")
    ap.add_argument("--profile-case", choices=["chain", "full", "replay", "chain-cached", "full-cached", "plus-cached",
                                               "replay-field", "replay-mixed", "lce", "lowrank", "push-rates", "eggroll", "eggroll-gated", "eggroll-forward",
                                               "mezo-step", "lora-step"],
                    default=None,
                    help="small case for ncu: one bf16 tensor of 2^28 elements, 3 launches of the "
                         "-2eps pass (chain) or of the restore+accumulate+perturb pass (full); or 3 "
                         "EGGROLL linear launches (rank-4 term as a K-slab) on the 8B gate_proj shape, 16 "
                         "members x 1024 rows (eggroll), or 3 gated gate/up/SwiGLU launches on it "
                         "(eggroll-gated); or one 16-member EGGROLL population chunk of the 8B model inside "
                         "the NVTX range 'egg_chunk' (eggroll-forward)")
    ap.add_argument("--eggroll-gemm", action="store_true",
                    help="time the EGGROLL population linear layer on the Llama-3-8B layer shapes")
    return ap.parse_args()


EGG_SHAPES = {  # Llama-3-8B linear layers (N, K): out x in
    "q_proj/o_proj": (4096, 4096), "k_proj/v_proj": (1024, 4096), "gate_proj/up_proj": (14336, 4096),
    "down_proj": (4096, 14336)}


def eggroll_inputs(M, N, K, T, dev, seed=0):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    members = M // T
    x = (torch.randn(M, K, device=dev, generator=g)).bfloat16()
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
    a = torch.randn(members, N, 4, device=dev, generator=g)
    b = torch.randn(members, K, 4, device=dev, generator=g)
    sigma = torch.full((members,), 1e-3, device=dev)
    return x, w, a, b, sigma


def eggroll_gemm_bench(rows: int = 16384, T: int = 1024, reps: int = 10):
    """TFLOP/s of zt_eggroll_linear (base GEMM FLOPs 2*M*N*K) per Llama-3-8B layer shape,
    with torch.matmul (cuBLAS) of the plain GEMM on the same shapes for context."""
    import torch

    from zotitan_b200 import kernels as K_
    dev = torch.device("cuda")
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("bf16_tflops", 1590.0)
    res = {}
    for name, (N, Kd) in EGG_SHAPES.items():
        x, w, a, b, sigma = eggroll_inputs(rows, N, Kd, T, dev)
        y = torch.empty(rows, N, dtype=torch.bfloat16, device=dev)
        xb = torch.empty(rows, 4, dtype=torch.float32, device=dev)

        def timed(fn):
            fn(); torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(reps):
                fn()
            e.record(); torch.cuda.synchronize()
            return s.elapsed_time(e) / reps
        ms = timed(lambda: K_.eggroll_linear(x, w, a, b, sigma, T, out=y, xb=xb))
        ms_cublas = timed(lambda: torch.matmul(x, w.T))
        flops = 2.0 * rows * N * Kd
        res[name] = {"M": rows, "N": N, "K": Kd, "ms": ms, "tflops": flops / ms / 1e9,
                     "frac_of_peak": flops / ms / 1e9 / peak, "cublas_plain_gemm_tflops": flops / ms_cublas / 1e9}
    assert K_.eggroll_take_error() == 0
    print(json.dumps({"eggroll_gemm": res, "peak_tflops": peak,
                      "peak_source": "MEASURED_PEAKS.json bf16_tflops" if "bf16_tflops" in peaks else "fallback"}))


def _profile_push_rates():
    """Peer-to-peer push rates between the ranks of one node (run under torchrun, one rank
    per GPU): copy-engine pushes of 512 MB per (sender, receiver) into CUDA-IPC-mapped
    buffers with every peer at once, issued in the same peer order on every rank or
    starting at each rank's next peer (1, 2 or 4 streams per peer), one peer at a time in
    rotating order (rank r sends to r + 1, r + 2, ...: every moment a permutation), every
    rank to its next neighbour only, and NCCL all_to_all_single of the same volume. CUDA
    events around each test between barriers, best of 3, max over ranks; rank 0 prints one
    JSON line per test (GB/s sent per GPU)."""
    import ctypes

    import torch
    import torch.distributed as dist

    from zotitan_b200 import _lib as L
    from zotitan_b200.distributed import init_process_group_from_env
    init_process_group_from_env("nccl", timeout_s=300)
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    lib = L.load()
    slot = 512 << 20
    store = torch.empty(world * slot, dtype=torch.uint8, device=dev)
    src = torch.full((world * slot,), rank, dtype=torch.uint8, device=dev)
    h = (ctypes.c_ubyte * L.ZT_IPC_HANDLE_BYTES)()
    off = ctypes.c_uint64()
    L.check(lib.zt_ipc_export(store.data_ptr(), h, ctypes.byref(off)), "zt_ipc_export")
    handles = [None] * world
    dist.all_gather_object(handles, (bytes(h), off.value))
    peer, opened = [0] * world, []
    for p, (hb, o) in enumerate(handles):
        if p == rank:
            peer[p] = store.data_ptr()
            continue
        base = ctypes.c_void_p()
        L.check(lib.zt_ipc_open((ctypes.c_ubyte * L.ZT_IPC_HANDLE_BYTES).from_buffer_copy(hb), ctypes.byref(base)),
                "zt_ipc_open")
        opened.append(base.value)
        peer[p] = base.value + o

    def timed(fn):
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def copies(plan):   # plan: list of (stream index, peer, piece index, pieces)
        streams = [torch.cuda.Stream(dev) for _ in range(1 + max(q for q, _, _, _ in plan))]

        def run():
            cur = torch.cuda.current_stream(dev)
            for st in streams:
                st.wait_stream(cur)
            for q, p, i, k in plan:
                piece = slot // k
                L.check(lib.zt_copy_async(peer[p] + rank * slot + i * piece, src.data_ptr() + p * slot + i * piece,
                                          piece, ctypes.c_void_p(streams[q].cuda_stream)), "zt_copy_async")
            for st in streams:
                cur.wait_stream(st)
        return run

    others = [(rank + k) % world for k in range(1, world)]
    tests = []
    # every rank issuing its copies in the same peer order (lowest rank first): the ranks'
    # first copies all land on the same receiver
    same = [p for p in range(world) if p != rank]
    tests.append(("every_peer_at_once_same_order", copies([(j, p, 0, 1) for j, p in enumerate(same)]),
                  len(others) * slot))
    for k in (1, 2, 4):
        plan = [(j * k + i, p, i, k) for j, p in enumerate(others) for i in range(k)]
        tests.append((f"every_peer_at_once_{k}_streams_per_peer", copies(plan), len(others) * slot))
    tests.append(("one_peer_at_a_time_rotating", copies([(0, p, 0, 1) for p in others]), len(others) * slot))
    tests.append(("next_neighbour_only", copies([(0, others[0], 0, 1)]), slot))
    out = torch.empty_like(src)
    tests.append(("nccl_all_to_all_single", lambda: dist.all_to_all_single(out, src), len(others) * slot))
    rows = []
    for name, fn, nbytes in tests:
        fn()
        ms = min(timed(fn) for _ in range(3))
        rows.append({"profile_case": "push-rates", "world": world, "test": name, "ms": ms,
                     "gbs_sent_per_gpu": nbytes / ms / 1e6})
    torch.cuda.synchronize()
    for base in opened:
        lib.zt_ipc_close(ctypes.c_void_p(base))
    dist.barrier()
    if rank == 0:
        for r in rows:
            print(json.dumps(r))
    dist.destroy_process_group()


def _profile_lowrank():
    """The fused low-rank direction (zt_lowrank_prepare / zt_lowrank_apply) on a
    [16384, 8192] bf16 matrix (268 MB, larger than L2) at rank 64, against the reference's
    materialised ops (P @ Psi on cuBLAS, norm, scale, foreach add). Algorithmic bytes of
    one apply: the parameter read and written, 4 B per element."""
    import torch

    from zotitan_b200 import kernels as K
    from zotitan_b200.kernels import param_key, randn
    m, n, r = 16384, 8192, 64
    g = torch.Generator(device="cuda").manual_seed(0)
    theta = (torch.randn(m, n, device="cuda", generator=g) * 0.02).bfloat16()
    ge = torch.zeros_like(theta)
    keys = [param_key(s, 3, 0) for s in range(8)], [param_key(s, 3, 1) for s in range(8)]
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def timed(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    one = K.LowRankFactors((m, n), r, torch.bfloat16, keys[0][:1], keys[1][:1], "cuda")
    ms_prep = timed(lambda: K.LowRankFactors((m, n), r, torch.bfloat16, keys[0][:1], keys[1][:1], "cuda"), 5)
    ms_apply = timed(lambda: one.apply(src=theta, dst=theta, alphas=(1e-3,)), 10)
    eight = K.LowRankFactors((m, n), r, torch.bfloat16, keys[0], keys[1], "cuda")
    ms_ge8 = timed(lambda: eight.apply(ge=ge, coefs=[0.1] * 8, ge_init=True), 5)

    def materialised():
        P = randn(keys[0][0], m * r, "cuda").view(m, r).bfloat16()
        Psi = randn(keys[1][0], r * n, "cuda").view(r, n).bfloat16()
        z = P @ Psi
        z = z * ((m * n) ** 0.5 / (z.norm() + 1e-7))
        torch._foreach_add_([theta], [z], alpha=1e-3)
    ms_mat = timed(materialised, 5)
    try:
        peak = json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["hbm_gbs"]
    except (OSError, ValueError, KeyError):
        peak = 6650.0
    gbs = 4.0 * m * n / ms_apply / 1e6
    print(json.dumps({"profile_case": "lowrank", "shape": [m, n], "rank": r, "ms_prepare": ms_prep,
                      "ms_apply": ms_apply, "apply_gbs": gbs, "apply_frac_of_measured_hbm": gbs / peak,
                      "ms_ge_8_streams": ms_ge8, "ms_materialised_one_use": ms_mat,
                      "error": K.lowrank_take_error()}))


def _profile_step(kind: str):
    """CUDA kernel table (torch.profiler) of one ZO step after two warm-up steps: the MeZO
    full fine-tune of the Llama-1B shape (8 pairs, 16 x 512 tokens each) or the seed-window
    MeZO-Adam step on rank-16 LoRA adapters of the Llama-8B shape (8 x 1024 tokens)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from zotitan_b200.data import synthetic_token_batch
    from zotitan_b200.llama_fused import fuse_llama
    from zotitan_b200.lora import LoRAConfig, make_lora
    from zotitan_b200.objective import SyntheticTokensObjective
    from zotitan_b200.synthetic import LLAMA_1B, LLAMA_8B, build_llama
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer
    cfg = ZOConfig()
    if kind == "mezo-step":
        shape, B, S = LLAMA_1B, 16, 512
        model = build_llama(shape, device="cuda", seed=0, max_positions=S)
        objective = SyntheticTokensObjective(shape.vocab, S, z_loss_weight=1e-4)
        cfg.eps, cfg.z_batch, cfg.base.lr = EPS, 8, 1e-5
    else:
        shape, B, S = LLAMA_8B, 8, 1024
        model = build_llama(shape, device="cuda", seed=0, max_positions=S)
        make_lora(model, LoRAConfig(r=16, alpha=32, dtype="fp32"))
        objective = SyntheticTokensObjective(shape.vocab, S)
        cfg.eps, cfg.z_batch, cfg.base.lr = EPS, 1, 1e-5
        cfg.mom.momentum_method, cfg.mom.beta1, cfg.mom.beta2, cfg.mom.second_moment = "seed_window", 0.9, 0.999, True
        cfg.seed_window.size = 16
    fuse_llama(model)
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    opt = ZOOptimizer(named, cfg, objective.score, total_steps=10)
    batches = [synthetic_token_batch(shape.vocab, B, S, j, device="cuda") for j in range(cfg.z_batch)]
    for _ in range(2):
        opt.step(model, batches)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        opt.step(model, batches)
        torch.cuda.synchronize()
    print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=20, max_name_column_width=90))


def profile_case(kind: str):
    """A few launches of one pass kind on a 512 MB bf16 tensor (larger than L2)."""
    import torch

    from zotitan_b200 import _lib as L
    from zotitan_b200 import kernels as K
    if kind in ("mezo-step", "lora-step"):
        _profile_step(kind)
        return
    if kind == "eggroll-forward":
        from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
        from zotitan_b200.synthetic import LLAMA_8B, build_llama
        model = build_llama(LLAMA_8B, device="cuda", seed=0, max_positions=1024)
        pop = EggrollPopulation(model, EggrollConfig(sigma=1e-3))
        tokens = torch.randint(0, LLAMA_8B.vocab, (4, 256), generator=torch.Generator().manual_seed(7)).cuda()
        pop.evaluate(tokens, list(range(8)))      # warm-up chunk
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("egg_chunk")
        a.record()
        losses = pop.evaluate(tokens, list(range(8, 16)))
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": kind, "members": 16, "ms": a.elapsed_time(b),
                          "mean_loss": float(losses.mean()), "error": K.eggroll_take_error()}))
        return
    if kind == "lce":   # the config-3 scorer: 16 x 512 rows, vocabulary 128256, d 2048
        rows, vocab, k = 16 * 512, 128256, 2048
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(rows, k, device="cuda", generator=g).bfloat16()
        w = (torch.randn(vocab, k, device="cuda", generator=g) * 0.02).bfloat16()
        t = torch.randint(0, vocab, (rows,), device="cuda", generator=g)
        for _ in range(3):
            K.linear_xent(x, w, t)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        a.record()
        for _ in range(reps):
            K.linear_xent(x, w, t)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        # the path it replaces: cuBLAS lm_head in 8192-row chunks + zt_xent_rows (warmed up:
        # the logits buffer allocated and cuBLAS's choice made before the timed calls)
        from zotitan_b200.losses import CHUNK_ROWS
        for _ in range(3):
            for r0 in range(0, rows, CHUNK_ROWS):
                K.xent_rows(torch.nn.functional.linear(x[r0:r0 + CHUNK_ROWS], w), t[r0:r0 + CHUNK_ROWS])
        torch.cuda.synchronize()
        a.record()
        for _ in range(reps):
            for r0 in range(0, rows, CHUNK_ROWS):
                K.xent_rows(torch.nn.functional.linear(x[r0:r0 + CHUNK_ROWS], w), t[r0:r0 + CHUNK_ROWS])
        b.record()
        torch.cuda.synchronize()
        ms_old = a.elapsed_time(b) / reps
        flops = 2.0 * rows * vocab * k
        print(json.dumps({"profile_case": kind, "ms": ms, "tflops": flops / ms / 1e9, "ms_gemm_then_xent": ms_old,
                          "tflops_gemm_then_xent": flops / ms_old / 1e9, "error": K.linear_xent_take_error()}))
        return
    if kind == "lowrank":   # one low_rank direction of a [16384, 8192] bf16 matrix, rank 64
        _profile_lowrank()
        return
    if kind == "push-rates":   # under torchrun: peer-to-peer push rates of the field exchange
        _profile_push_rates()
        return
    n = 1 << 28
    p = (torch.randn(n, device="cuda") * 0.02).bfloat16()
    f = lambda x: float(np.float32(x))  # noqa: E731
    if kind in ("eggroll", "eggroll-gated"):
        M, N, Kd, T = 16384, 14336, 4096, 1024
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(M, Kd, device="cuda", generator=g).bfloat16()
        w = (torch.randn(N, Kd, device="cuda", generator=g) * 0.02).bfloat16()
        bt = torch.zeros((M // T, 16, Kd), dtype=torch.bfloat16, device="cuda")
        fg = K.eggroll_factors(list(range(8)), list(range(8, 16)), N, Kd, 1e-3, "cuda", ext_slot=0, b_ext=bt)
        if kind == "eggroll":
            xe = K.eggroll_xb_ext(x, [fg[1]], [fg[2]], [0], T, bt=bt)[0]
            y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            run = lambda: K.eggroll_linear(x, w, fg[0], None, fg[2], T, out=y, x_ext=xe, w_ext=fg[3])  # noqa: E731
            flops = 2.0 * M * N * Kd
        else:
            fu = K.eggroll_factors(list(range(16, 24)), list(range(24, 32)), N, Kd, 1e-3, "cuda", ext_slot=1, b_ext=bt,
                                   b_ext_row=4)
            xe = K.eggroll_xb_ext(x, [fg[1], fu[1]], [fg[2], fu[2]], [1, 2], T, bt=bt)[0]
            run = lambda: K.eggroll_gated(x, w, w, fg, fu, None, None, T, x_ext=xe)  # noqa: E731
            flops = 4.0 * M * N * Kd
        for _ in range(2):
            run()
        torch.cuda.synchronize()
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        run()
        b_.record()
        torch.cuda.synchronize()
        ms = a_.elapsed_time(b_)
        print(json.dumps({"profile_case": kind, "ms": ms, "tflops": flops / ms / 1e9, "error": K.eggroll_take_error()}))
        return
    if kind == "chain":
        tab = K.ParamTable([p])
        cfg, streams = K.PassCfg(), [K.Stream(5, (f(-2e-3),))]
    elif kind == "chain-cached":   # the -2eps pass reading z from the noise cache
        tab = K.ParamTable([p])
        zc = tab.noise_cache()
        tab.run(K.PassCfg(zcache=zc.data_ptr()), [K.Stream(5, (f(1e-3),), z_store=True)])
        cfg, streams = K.PassCfg(zcache=zc.data_ptr()), [K.Stream(5, (f(-2e-3),), z_load=True)]
    elif kind == "full-cached":    # restore (z from the cache) + grad_est + next perturb (z stored)
        ge = torch.zeros_like(p)
        vals = torch.tensor([2.01, 2.0], device="cuda")
        tab = K.ParamTable([p], ge=[ge])
        zc = tab.noise_cache()
        tab.run(K.PassCfg(zcache=zc.data_ptr()), [K.Stream(4, (f(1e-3),), z_store=True)])
        cfg = K.PassCfg(ge_mode=L.ZT_GE_ACCUM, ge_load=True, ge_store=True, dev_vals=vals.data_ptr(),
                        dev_inv2eps=f(500.0), dev_invz=f(1 / 64), dev_tau=float("inf"), zcache=zc.data_ptr())
        # repeated launches read back the field the previous launch stored: the values
        # differ from a real schedule's, the work per element is the same
        streams = [K.Stream(4, (f(1e-3),), ge_dev=True, z_load=True), K.Stream(5, (f(1e-3),), z_store=True)]
    elif kind == "plus-cached":   # the sharded +eps pass: live = master + eps z, z written to the cache
        live = torch.empty_like(p)
        tab = K.ParamTable([p], live=[live])
        zc = tab.noise_cache()
        cfg = K.PassCfg(src=L.ZT_BUF_DATA, dst=L.ZT_BUF_LIVE, zcache=zc.data_ptr())
        streams = [K.Stream(5, (f(1e-3),), z_store=True)]
    elif kind in ("replay-field", "replay-mixed"):
        # the sharded last pass, 16 pairs' fields read from a field store (replay-mixed: every
        # other pair's field regenerated instead, as when the store holds only some pairs)
        n = 1 << 25
        p = p[:n]
        tab = K.ParamTable([p])
        units = int(tab.plan.n_units)
        store = torch.randn(16 * units * 2048, device="cuda")
        cfg = K.PassCfg(ge_mode=L.ZT_GE_ACCUM, update=True, lr=f(1e-5), zfield=store.data_ptr(),
                        zfield_stride=units * 2048)
        mixed = kind == "replay-mixed"
        streams = [K.Stream(100 + j, (f(1e-3), f(-2e-3), f(1e-3)), ge=f(0.01 * (j - 8)),
                            z_field=None if mixed and j % 2 else j) for j in range(16)]
    elif kind == "replay":   # the sharded step's last pass: 16 pairs' chains + grad_est + SGD
        tab = K.ParamTable([p])
        cfg = K.PassCfg(ge_mode=L.ZT_GE_ACCUM, update=True, lr=f(1e-5))
        streams = [K.Stream(100 + j, (f(1e-3), f(-2e-3), f(1e-3)), ge=f(0.01 * (j - 8))) for j in range(16)]
    else:
        ge = torch.zeros_like(p)
        vals = torch.tensor([2.01, 2.0], device="cuda")
        tab = K.ParamTable([p], ge=[ge])
        cfg = K.PassCfg(ge_mode=L.ZT_GE_ACCUM, ge_load=True, ge_store=True, dev_vals=vals.data_ptr(),
                        dev_inv2eps=f(500.0), dev_invz=f(1 / 64), dev_tau=float("inf"))
        streams = [K.Stream(4, (f(1e-3),), ge_dev=True), K.Stream(5, (f(1e-3),))]
    for _ in range(3):
        tab.run(cfg, streams)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10   # back to back, so the host's launch latency stays off the device clock
    a.record()
    for _ in range(reps):
        tab.run(cfg, streams)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    print(json.dumps({"profile_case": kind, "elements": n, "streams": len(streams), "ms": ms,
                      "G_elem_per_s": n / ms / 1e6, "G_stream_elem_per_s": n * len(streams) / ms / 1e6}))


def env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


# ── clocks ─────────────────────────────────────────────────────────────────────────

class ClockSampler:
    """nvidia-smi sampled every 200 ms during the timed region (reading only)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.gpu_id], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}


# ── CPU baseline: the oracle port on host cores ───────────────────────────────────────

def workload_config(world: int, seeds: int, numel: int, n_tensors: int) -> dict:
    """The `config` of the microbench line, the same in both arms."""
    return {"workload": "Llama-3.2-1B-shaped parameter set, 64 seeds/step (kernel microbench)",
            "params": numel, "tensors": n_tensors, "seeds_per_step": seeds, "eps": EPS,
            "parallelism": f"seed-sharded x{world}", "l2": "inputs (2.47 GB of bf16 parameters) larger than L2"}


class PortStep:
    """The reference's per-pair algorithm (materialise z, three perturb ops, one grad_est
    accumulation, zotitan/train_zo.py:534-556; the update, :376-407) in the C oracle, over
    the FULL parameter set (every element of the 1.236e9), one thread per host core
    (ctypes releases the GIL). theta and grad_est are fp32 carriers of bf16 values; z is
    generated block by block per thread. A step of 64 pairs is 64 pair passes and the
    update, so a pair and the update are timed and only the pair count is extrapolated."""

    BLOCK = 1 << 20

    def __init__(self, total_numel: int, n_tensors: int):
        from concurrent.futures import ThreadPoolExecutor

        from oracle import philox as ph
        self.ph, self.lib = ph, ph.lib()
        self.n, self.n_tensors = total_numel, n_tensors
        self.cores = os.cpu_count() or 1
        self.th = np.full(total_numel, 2.0 ** -7, dtype=np.float32)    # bf16-exact values
        self.ge = np.zeros(total_numel, dtype=np.float32)
        chunk = (total_numel + self.cores - 1) // self.cores
        self.spans = [(i * chunk, min(total_numel, (i + 1) * chunk)) for i in range(self.cores)
                      if i * chunk < total_numel]
        self.pool = ThreadPoolExecutor(self.cores)
        self.a_p, self.a_m = float(np.float32(EPS)), float(np.float32(-2 * EPS))

    def _pair_span(self, args):
        key, lo, hi, c = args
        ph, lib = self.ph, self.lib
        z = np.empty(self.BLOCK, np.float32)
        for b in range(lo, hi, self.BLOCK):
            n = min(self.BLOCK, hi - b)
            lib.zo_randn(key, b, n, ph._p(z))
            t, g = self.th[b:b + n], self.ge[b:b + n]
            for a in (self.a_p, self.a_m, self.a_p):
                lib.zo_add_scaled(ph.BF16, ph._p(t), ph._p(z), a, n)
            lib.zo_add_scaled(ph.BF16, ph._p(g), ph._p(z), c, n)

    def _update_span(self, args):
        lo, hi = args
        ph = self.ph
        self.lib.zo_add_scaled(ph.BF16, ph._p(self.th[lo:hi]), ph._p(self.ge[lo:hi]), -float(np.float32(LR)), hi - lo)

    def pair(self, j: int) -> float:
        t0 = time.perf_counter()
        key = self.ph.param_key(j, self.n_tensors, 0)
        list(self.pool.map(self._pair_span, [(key, lo, hi, 0.01) for lo, hi in self.spans]))
        return time.perf_counter() - t0

    def update(self) -> float:
        t0 = time.perf_counter()
        list(self.pool.map(self._update_span, self.spans))
        return time.perf_counter() - t0

    def close(self):
        self.pool.shutdown()
        self.th = self.ge = None


def cpu_port_baseline(total_numel: int, n_tensors: int, n_seeds: int) -> dict:
    """One pair and the update over the full parameter set; steps/s = 1 / (seeds x pair + update)."""
    port = PortStep(total_numel, n_tensors)
    t_pair = port.pair(0)
    t_upd = port.update()
    port.close()
    return {"value": 1.0 / (n_seeds * t_pair + t_upd), "unit": UNIT, "cores": port.cores, "kind": "port",
            "sample": f"one pair (z materialised, +eps, -2eps, +eps, grad_est) and the update over all "
                      f"{total_numel} elements in the C oracle with {port.cores} threads: {t_pair:.2f} s + "
                      f"{t_upd:.2f} s; the step's {n_seeds} pairs extrapolated from the one"}


def reference_config1_subprocess():
    """Start the reference's own config-1 CPU step (baseline/reference_steps.py) in the
    background; returns a collector. It runs on its own host threads with CUDA hidden."""
    script = os.path.join(HERE, "baseline", "reference_steps.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", REF_CPU_THREADS="4", OMP_NUM_THREADS="4")
    try:
        proc = subprocess.Popen([sys.executable, script, "cpu-config1"], stdout=subprocess.PIPE,
                                stderr=subprocess.PIPE, text=True, env=env)
    except OSError as e:
        return lambda: {"unavailable": f"could not start: {e}"}

    def collect(timeout_s: float = 300.0) -> dict:
        try:
            out, err = proc.communicate(timeout=timeout_s)
        except subprocess.TimeoutExpired:
            proc.kill()
            return {"unavailable": f"did not finish within {timeout_s:.0f} s"}
        lines = [x for x in out.strip().splitlines() if x.startswith("{")]
        if proc.returncode != 0 or not lines:
            return {"unavailable": (err.strip().splitlines() or ["no output"])[-1][:300]}
        return json.loads(lines[-1])
    return collect


def reference_gpu_microbench(seeds: int) -> dict:
    """The reference's own ZOOptimizer.step on this GPU over the same parameter set, seeds
    and pair values (baseline/reference_steps.py gpu-microbench), in a separate process."""
    script = os.path.join(HERE, "baseline", "reference_steps.py")
    try:
        r = subprocess.run([sys.executable, script, "gpu-microbench", "--seeds", str(seeds), "--steps", "2",
                            "--warmup", "1"], capture_output=True, text=True, timeout=600)
    except (OSError, subprocess.TimeoutExpired) as e:
        return {"unavailable": str(e)[:300]}
    lines = [x for x in r.stdout.strip().splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"unavailable": (r.stderr.strip().splitlines() or ["no output"])[-1][:300]}
    return json.loads(lines[-1])


# ── reference arm ───────────────────────────────────────────────────────────────────

def run_reference(args, rank, world):
    """The reference arm: the oracle port of the reference's CPU algorithm on the host
    cores (the reference is Python; nothing of it compiles to a native library). Each
    timed step is one pair over the full parameter set; the update is timed once in the
    warm-up; value = 1 / (seeds x mean pair time + update time)."""
    if rank != 0:
        return
    from zotitan_b200.synthetic import LLAMA_1B, llama_param_shapes, numel
    shapes = llama_param_shapes(LLAMA_1B)
    total = numel(shapes)
    port = PortStep(total, len(shapes))
    t_upd = port.update()
    for j in range(args.warmup):
        port.pair(j)
    w0 = time.perf_counter()
    pairs = [port.pair(args.warmup + j) for j in range(args.steps)]
    wall = time.perf_counter() - w0
    port.close()
    t_pair = statistics.mean(pairs)
    v = 1.0 / (args.seeds * t_pair + t_upd)
    sample = (f"each timed step: one pair (z materialised, +eps, -2eps, +eps, grad_est) over all {total} "
              f"elements in the C oracle with {port.cores} threads, mean {t_pair:.2f} s; update {t_upd:.2f} s "
              f"(timed once); value extrapolates the pair count to {args.seeds}")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * t_pair, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(world, args.seeds, total, len(shapes)),
            "timed_region_s": wall, "full_step_s": args.seeds * t_pair + t_upd,
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": port.cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ── EGGROLL population evaluation (Llama-3-8B shape) ─────────────────────────────────────

def eggroll_member_evals(dev, rank: int, world: int, total_pairs: int = 512, pairs_per_chunk: int = 8):
    """Member-evals/s of the EGGROLL population forward on the
    Llama-3-8B-shaped bf16 model, 1024 members (512 antithetic pairs, seeds 0..511) each
    scored with cross-entropy on a shared 4 x 256-token batch, sigma = 1e-3, rank-4
    perturbations regenerated from Philox seeds, the population sharded over the ranks
    (rank r scores pairs r, r+W, ... in chunks of 8 pairs) and one all-gather of the member
    losses. Strong scaling: the population is fixed. Timed with CUDA events, max over
    ranks. The ES update every rank then applies (rank-4*512 GEMMs over every weight) is
    timed separately."""
    import torch
    import torch.distributed as dist

    from zotitan_b200 import kernels as K
    from zotitan_b200.distributed import gather_pair_values, local_pairs
    from zotitan_b200.eggroll import EggrollConfig, EggrollPopulation
    from zotitan_b200.synthetic import LLAMA_8B, build_llama, linear_flops_per_token
    model = build_llama(LLAMA_8B, device=dev, seed=0, max_positions=1024)
    pop = EggrollPopulation(model, EggrollConfig(sigma=1e-3))
    g = torch.Generator().manual_seed(7)
    tokens = torch.randint(0, LLAMA_8B.vocab, (4, 256), generator=g).to(dev)
    mine = local_pairs(total_pairs, rank, world)
    pop.evaluate(tokens, list(range(10_000, 10_000 + pairs_per_chunk)))   # warm-up chunk (other seeds)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    local = pop.evaluate_all(tokens, mine, pairs_per_chunk).view(-1, 2)
    rows = gather_pair_values(local, total_pairs, rank, world) if world > 1 else local
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    # the ES update every rank applies after the all-gather: rank-4*512 GEMMs over all 2-D
    # tensors of the model, timed on its own after an untimed warm-up (W unchanged by it)
    all_pairs = list(range(total_pairs))
    coefs = [((j % 7) - 3) / (7.0 * total_pairs) for j in all_pairs]
    pop.apply_update(all_pairs, [0.0] * total_pairs, lr=1e-6)
    torch.cuda.synchronize()
    u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    u0.record()
    pop.apply_update(all_pairs, coefs, lr=1e-6)
    u1.record()
    torch.cuda.synchronize()
    upd_ms = u0.elapsed_time(u1)
    err = K.eggroll_take_error()
    if world > 1:
        t = torch.tensor([ms, upd_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, upd_ms = t.tolist()
    members = 2 * total_pairs
    tokens_per_member = tokens.numel()
    lin_flops = linear_flops_per_token(LLAMA_8B) * tokens_per_member * members
    mean_loss = float(rows.mean())
    del pop, model
    torch.cuda.empty_cache()
    return {"metric": "EGGROLL member-evals/s (Llama-3-8B shape)", "value": members / (ms * 1e-3),
            "unit": "member-evals/s", "members": members, "members_per_rank": 2 * len(mine),
            "tokens_per_member": tokens_per_member, "sigma": 1e-3, "rank": 4, "scaling": "strong",
            "ms": ms, "linear_tflops": lin_flops / (ms * 1e-3) / 1e12, "device_error": err,
            "mean_loss": mean_loss, "es_update_ms": upd_ms, "es_update_pairs": total_pairs,
            "es_step_members_per_s": members / ((ms + upd_ms) * 1e-3)}


def mezo_full_ft_steps(dev, rank: int, world: int, steps: int = 3, warmup: int = 2, pairs: int = 8):
    """ZO steps/s of MeZO full fine-tuning on the Llama-3.2-1B-shaped bf16 model (tied
    embeddings, N(0,0.02) weights from seed 0): 8 antithetic pairs per step sharded over
    the ranks (rank r scores pairs r, r+W, ...), each pair on its own 16 x 512 batch of
    uniform random tokens (batch of pair j at step t from seed 1000*t + j), next-token
    CE + 1e-4 z-loss through the fused CUDA scorer, eps = 1e-3, lr = 1e-5. One step =
    2 forwards per local pair (transformers' Llama with the fused RMSNorm, RoPE and
    SwiGLU forwards of zotitan_b200.llama_fused; on one GPU `graphed_forwards` times the
    same steps with the forwards replayed from CUDA graphs by GraphedScore) + the fused
    perturb/restore/update passes + the all-gather
    of the pair losses (and, with W > 1, the sharded update's parameter all-gather).
    Batches are built on the device before the timed region. Timed with CUDA events
    over `steps` steps, max over ranks; weak in pairs per rank only when W divides 8."""
    import torch
    import torch.distributed as dist

    from zotitan_b200.data import synthetic_token_batch
    from zotitan_b200.graphs import GraphedScore
    from zotitan_b200.objective import SyntheticTokensObjective
    from zotitan_b200.synthetic import LLAMA_1B, build_llama
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer
    from zotitan_b200.llama_fused import fuse_llama
    B, S = 16, 512
    model = build_llama(LLAMA_1B, device=dev, seed=0, max_positions=S)
    fuse_llama(model)   # fused RMSNorm / in-place RoPE / SwiGLU in the no-grad forwards
    objective = SyntheticTokensObjective(LLAMA_1B.vocab, S, z_loss_weight=1e-4)
    cfg = ZOConfig()
    cfg.eps, cfg.z_batch, cfg.base.lr = EPS, pairs, 1e-5
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    opt = ZOOptimizer(named, cfg, objective.score, total_steps=steps + warmup)
    mine = set(range(rank, pairs, world))

    def batches_for(t):
        return [synthetic_token_batch(LLAMA_1B.vocab, B, S, 1000 * t + j, device=dev) if j in mine else None
                for j in range(pairs)]

    plan = [batches_for(t) for t in range(warmup + steps)]

    def timed(opt):
        for t in range(warmup):
            opt.step(model, plan[t])
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for t in range(warmup, warmup + steps):
            m = opt.step(model, plan[t])
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1)
        if world > 1:
            tt = torch.tensor([ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        return ms, m

    ms, m = timed(opt)   # the default path: forwards issued from Python
    cached = opt.zcache is not None
    opt.close()
    del opt
    # the same steps with the noise cache set the other way (default: on when it fits)
    ms_nc, _ = timed(ZOOptimizer(named, cfg, objective.score, total_steps=steps + warmup, noise_cache=not cached))
    graphed = None
    if world == 1:   # the forwards replayed from CUDA graphs (zotitan_b200.graphs.GraphedScore, opt-in)
        try:
            ms_g, _ = timed(ZOOptimizer(named, cfg, GraphedScore(objective.score), total_steps=steps + warmup))
            graphed = {"value": steps / (ms_g * 1e-3), "ms_per_step": ms_g / steps}
        except RuntimeError as e:   # reported, not fatal: the headline path is the eager one
            graphed = {"error": str(e)[:200]}
    n_params = sum(p.numel() for _, p in named)
    del model, named, plan
    torch.cuda.empty_cache()
    return {"metric": "ZO steps/s (MeZO full fine-tune, Llama-3.2-1B shape)", "value": steps / (ms * 1e-3),
            "unit": "ZO steps/s", "ms_per_step": ms / steps, "steps": steps, "warmup": warmup,
            "pairs_per_step": pairs, "forwards_per_step": 2 * pairs, "batch": B, "seq_len": S,
            "tokens_per_step": 2 * pairs * B * S, "params": n_params, "z_loss": 1e-4,
            "scorer": "fused linear cross-entropy (zt_linear_xent: lm_head GEMM + CE statistics in one kernel)", "parallelism": f"pair-sharded x{world}",
            "loss_last_step": m["loss"], "proj_grad_last_step": m["proj_grad"],
            "noise_cache": cached, "graphed_forwards": graphed,
            ("no_noise_cache" if cached else "with_noise_cache"): {
                "value": steps / (ms_nc * 1e-3), "ms_per_step": ms_nc / steps, "cache_bytes": 4 * n_params}}


def mezo_adam_lora_steps(dev, rank: int, world: int, steps: int = 3, warmup: int = 2):
    """ZO steps/s of MeZO-Adam with seed-window momentum (K = 16 past seeds) and second
    moment on rank-16 LoRA adapters (q/k/v/o/gate/up/down, fp32, A ~ N(0, 1/r), B = 0) of
    the Llama-3-8B-shaped bf16 model: one antithetic pair per step (z_batch = 1), next-token
    CE on an 8 x 1024 batch of uniform random tokens (pair batch of step t from seed t),
    eps = 1e-3, lr = 1e-5, beta1 = 0.9, beta2 = 0.999. One step = 2 forwards of the
    LoRA-wrapped model + the fused perturb/restore passes + the last pass replaying the
    16-step seed window (momentum rebuilt in registers) with the Adam update, over the
    448 adapter tensors (41,943,040 fp32 parameters). z_batch = 1 gives nothing to shard:
    with W > 1 every rank runs its own replica and the slowest rank's time is reported."""
    import torch
    import torch.distributed as dist

    from zotitan_b200.data import synthetic_token_batch
    from zotitan_b200.lora import LoRAConfig, make_lora, trainable_params
    from zotitan_b200.objective import SyntheticTokensObjective
    from zotitan_b200.synthetic import LLAMA_8B, build_llama
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer
    from zotitan_b200.llama_fused import fuse_llama
    B, S, r = 8, 1024, 16
    model = build_llama(LLAMA_8B, device=dev, seed=0, max_positions=S)
    make_lora(model, LoRAConfig(r=r, alpha=32, dtype="fp32"))
    fuse_llama(model)   # fused RMSNorm / in-place RoPE / SwiGLU in the no-grad forwards
    g = torch.Generator(device=dev).manual_seed(1)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if "lora_A" in n:
                p.normal_(0.0, (1.0 / r) ** 0.5, generator=g)
    objective = SyntheticTokensObjective(LLAMA_8B.vocab, S)
    cfg = ZOConfig()
    cfg.eps, cfg.z_batch, cfg.base.lr = EPS, 1, 1e-5
    cfg.mom.momentum_method, cfg.mom.beta1, cfg.mom.beta2, cfg.mom.second_moment = "seed_window", 0.9, 0.999, True
    cfg.seed_window.size = 16
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    group = None
    if world > 1:   # a one-rank group per rank: every rank is an independent replica
        groups = [dist.new_group([r]) for r in range(world)]
        group = groups[rank]
    opt = ZOOptimizer(named, cfg, objective.score, total_steps=steps + warmup + 16, process_group=group)
    plan = [[synthetic_token_batch(LLAMA_8B.vocab, B, S, t, device=dev)] for t in range(warmup + steps)]
    for t in range(warmup):
        opt.step(model, plan[t])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for t in range(warmup, warmup + steps):
        m = opt.step(model, plan[t])
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    n_train, n_total = trainable_params(model)
    n_tensors = len(named)
    del opt, model, named, plan
    torch.cuda.empty_cache()
    return {"metric": "ZO steps/s (MeZO-Adam, seed window 16, LoRA r16 on Llama-3-8B shape)",
            "value": steps / (ms * 1e-3), "unit": "ZO steps/s", "ms_per_step": ms / steps, "steps": steps,
            "warmup": warmup, "batch": B, "seq_len": S, "trainable_params": n_train, "trainable_tensors": n_tensors,
            "total_params": n_total, "parallelism": f"replicas x{world}", "loss_last_step": m["loss"],
            "proj_grad_last_step": m["proj_grad"]}


# ── our arm ─────────────────────────────────────────────────────────────────────────

class PassTimer:
    """CUDA events on the launching stream around every fused pass of the timed steps,
    grouped by kind, with each launch's algorithmic bytes (bf16 parameters):
      plus    +eps pass (one stream storing its field, or regenerating it): theta read and
              written (the master read and the live copy written when sharded), + 4 B of z
              per element written to the noise cache;
      perturb -2eps pass: theta read and written, + 4 B of z read from the cache;
      accum   restore of pair j (z_j from the cache) + its grad_est term + perturb of pair
              j+1 (z_{j+1} regenerated and cached): theta and grad_est read and written,
              z read and written (16 B per element; 8 without the cache);
      replay  the step's last pass (on this rank's share, chunk by chunk, when sharded):
              theta read and written, + 4 B per element for every field read from memory
              (noise cache or field store)."""

    KINDS = ("plus", "perturb", "accum", "replay")

    def __init__(self, opt, esz: int = 2):
        import torch
        self.torch = torch
        self.opt, self.esz = opt, esz
        self.events = {k: [] for k in self.KINDS}
        self.on, self.launches = False, 0
        layout = opt.layout
        self.n_units = int(opt.table.plan.n_units)
        self.numel = opt.table.numel
        # elements per unit range: tensors are unit-aligned back to back
        sizes = [p.numel() for p in opt.table.params]
        self.unit_elems = np.zeros(self.n_units, dtype=np.int64)
        u = 0
        for n in sizes:
            k = (n + 2047) // 2048
            self.unit_elems[u:u + k] = 2048
            if n % 2048:
                self.unit_elems[u + k - 1] = n % 2048
            u += k
        self.cum = np.concatenate([[0], np.cumsum(self.unit_elems)])
        self.layout = layout
        self._orig = opt.table.run
        opt.table.run = self.run

    @staticmethod
    def kind(cfg, streams) -> str:
        if cfg.update:
            return "replay"
        if any(s.ge_dev for s in streams):
            return "accum"
        if len(streams) == 1 and streams[0].chain and streams[0].chain[0] < 0:
            return "perturb"
        return "plus"

    def launch_bytes(self, cfg, streams) -> tuple[int, int]:
        ub, ue = cfg.unit_begin, cfg.unit_end
        ue = self.n_units if ue <= 0 or ue > self.n_units else ue
        elems = int(self.cum[ue] - self.cum[ub])
        dst = bin(cfg.dst).count("1")
        per = self.esz * (1 + dst + int(cfg.ge_load) + int(cfg.ge_store))
        per += 4 * sum(1 for st in streams if st.z_load or st.z_store or st.z_field is not None)
        return elems, elems * per

    def run(self, cfg, streams):
        if not self.on:
            return self._orig(cfg, streams)
        self.launches += 1
        k = self.kind(cfg, streams)
        elems, nbytes = self.launch_bytes(cfg, streams)
        a = self.torch.cuda.Event(enable_timing=True)
        b = self.torch.cuda.Event(enable_timing=True)
        a.record()
        self._orig(cfg, streams)
        b.record()
        self.events[k].append((a, b, elems, nbytes))

    def summary(self, steps: int) -> dict:
        out = {}
        for k, evs in self.events.items():
            if not evs:
                continue
            ms = [a.elapsed_time(b) for a, b, _, _ in evs]
            nbytes = [x for _, _, _, x in evs]
            elems = [e for _, _, e, _ in evs]
            out[k] = {"launches_per_step": len(evs) / steps, "ms_per_launch": float(np.mean(ms)),
                      "ms_per_step": float(np.sum(ms)) / steps,
                      "bytes_per_launch": float(np.mean(nbytes)), "elems_per_launch": float(np.mean(elems)),
                      "gbs": float(np.sum(nbytes)) / (float(np.sum(ms)) * 1e-3) / 1e9,
                      "g_elem_per_s": float(np.sum(elems)) / (float(np.sum(ms)) * 1e-3) / 1e9}
        return out


def global_pair_score(vals, planner, seeds: int):
    """Synthetic pair values indexed by the global pair: the k-th score call of a step on
    this rank belongs to its (k // 2)-th own pair, sign k % 2. Every rank count then scores
    pair j with the same two values, so the runs are comparable across N."""
    from zotitan_b200.objective import Score
    state = {"k": 0}

    def score(model, batch):
        local = planner.local
        k = state["k"]
        state["k"] = (k + 1) % (2 * len(local))
        j = local[k // 2]
        return Score(vals[2 * j + (k % 2)], {})
    return score


def param_digest(tensors):
    """Per-tensor int64 sum of the bf16 bit patterns (as int16): equal digests on every
    rank (and at every GPU count, the schedules being bit-identical) mean equal parameters
    up to a collision of the sums."""
    import torch
    return torch.stack([t.detach().reshape(-1).view(torch.int16).sum(dtype=torch.int64) for t in tensors])


def replicas_identical(digest, world: int):
    import torch.distributed as dist
    if world == 1:
        return True
    allv = [digest.clone() for _ in range(world)]
    dist.all_gather(allv, digest)
    return all(bool((x == allv[0]).all()) for x in allv)


def microbench_variant(args, named, cfg, vals_dev, dev, world, barrier, noise_cache: bool):
    """The kernel microbench again with the noise cache set the other way (noise_cache=False:
    every pass regenerates its fields in registers, three noise evaluations per element and
    pair; True: one). Same seeds, values and steps as the headline run; per-launch CUDA
    events by pass kind."""
    import torch
    import torch.distributed as dist

    from zotitan_b200.train_zo import ZOOptimizer

    opt = ZOOptimizer(named, cfg, None, noise_cache=noise_cache)
    opt.score_fn = global_pair_score(vals_dev, opt.planner, args.seeds)
    rng = np.random.default_rng(12345)
    opt.planner._draw_seeds = lambda n: [int(x) for x in rng.integers(0, 2**64 - 1, n, dtype=np.uint64)]
    timer = PassTimer(opt)
    batches = [None] * args.seeds
    for _ in range(args.warmup):
        opt.step(None, batches)
    barrier()
    timer.on = True
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        opt.step(None, batches)
    t1.record()
    barrier()
    timer.on = False
    ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    passes = timer.summary(args.steps)
    cache_bytes = opt.zcache.numel() * 4 if opt.zcache is not None else 0
    opt.close()
    del opt, timer
    torch.cuda.empty_cache()
    return {"value": args.steps / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms / args.steps,
            "noise_cache": noise_cache, "cache_bytes": cache_bytes, "passes": passes}


def roofline_of(passes: dict, peaks: dict, clk: dict, world: int, traffic_db: dict) -> dict:
    """Roofline of the kind with the largest time per step (the dominant kernel)."""
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    kind = max(passes, key=lambda k: passes[k]["ms_per_step"])
    p = passes[kind]
    achieved = p["bytes_per_launch"] / (p["ms_per_launch"] * 1e-3) / 1e9
    entry = traffic_db.get(kind, {})
    traffic = entry.get("dram_bytes_per_elem")
    line = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "traffic": traffic * p["elems_per_launch"] if traffic else None,
            "kernel": entry.get("kernel", kind), "kind": kind,
            "algorithmic_bytes_per_launch": p["bytes_per_launch"],
            "share_of_step": p["ms_per_step"] / sum(x["ms_per_step"] for x in passes.values()),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks else "fallback 6650 GB/s"}
    wi = entry.get("warp_inst_per_elem")
    sm = clk.get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)
    if wi:
        issue = p["elems_per_launch"] * wi / (p["ms_per_launch"] * 1e-3)
        line["issue"] = {"achieved_warp_inst_per_s": issue, "peak": 4 * 148 * sm * 1e6,
                         "frac": issue / (4 * 148 * sm * 1e6), "warp_inst_per_elem": wi,
                         "note": "4 warp-instructions per clock per SM x 148 SMs x the median sampled SM clock; "
                                 "instructions per element from ncu (profiles/pass_kernel_traffic.json)"}
    if entry.get("note"):
        line["note"] = entry["note"]
    return line


def traffic_key(kind: str, cached: bool, exchange: bool) -> str:
    if kind == "replay" and exchange:
        return "replay+field"
    return kind + ("+cache" if cached else "")


def run_ours(args, rank, local_rank, world):
    import hashlib

    import torch
    import torch.distributed as dist

    from zotitan_b200.synthetic import LLAMA_1B, llama_param_shapes, make_params, numel as count
    from zotitan_b200.train_zo import ZOConfig, ZOOptimizer

    shapes = llama_param_shapes(LLAMA_1B)
    cpu_line, ref_c1 = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_line = cpu_port_baseline(count(shapes), len(shapes), args.seeds)   # before any CUDA work
        ref_c1 = reference_config1_subprocess()     # the reference's own CPU step, in the background

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from zotitan_b200.distributed import init_process_group_from_env
        init_process_group_from_env("nccl", timeout_s=300)

    named = make_params(shapes, torch.bfloat16, dev, seed=0)
    numel = sum(p.numel() for _, p in named)
    n_tensors = len(named)
    cfg = ZOConfig()
    cfg.eps, cfg.z_batch, cfg.base.lr = EPS, args.seeds, LR

    # synthetic pair values (no forward in this microbench), indexed by global pair
    g = torch.Generator().manual_seed(1)
    vals_host = (2.0 + 0.01 * torch.randn(2 * args.seeds, generator=g)).float()
    vals_dev = vals_host.to(dev)
    vals_pinned = vals_host.pin_memory()

    class HostVals:   # e2e: each value arrives from pinned host memory
        def __getitem__(self, i):
            return vals_pinned[i:i + 1].to(dev, non_blocking=True)[0]

    opt = ZOOptimizer(named, cfg, None, field_exchange=args.field_exchange or False, exchange_mode=args.exchange_mode,
                      push_order=args.push_order, push_streams=args.push_streams,
                      **({"push_after": args.push_after} if args.push_after else {}))
    opt.score_fn = global_pair_score(vals_dev, opt.planner, args.seeds)
    rng = np.random.default_rng(12345)   # seeded uint64 seed stream, identical on every rank
    opt.planner._draw_seeds = lambda n: [int(x) for x in rng.integers(0, 2**64 - 1, n, dtype=np.uint64)]
    timer = PassTimer(opt)
    batches = [None] * args.seeds

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        opt.step(None, batches)
    gpu_uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    clocks = ClockSampler(gpu_uuid)
    barrier()
    clocks.start()
    timer.on = True
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    stored_per_step = []      # the field exchange's stored-pair count of each timed step
    for _ in range(args.steps):
        if opt.exchange is not None:
            stored_per_step.append(opt.exchange.active)
        opt.step(None, batches)
    t1.record()
    barrier()
    timer.on = False
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    passes = timer.summary(args.steps)
    launches = timer.launches

    # e2e: the same steps through the public API with every pair value copied from pinned host memory
    opt.score_fn = global_pair_score(HostVals(), opt.planner, args.seeds)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        m = opt.step(None, batches)
    e1.record()
    barrier()
    wall_e2e = time.perf_counter() - w0
    e2e_ms = e0.elapsed_time(e1)

    digest = param_digest([p for _, p in named])
    same = replicas_identical(digest, world)
    pdig = hashlib.sha256(digest.cpu().numpy().tobytes()).hexdigest()[:16]
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
        # the dominant kind is the one with the largest max-over-ranks time per step
        for k in sorted(passes):
            t = torch.tensor([passes[k]["ms_per_step"], passes[k]["ms_per_launch"]], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            passes[k]["ms_per_step"], passes[k]["ms_per_launch"] = t.tolist()
    cached = opt.zcache is not None
    exchange = {"mode": "in_pass" if opt.exchange.in_pass else "copies", "push_order": opt.exchange.push_order,
                "push_after": opt.push_after,
                "slots": opt.exchange.n_slots,
                "pairs_stored": opt.exchange.active, "pairs_stored_per_step": stored_per_step,
                "store_bytes": opt.exchange.store.numel() * 4} if opt.exchange is not None else None
    opt.close()
    del opt, timer
    torch.cuda.empty_cache()
    # the other schedule: every field regenerated in registers (or cached, if the default was off)
    alt = microbench_variant(args, named, cfg, vals_dev, dev, world, barrier, noise_cache=not cached)
    # release the microbench's buffers, then the EGGROLL population measurement (all ranks)
    del named
    torch.cuda.empty_cache()
    egg = eggroll_member_evals(dev, rank, world) if not args.no_eggroll else None
    mezo = mezo_full_ft_steps(dev, rank, world) if not args.no_mezo else None
    lora = mezo_adam_lora_steps(dev, rank, world) if not args.no_lora else None
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    torch.cuda.empty_cache()
    ref_gpu = reference_gpu_microbench(args.seeds) if world == 1 and not args.no_reference_gpu else None

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    traffic_db = {}
    try:
        db = json.load(open(os.path.join(HERE, "profiles", "pass_kernel_traffic.json"))).get("kinds", {})
        for k in PassTimer.KINDS:
            key = traffic_key(k, cached, exchange is not None)
            if key in db:
                traffic_db[k] = db[key]
    except (OSError, ValueError):
        pass
    roof = roofline_of(passes, peaks, clk, world, traffic_db)
    value = args.steps / (ms * 1e-3)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": workload_config(world, args.seeds, numel, n_tensors),
        "noise_cache": cached, "field_exchange": exchange,
        "passes": passes,
        "perturb_pass_gbs": passes.get("perturb", {}).get("gbs"),
        "roofline": roof,
        "clocks": clk,
        "gpu_launches": launches,
        "e2e": {"value": args.steps / (e2e_ms * 1e-3), "unit": UNIT, "wall_value": args.steps / wall_e2e,
                "h2d_bytes_per_step": 4 * 2 * args.seeds, "d2h_bytes_per_step": 4 * 2 * args.seeds},
        "replicas_identical": same, "param_digest": pdig,
        "metrics_last_step": {k: m[k] for k in ("loss", "proj_grad")},
    }
    line["no_noise_cache" if cached else "noise_cache_variant"] = alt
    if cpu_line is not None:
        line["cpu_baseline"] = cpu_line
    if ref_c1 is not None:
        line["cpu_baseline"]["reference_code_config1"] = ref_c1()
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
    if egg is not None:
        line["eggroll"] = egg
    if mezo is not None:
        line["mezo_full_ft"] = mezo
    if lora is not None:
        line["mezo_adam_lora"] = lora
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    rank, local_rank, world = env_rank()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    if args.eggroll_gemm:
        eggroll_gemm_bench()
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    main()
