#!/usr/bin/env python
"""Time the UNMODIFIED reference (zotitan, installed into baseline/_ref by
baseline/install_reference.sh) through its own ZOOptimizer.step; prints one JSON line.

    python baseline/reference_steps.py cpu-config1
        The reference's CPU MeZO workload: one step of ZOOptimizer.step
        (zotitan/train_zo.py:510-606) on the 4-layer Llama (d 256, 4 heads, FFN 1024,
        vocab 4096, 6.29M fp32 parameters N(0, 0.02) from seed 0), batch 8 x 128 random
        tokens, next-token cross-entropy through the reference's own objective
        (zotitan/objective.py, torch path of zotitan/losses.py:55-79), eps 1e-3, lr 1e-6,
        one pair, seed counter 1234. Its Triton noise kernel (zotitan/train_zo.py:18-28)
        runs under Triton's CPU interpreter (TRITON_INTERPRET=1) and its torch.compile
        wrappers are disabled (TORCHDYNAMO_DISABLE=1): the way the reference runs on a host
        without a GPU. CUDA is hidden from this process.

    python baseline/reference_steps.py gpu-microbench [--seeds 64] [--steps 2] [--warmup 1]
        The kernel microbench workload on the GPU: ZOOptimizer.step over the
        Llama-3.2-1B-shaped parameter set (146 bf16 tensors, 1,235,814,400 parameters,
        N(0, 0.02) from seed 0), 64 pairs per step with seeds from the seeded uint64
        stream the microbench uses (numpy PCG64(12345)), eps 1e-3, lr 1e-6, no forward (the
        pair values are the microbench's synthetic ones, indexed by pair). The reference's
        stock GPU path: native Triton noise, torch foreach ops, _apply_update compiled by
        torch.compile. Timed with CUDA events around the timed steps.

Nothing of zotitan_b200's kernels runs here; the parameter set is built by
zotitan_b200.synthetic (plain torch) so both implementations start from the same tensors.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")


def import_reference():
    if not os.path.isdir(os.path.join(REF, "zotitan")):
        raise SystemExit(json.dumps({"unavailable": "baseline/_ref holds no zotitan install "
                                                    "(run baseline/install_reference.sh)"}))
    sys.path.insert(0, REF)
    import zotitan.train_zo as tz  # noqa: E402
    return tz


def cpu_config1() -> dict:
    import torch
    tz = import_reference()
    from transformers import LlamaConfig, LlamaForCausalLM
    from zotitan.objective import CrossEntropyCriterion, RubricObjective
    threads = int(os.environ.get("REF_CPU_THREADS", "4"))
    torch.set_num_threads(threads)
    shape = dict(vocab_size=4096, hidden_size=256, intermediate_size=1024, num_hidden_layers=4, num_attention_heads=4,
                 num_key_value_heads=4, max_position_embeddings=256, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(LlamaConfig(**shape, attn_implementation="sdpa"))
    torch.manual_seed(0)
    with torch.no_grad():
        for _, p in model.named_parameters():
            p.normal_(0.0, 0.02)
    model = model.float().eval()
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    cfg = tz.ZOConfig()
    cfg.eps, cfg.z_batch, cfg.base.lr = 1e-3, 1, 1e-6
    obj = RubricObjective([(CrossEntropyCriterion(compile_enabled=False, z_loss_weight=0.0, fused=False), 1.0)])
    opt = tz.ZOOptimizer(named, cfg, obj.score)
    opt._seed_ctr = 1234
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 4096, (8, 128), generator=g)
    batch = {"input_ids": ids, "labels": ids.clone()}
    t0 = time.perf_counter()
    with torch.inference_mode():
        metrics = opt.step(model, [batch])
    dt = time.perf_counter() - t0
    n = sum(p.numel() for _, p in named)
    return {"value": 1.0 / dt, "unit": "ZO steps/s", "seconds_per_step": dt, "cores": threads, "kind": "reference",
            "workload": f"reference ZOOptimizer.step, Llama 4L/d256 ({n} fp32 params), batch 8x128, 1 pair, "
                        "Triton interpreter noise (TRITON_INTERPRET=1), torch CPU forward",
            "loss": metrics["loss"], "proj_grad": metrics["proj_grad"]}


def gpu_microbench(seeds: int, steps: int, warmup: int) -> dict:
    import numpy as np
    import torch
    tz = import_reference()
    sys.path.insert(0, ROOT)
    from zotitan_b200.synthetic import LLAMA_1B, llama_param_shapes, make_params
    dev = torch.device("cuda", 0)
    named = make_params(llama_param_shapes(LLAMA_1B), torch.bfloat16, dev, seed=0)
    cfg = tz.ZOConfig()
    cfg.eps, cfg.z_batch, cfg.base.lr = 1e-3, seeds, 1e-6
    g = torch.Generator().manual_seed(1)
    vals = (2.0 + 0.01 * torch.randn(2 * seeds, generator=g)).float().to(dev)
    k = [0]

    class Score:
        def __init__(self, value):
            self.value, self.metrics = value, {}

    def score(model, batch):
        v = vals[k[0] % (2 * seeds)]
        k[0] += 1
        return Score(v)

    opt = tz.ZOOptimizer(named, cfg, score)
    rng = np.random.default_rng(12345)
    # the workload's seed source (a seeded uint64 stream) in place of the step counter
    opt._draw_seeds = lambda n: [int(x) for x in rng.integers(0, 2**64 - 1, n, dtype=np.uint64)]
    batches = [None] * seeds
    t_compile = time.perf_counter()
    for _ in range(warmup):
        opt.step(None, batches)
    torch.cuda.synchronize()
    t_compile = time.perf_counter() - t_compile
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        m = opt.step(None, batches)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    return {"value": 1000.0 / ms, "unit": "ZO steps/s", "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "warmup_s_incl_compile": t_compile, "impl": "reference (unmodified zotitan, baseline/_ref)",
            "how": "ZOOptimizer.step on the GPU: native Triton _philox_randn per tensor and pair, torch foreach "
                   "perturb / restore / grad_est ops, torch.compile'd _apply_update; CUDA events",
            "metrics_last_step": {"loss": m["loss"], "proj_grad": m["proj_grad"]}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["cpu-config1", "gpu-microbench"])
    ap.add_argument("--seeds", type=int, default=64)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    args = ap.parse_args()
    if args.mode == "cpu-config1":
        os.environ["CUDA_VISIBLE_DEVICES"] = ""
        os.environ["TRITON_INTERPRET"] = "1"
        os.environ["TORCHDYNAMO_DISABLE"] = "1"
        out = cpu_config1()
    else:
        out = gpu_microbench(args.seeds, args.steps, args.warmup)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
