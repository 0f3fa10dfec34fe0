"""Generate golden vectors by running the REFERENCE's own code on CPU.

Imports zotitan.train_zo / zotitan.objective from the reference checkout and runs
its Triton noise kernel under Triton's interpreter (TRITON_INTERPRET=1) and its
optimizer step eagerly (TORCHDYNAMO_DISABLE=1: the reference's torch.compile
wrappers cannot build on this CPU). Writes:

  ref_noise.npz   _philox_randn(seed, n) (zotitan/train_zo.py:25-28) and the Triton
                  words/Gaussians at the native fixture's offsets, interpreter-evaluated
  ref_sample_z.npz ZOOptimizer._sample_z (zotitan/train_zo.py:295-322), gaussian + low_rank
  ref_steps.npz   ZOOptimizer.step (zotitan/train_zo.py:510-606) on toy Llama models under
                  every optimizer branch: per-forward values/metrics, the perturbed
                  parameters seen by the first two forwards, parameters after each step
  ref_config1.npz one MeZO step of the 4-layer Llama (d256, 6.29M fp32 params):
                  loss / proj_grad and a seeded sample of parameter positions

    python tests/golden/make_golden.py /path/to/reference [--skip-config1]
"""
from __future__ import annotations

import json
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, ".."))
from toy_models import TOY, C1, build_llama, token_batch  # noqa: E402

STEP_CONFIGS = {
    # name: (dtype, lora, steps, kwargs for ZOConfig tree, total_steps)
    "mezo_f32_z1": ("f32", False, 2, dict(z_batch=1, lr=1e-2), 0),
    "mezo_bf16_z3": ("bf16", False, 2, dict(z_batch=3, lr=5e-2), 0),
    "mezo_f32_wsd": ("f32", False, 3, dict(z_batch=2, lr=1e-2, warmup_frac=0.5, decay_frac=0.3), 4),
    "ema_adam_f32_z2": ("f32", False, 3, dict(z_batch=2, lr=1e-3, momentum_method="stored_ema",
                                              second_moment=True), 0),
    "ema_bf16_z1": ("bf16", False, 2, dict(z_batch=1, lr=5e-2, momentum_method="stored_ema"), 0),
    "seedwin_adam_bf16_z2": ("bf16", False, 4, dict(z_batch=2, lr=1e-3, momentum_method="seed_window",
                                                    window=3, second_moment=True), 0),
    "seedwin_f32_z1": ("f32", False, 3, dict(z_batch=1, lr=1e-2, momentum_method="seed_window", window=2), 0),
    "rmsprop_bf16_z1": ("bf16", False, 2, dict(z_batch=1, lr=1e-3, second_moment=True), 0),
    "wd_standard_f32": ("f32", False, 2, dict(z_batch=2, lr=1e-2, wd="standard", wd_lambda=0.5), 0),
    "wd_anchored_l1_bf16": ("bf16", False, 2, dict(z_batch=2, lr=5e-2, wd="anchored", wd_lambda=0.5,
                                                   penalty="l1"), 0),
    "wd_anchored_l2_f32": ("f32", False, 2, dict(z_batch=1, lr=1e-2, wd="anchored", wd_lambda=0.5), 0),
    "clip_per_pair_f32": ("f32", False, 3, dict(z_batch=3, lr=1e-2, clip="per_pair", clip_pct=0.3,
                                                clip_window=10), 0),
    "clip_norm_bf16": ("bf16", False, 3, dict(z_batch=3, lr=5e-2, clip="norm", clip_pct=0.3,
                                              clip_window=10), 0),
    "es_rank_f32": ("f32", False, 2, dict(z_batch=4, lr=1e-2, fitness="centered_rank", shared=True), 0),
    "grpo_bf16": ("bf16", False, 2, dict(z_batch=3, lr=5e-2, fitness="grpo", shared=True), 0),
    "lora_seedwin_adam": ("bf16", True, 3, dict(z_batch=1, lr=1e-3, momentum_method="seed_window",
                                                window=3, second_moment=True), 0),
    "lowrank_f32_z2": ("f32", False, 1, dict(z_batch=2, lr=1e-2, distribution="low_rank", rank=2), 0),
}

Z_LOSS = 1e-4


def make_cfg(tz, kw):
    cfg = tz.ZOConfig()
    cfg.eps = 1e-3
    cfg.z_batch = kw.get("z_batch", 1)
    cfg.shared_batch = kw.get("shared", False)
    cfg.base.lr = kw["lr"]
    cfg.base.lr_wsd.warmup_frac = kw.get("warmup_frac", 0.0)
    cfg.base.lr_wsd.decay_frac = kw.get("decay_frac", 0.0)
    cfg.mom.momentum_method = kw.get("momentum_method", "none")
    cfg.mom.second_moment = kw.get("second_moment", False)
    cfg.seed_window.size = kw.get("window", 0)
    cfg.perturbation.distribution = kw.get("distribution", "gaussian")
    cfg.perturbation.rank = kw.get("rank", 64)
    cfg.clip.strategy = kw.get("clip", "none")
    cfg.clip.clip_pct = kw.get("clip_pct", 0.0)
    cfg.clip.window = kw.get("clip_window", 1000)
    cfg.fitness.strategy = kw.get("fitness", "none")
    cfg.weight_decay.strategy = kw.get("wd", "none")
    cfg.weight_decay.lambda_ = kw.get("wd_lambda", 0.0)
    cfg.weight_decay.penalty = kw.get("penalty", "l2")
    return cfg


def cfg_to_dict(cfg):
    import dataclasses
    return dataclasses.asdict(cfg)


def flat(params):
    return np.concatenate([p.detach().float().reshape(-1).numpy() for p in params])


def run_steps(tz, obj, name, spec):
    dtype_s, lora, n_steps, kw, total = spec
    dtype = torch.bfloat16 if dtype_s == "bf16" else torch.float32
    model = build_llama(TOY, dtype=dtype, seed=0)
    if lora:
        from zotitan.lora import LoRAConfig, make_lora
        torch.manual_seed(1)
        model = make_lora(model, LoRAConfig(strategy="standard", r=2, alpha=4))
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    cfg = make_cfg(tz, kw)
    calls = []

    def score_fn(m, batch):
        s = obj.score(m, batch)
        rec = {"value": float(s.value), **{k: float(v) for k, v in s.metrics.items()}}
        if len(calls) < 2:
            rec["snapshot"] = flat([p for _, p in named])
        calls.append(rec)
        return s

    opt = tz.ZOOptimizer(named, cfg, score_fn, total_steps=total)
    out = {"init": flat([p for _, p in named]),
           "numels": np.array([p.numel() for _, p in named]),
           "names": np.array([n for n, _ in named]),
           "dtypes": np.array([str(p.dtype) for _, p in named])}
    metrics = []
    with torch.inference_mode():
        for step in range(n_steps):
            if cfg.shared_batch:
                b = token_batch(TOY["vocab_size"], 2, 8, seed=1000 * step)
                batches = [b] * cfg.z_batch
            else:
                batches = [token_batch(TOY["vocab_size"], 2, 8, seed=1000 * step + j)
                           for j in range(cfg.z_batch)]
            metrics.append(opt.step(model, batches))
            out[f"after_{step}"] = flat([p for _, p in named])
    out["values"] = np.array([c["value"] for c in calls], dtype=np.float64)
    out["ce"] = np.array([c.get("ce", np.nan) for c in calls], dtype=np.float64)
    out["acc"] = np.array([c.get("acc", np.nan) for c in calls], dtype=np.float64)
    out["z_loss"] = np.array([c.get("z_loss", np.nan) for c in calls], dtype=np.float64)
    out["snap_pos"] = calls[0]["snapshot"]
    out["snap_neg"] = calls[1]["snapshot"]
    out["metrics"] = np.array(json.dumps(metrics))
    out["cfg"] = np.array(json.dumps(cfg_to_dict(cfg)))
    out["spec"] = np.array(json.dumps({"dtype": dtype_s, "lora": lora, "steps": n_steps, "kw": kw,
                                       "total_steps": total, "z_loss": Z_LOSS}))
    return {f"{name}/{k}": v for k, v in out.items()}


def main(ref_root: str, skip_config1: bool):
    sys.path.insert(0, ref_root)
    import triton
    import triton.language as tl  # noqa: F401
    import zotitan.train_zo as tz
    from zotitan.objective import CrossEntropyCriterion, RubricObjective
    sys.path.insert(0, os.path.join(HERE, "..", ".."))
    from oracle import triton_native as tn

    # -- noise ---------------------------------------------------------------
    nat = np.load(os.path.join(HERE, "native_triton_randn.npz"))
    noise = {}
    for key in [0, 1, 7, 1234, 2**31 - 1, 987654321]:
        noise[f"randn_{key}"] = tz._philox_randn(key, 3000, "cpu").numpy()
        offs = torch.from_numpy(nat[f"offs_{key}"])
        noise[f"offs_{key}"] = nat[f"offs_{key}"]
        noise[f"words_{key}"] = tn.words_at(key, offs).numpy().view(np.uint32)
        noise[f"randn_at_{key}"] = tn.randn_at(key, offs).numpy()
    noise["triton_version"] = np.array(triton.__version__)
    np.savez_compressed(os.path.join(HERE, "ref_noise.npz"), **noise)
    print("ref_noise.npz")

    # -- _sample_z ------------------------------------------------------------
    sz = {}
    shapes = [((5, 7), torch.float32), ((33,), torch.bfloat16), ((4, 3), torch.float32), ((6, 8), torch.bfloat16)]
    named = [(f"p{i}", torch.nn.Parameter(torch.zeros(s, dtype=d))) for i, (s, d) in enumerate(shapes)]
    for dist, rank in [("gaussian", 64), ("low_rank", 2)]:
        cfg = tz.ZOConfig()
        cfg.perturbation.distribution = dist
        cfg.perturbation.rank = rank
        opt = tz.ZOOptimizer(named, cfg, None)
        for seed in [0, 5, 2**40 + 3]:
            for i, z in enumerate(opt._sample_z(seed)):
                sz[f"{dist}/{seed}/{i}"] = z.float().numpy()
    np.savez_compressed(os.path.join(HERE, "ref_sample_z.npz"), **sz)
    print("ref_sample_z.npz")

    # -- optimizer steps on toy models ----------------------------------------
    # Anchored weight decay pins theta_0 in host memory (zotitan/train_zo.py:274),
    # which needs a CUDA driver; pinning changes no value, so it is a no-op here.
    torch.Tensor.pin_memory = lambda self, *a, **k: self
    crit = CrossEntropyCriterion(compile_enabled=False, z_loss_weight=Z_LOSS, fused=False)
    obj = RubricObjective([(crit, 1.0)])
    steps = {}
    for name, spec in STEP_CONFIGS.items():
        steps.update(run_steps(tz, obj, name, spec))
        print("step", name)
    np.savez_compressed(os.path.join(HERE, "ref_steps.npz"), **steps)
    print("ref_steps.npz")

    if skip_config1:
        return
    # -- one MeZO step of the 4-layer Llama, 6.29M fp32 params -------------------
    model = build_llama(C1, dtype=torch.float32, seed=0)
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    cfg = tz.ZOConfig()
    cfg.eps, cfg.z_batch, cfg.base.lr = 1e-3, 1, 1e-6
    crit1 = CrossEntropyCriterion(compile_enabled=False, z_loss_weight=0.0, fused=False)
    obj1 = RubricObjective([(crit1, 1.0)])
    vals = []

    def score1(m, b):
        s = obj1.score(m, b)
        vals.append(float(s.value))
        return s

    opt = tz.ZOOptimizer(named, cfg, score1)
    opt._seed_ctr = 1234
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 4096, (8, 128), generator=g)
    batch = {"input_ids": ids, "labels": ids.clone()}
    before = flat([p for _, p in named])
    torch.set_num_threads(8)
    with torch.inference_mode():
        metrics = opt.step(model, [batch])
    after = flat([p for _, p in named])
    rng = np.random.default_rng(0)
    idx = np.sort(rng.choice(before.size, 8192, replace=False))
    numels = np.array([p.numel() for _, p in named])
    starts = np.concatenate([[0], np.cumsum(numels)[:-1]])
    delta_sums = np.array([np.sum((after[s:s + n].astype(np.float64) - before[s:s + n]))
                           for s, n in zip(starts, numels)])
    np.savez_compressed(os.path.join(HERE, "ref_config1.npz"), idx=idx, before=before[idx], after=after[idx],
                        delta_sums=delta_sums, numels=numels, values=np.array(vals),
                        metrics=np.array(json.dumps(metrics)), seed=np.array(1234))
    print("ref_config1.npz", metrics)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if len(args) != 1:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference [--skip-config1]")
    main(args[0], "--skip-config1" in sys.argv)
