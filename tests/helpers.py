"""Shared test helpers: golden-fixture access and tolerance metrics."""
import json
import os
from types import SimpleNamespace

import numpy as np

from oracle import philox as ph

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def ns(d):
    """dict tree -> attribute tree (a ZOConfig look-alike for the oracle)."""
    return SimpleNamespace(**{k: ns(v) if isinstance(v, dict) else v for k, v in d.items()})


def load(name):
    return np.load(os.path.join(GOLDEN, name))


class StepCase:
    """One recorded reference run from ref_steps.npz."""

    def __init__(self, G, name):
        g = lambda k: G[f"{name}/{k}"]  # noqa: E731
        self.name = name
        self.cfg_dict = json.loads(str(g("cfg")))
        self.cfg = ns(self.cfg_dict)
        self.spec = json.loads(str(g("spec")))
        self.numels = [int(x) for x in g("numels")]
        self.names = [str(x) for x in g("names")]
        self.dtypes = [ph.BF16 if "bfloat16" in d else ph.F32 for d in g("dtypes")]
        self.init = g("init")
        self.values = [float(x) for x in g("values")]
        self.snap_pos, self.snap_neg = g("snap_pos"), g("snap_neg")
        self.after = [g(f"after_{s}") for s in range(self.spec["steps"])]
        self.metrics = json.loads(str(g("metrics")))
        starts = np.concatenate([[0], np.cumsum(self.numels)[:-1]])
        self.starts = [int(s) for s in starts]

    def shapes(self):
        from toy_models import TOY, build_llama
        model = build_llama(TOY, seed=0)
        shapes = {n: tuple(p.shape) for n, p in model.named_parameters()}
        out = []
        for n in self.names:
            if "lora_A" in n or "lora_B" in n:
                base = shapes[n.replace(".lora_A.weight", ".weight").replace(".lora_B.weight", ".weight")]
                out.append((2, base[1]) if "lora_A" in n else (base[0], 2))
            else:
                out.append(shapes[n])
        return out

    def params(self):
        return [self.init[s:s + n].reshape(sh).copy() for s, n, sh in zip(self.starts, self.numels, self.shapes())]


def step_cases():
    G = load("ref_steps.npz")
    names = sorted({k.split("/")[0] for k in G.files})
    return G, names


def scale_ulps(a, b, before, dtypes_per_elem):
    """|a-b| in units of the param dtype's ulp at max(|a|, |b|, |before|)."""
    sc = np.maximum(np.maximum(np.abs(a), np.abs(b)), np.abs(before)).astype(np.float32)
    mant = np.where(dtypes_per_elem == ph.BF16, 7, 23)
    ulp = np.exp2(np.floor(np.log2(np.maximum(sc, 1e-30))) - mant)
    return np.abs(a.astype(np.float64) - b.astype(np.float64)) / ulp


def flat(ps):
    return np.concatenate([np.asarray(p, dtype=np.float32).reshape(-1) for p in ps])
