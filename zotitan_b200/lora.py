"""LoRA adapters for zeroth-order fine-tuning (zotitan/lora.py).

The reference's adapter surface, kept field for field so configurations carry over:
``LoRAConfig`` (:21-52), ``LoRALinear`` (:55-86: frozen base linear plus trainable A
[r, in] and B [out, r] in the adapter dtype, output base(x) + scale * B(A(x)) cast back to
the base dtype, scale = alpha / r), ``make_lora`` (:89-107: wrap every nn.Linear whose
name ends in a target, freeze everything but the adapters) and the merge helpers
(:117-166). The zeroth-order passes then perturb and update only the adapter tensors
(fp32 by default), in the trainable-list order ``model.named_parameters()`` gives.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Literal

import torch
import torch.nn as nn

DTypeStr = Literal["bf16", "fp32"]

LORA_R = 16
LORA_ALPHA = 32
LORA_TARGETS = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"}

_DTYPES: dict[str, torch.dtype] = {"bf16": torch.bfloat16, "fp32": torch.float32}
_FUSED_R = (4, 8, 16, 32, 64)   # adapter ranks of the fused CUDA tail


@dataclass
class LoRAConfig:
    strategy: Literal["none", "standard", "relora", "continual"] = "none"
    """none: full fine-tuning; standard: adapters merged at the end; relora: cyclic
    merge-and-reinit; continual: merge every step, keeping the wrappers."""
    relora_cycles: int = 5
    r: int = LORA_R
    alpha: int = LORA_ALPHA
    targets: list[str] = field(default_factory=lambda: list(LORA_TARGETS))
    dtype: DTypeStr = "fp32"
    """Adapter dtype; fp32 keeps small perturbations from being rounded away."""
    init: Literal["kaiming", "gaussian"] = "kaiming"
    """lora_A initialisation (lora_B is zero): kaiming_uniform_(a=sqrt(5)) or kaiming_normal_."""


class LoRALinear(nn.Module):
    def __init__(self, base: nn.Linear, r: int, lora_alpha: int, dtype: DTypeStr = "fp32", init: str = "kaiming"):
        super().__init__()
        self.base_linear = base
        base.weight.requires_grad_(False)
        if base.bias is not None:
            base.bias.requires_grad_(False)
        self.lora_dtype = _DTYPES[dtype]
        dev = base.weight.device
        self.lora_A = nn.Linear(base.in_features, r, bias=False, dtype=self.lora_dtype, device=dev)
        self.lora_B = nn.Linear(r, base.out_features, bias=False, dtype=self.lora_dtype, device=dev)
        if init == "kaiming":
            nn.init.kaiming_uniform_(self.lora_A.weight, a=math.sqrt(5))
        else:
            nn.init.kaiming_normal_(self.lora_A.weight)
        nn.init.zeros_(self.lora_B.weight)
        self.scaling = lora_alpha / r

    def forward(self, x):
        out = self.base_linear(x)
        aw, bw = self.lora_A.weight, self.lora_B.weight
        if (not torch.is_grad_enabled() and out.is_cuda and out.dtype == torch.bfloat16 and x.dtype == torch.bfloat16
                and aw.dtype == torch.float32 and bw.dtype == torch.float32 and bw.shape[1] in _FUSED_R
                and out.is_contiguous() and aw.is_contiguous() and bw.is_contiguous()):
            # Gradients off (the zeroth-order step): x A^T on the tensor cores from the bf16
            # activations against A split into three bf16 parts that sum to it exactly
            # (zt_lora_split; each product exact, fp32 accumulation: the fp32 product up to
            # summation order), then the three partial products summed and lora_B(xa) *
            # scaling cast to bf16 and added to `out` in one pass (zt_lora_add3), with the
            # reference's rounding points. Three launches; no autograd record is made.
            from . import kernels as K
            r, n = bw.shape[1], out.shape[-1]
            a3 = K.lora_split(aw.detach()).view(3 * r, -1)                                # [3r, in] bf16
            x2 = x.reshape(-1, x.shape[-1])
            xa3 = torch.mm(x2, a3.T, out_dtype=torch.float32)                               # [rows, 3r]
            K.lora_add3_(out.view(-1, n), xa3, bw.detach(), self.scaling)   # sums the 3 parts, then the tail
            return out
        xa = self.lora_A(x.to(self.lora_dtype))
        delta = self.lora_B(xa) * self.scaling
        return out + delta.to(out.dtype)


def make_lora(model, cfg: LoRAConfig | None = None):
    """Wrap the target linears with adapters and freeze every other parameter."""
    cfg = cfg or LoRAConfig()
    targets = set(cfg.targets)
    for name, module in list(model.named_modules()):
        if not isinstance(module, nn.Linear) or not any(name.endswith(t) for t in targets):
            continue
        *path, leaf = name.split(".")
        parent = model
        for part in path:
            parent = getattr(parent, part)
        setattr(parent, leaf, LoRALinear(module, cfg.r, cfg.alpha, cfg.dtype, cfg.init))
    for name, p in model.named_parameters():
        if "lora_A" not in name and "lora_B" not in name:
            p.requires_grad_(False)
    return model


def trainable_params(model) -> tuple[int, int]:
    """(trainable, total) parameter counts."""
    return (sum(p.numel() for p in model.parameters() if p.requires_grad),
            sum(p.numel() for p in model.parameters()))


def _delta(m: LoRALinear) -> torch.Tensor:
    return m.lora_B.weight @ m.lora_A.weight


@torch.no_grad()
def merge_and_unload(model):
    """Fold each adapter into its base weight (W += scale * B A) and restore nn.Linear."""
    for name, m in list(model.named_modules()):
        if not isinstance(m, LoRALinear):
            continue
        *path, leaf = name.split(".")
        parent = model
        for part in path:
            parent = getattr(parent, part)
        m.base_linear.weight.data.add_(_delta(m), alpha=m.scaling)
        setattr(parent, leaf, m.base_linear)
    return model


@torch.no_grad()
def merge_and_zero_lora(model):
    """Fold each adapter into its base weight and zero lora_B, keeping the wrappers."""
    for m in model.modules():
        if isinstance(m, LoRALinear):
            m.base_linear.weight.data.add_(_delta(m), alpha=m.scaling)
            m.lora_B.weight.data.zero_()


@torch.no_grad()
def merged_state_dict(model) -> dict:
    """CPU state dict with the adapters folded in (fp32 merge, cast to the base dtype) and
    plain module names, leaving the live model untouched."""
    out = {}
    for name, m in model.named_modules():
        if isinstance(m, LoRALinear):
            w = (m.base_linear.weight.float() + _delta(m).float() * m.scaling).to(m.base_linear.weight.dtype)
            out[name + ".weight"] = w.cpu()
            if m.base_linear.bias is not None:
                out[name + ".bias"] = m.base_linear.bias.detach().cpu()
    for key, value in model.state_dict().items():
        if ".base_linear." in key or ".lora_A." in key or ".lora_B." in key:
            continue
        out[key] = value.detach().cpu()
    return out
