"""EGGROLL population evaluation on B200: many perturbed members in one forward.

Member i of a population scores the model with every trainable tensor perturbed by a
rank-4 term regenerated from its pair seed s (members 2j and 2j+1 form an antithetic
pair sharing s_j with signs +1 / -1). The perturbation follows the reference's
``low_rank`` branch (zotitan/train_zo.py:304-320), with sigma in place of eps:

  2-D tensor p [out, in] at position i of the n-long trainable list:
      P   = randn(key(s, n, i + 2n), out*4).view(out, 4)   -> A_i = P        (bf16-rounded)
      Psi = randn(key(s, n, i + n),  4*in).view(4, in)     -> B_i = Psi^T    (bf16-rounded)
      p_i = p + sign * sigma * c * P Psi,  c = sqrt(out*in) / (||P Psi||_F + 1e-7)
  1-D tensor p (norm weights):  p_i = p + sign * sigma * randn(key(s, n, i), numel)

The linear layers never materialise p_i: ``zt_eggroll_linear`` computes
x p^T + (sign sigma c) (x B_i) A_i^T with the base GEMM on the tensor cores and the
rank-4 term in its epilogue, for all members of a chunk at once (member i owns a
contiguous block of rows). ||P Psi||_F^2 = sum((P^T P) * (Psi Psi^T)) is a 4x4 product.
Norm weights and the embedding rows are perturbed per member directly.

The reference names EGGROLL (README.md:11) but has no implementation; this module is
the population forward the optimizer's fitness-shaping path (train_zo.py:474-508,
:568-578) scores.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import kernels as K

RANK = 4


@dataclass
class EggrollConfig:
    sigma: float = 1e-3
    """Perturbation scale."""
    normalize: bool = True
    """Scale each low-rank direction to ||z||_F = sqrt(numel), as the reference's low_rank branch does."""


def _key(seed: int, n: int, idx: int) -> int:
    return ((seed * n + idx) & 0xFFFFFFFFFFFFFFFF) & 0x7FFFFFFF


class _Population:
    """The member chunk being evaluated: pair seeds, signs and per-tensor caches."""

    def __init__(self, n_params: int, cfg: EggrollConfig):
        self.n_params = n_params
        self.cfg = cfg
        self.pair_seeds: list[int] = []
        self.rows_per_member = 0
        self.signs = None            # [members] fp32 (+1, -1, +1, -1, ...)

    @property
    def members(self) -> int:
        return 2 * len(self.pair_seeds)

    def low_rank(self, idx: int, out_f: int, in_f: int, device):
        """A [members, out, 4], B [members, in, 4] (fp32 holding bf16 values) and the signed
        scale [members] of tensor idx for the current chunk."""
        n = self.n_params
        kp = [_key(s, n, idx + 2 * n) for s in self.pair_seeds]
        kq = [_key(s, n, idx + n) for s in self.pair_seeds]
        P = K.randn_keys(kp, out_f * RANK, device).view(-1, out_f, RANK).bfloat16().float()
        Psi = K.randn_keys(kq, RANK * in_f, device).view(-1, RANK, in_f).bfloat16().float()
        if self.cfg.normalize:
            fro2 = torch.einsum("prs,prs->p", P.transpose(1, 2) @ P, Psi @ Psi.transpose(1, 2))
            c = (out_f * in_f) ** 0.5 / (fro2.clamp_min(0).sqrt() + 1e-7)
        else:
            c = torch.ones(len(self.pair_seeds), device=device)
        A = P.repeat_interleave(2, dim=0).contiguous()
        B = Psi.transpose(1, 2).repeat_interleave(2, dim=0).contiguous()
        scale = (self.cfg.sigma * c).repeat_interleave(2) * self.signs
        return A, B, scale.float().contiguous()

    def dense(self, idx: int, numel: int, device):
        """Full Gaussian field [members, numel] of a 1-D tensor, signs and sigma applied."""
        z = K.randn_keys([_key(s, self.n_params, idx) for s in self.pair_seeds], numel, device)
        return z.repeat_interleave(2, dim=0) * (self.cfg.sigma * self.signs)[:, None]


class PopLinear(nn.Module):
    def __init__(self, base: nn.Linear, idx: int, pop: _Population):
        super().__init__()
        if base.bias is not None:
            raise NotImplementedError("EGGROLL linear layers without bias only (Llama)")
        self.weight = base.weight
        self.idx, self.pop = idx, pop

    def forward(self, x):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).contiguous()
        out_f, in_f = self.weight.shape
        A, B, sig = self.pop.low_rank(self.idx, out_f, in_f, x.device)
        y = K.eggroll_linear(x2, self.weight.data, A, B, sig, self.pop.rows_per_member)
        return y.view(*shp[:-1], out_f)


class PopRMSNorm(nn.Module):
    """Llama RMSNorm with member i's weight w + sign_i sigma z_i on member i's rows."""

    def __init__(self, base, idx: int, pop: _Population):
        super().__init__()
        self.weight = base.weight
        self.eps = getattr(base, "variance_epsilon", getattr(base, "eps", 1e-6))
        self.idx, self.pop = idx, pop

    def forward(self, x):
        dt = x.dtype
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.eps)
        d = self.weight.shape[0]
        w = (self.weight.float()[None, :] + self.pop.dense(self.idx, d, x.device)).to(self.weight.dtype)
        P = self.pop.members
        return (w[:, None, :] * h.to(dt).reshape(P, -1, d)).reshape(x.shape)


class PopEmbedding(nn.Module):
    """Embedding rows of member i: E[t] + sign_i sigma c_i P_i[t] Psi_i, rounded to E's dtype."""

    def __init__(self, base: nn.Embedding, idx: int, pop: _Population):
        super().__init__()
        self.weight = base.weight
        self.idx, self.pop = idx, pop

    def forward(self, ids):
        V, d = self.weight.shape
        A, B, sig = self.pop.low_rank(self.idx, V, d, ids.device)   # A [m, V, 4], B [m, d, 4]
        P = self.pop.members
        ids_m = ids.reshape(P, -1)                                  # member i's token ids
        rows = torch.gather(A, 1, ids_m[..., None].expand(-1, -1, RANK))   # [m, tokens, 4]
        delta = (rows @ B.transpose(1, 2)) * sig[:, None, None]            # [m, tokens, d]
        e = self.weight[ids_m].float() + delta
        return e.to(self.weight.dtype).reshape(*ids.shape, d)


class EggrollPopulation:
    """Wraps a HF Llama causal LM for population evaluation (module surgery: its linear,
    RMSNorm and embedding modules are replaced; the model's own attention and MLP code run
    unchanged). ``trainable``: the reference's named-parameter list order (defaults to
    ``model.named_parameters()``), which fixes each tensor's seed index."""

    def __init__(self, model, cfg: EggrollConfig | None = None):
        self.model = model
        self.cfg = cfg or EggrollConfig()
        named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
        index = {id(p): i for i, (_, p) in enumerate(named)}
        self.pop = _Population(len(named), self.cfg)
        norm_types = tuple(t for t in (getattr(__import__("transformers.models.llama.modeling_llama", fromlist=["x"]),
                                               "LlamaRMSNorm", None),) if t is not None)
        replaced = set()
        for name, mod in list(model.named_modules()):
            new = None
            if isinstance(mod, nn.Linear) and id(mod.weight) in index:
                new = PopLinear(mod, index[id(mod.weight)], self.pop)
            elif isinstance(mod, nn.Embedding) and id(mod.weight) in index:
                new = PopEmbedding(mod, index[id(mod.weight)], self.pop)
            elif norm_types and isinstance(mod, norm_types) and id(mod.weight) in index:
                new = PopRMSNorm(mod, index[id(mod.weight)], self.pop)
            if new is None:
                continue
            parent = model
            *path, leaf = name.split(".")
            for p in path:
                parent = getattr(parent, p)
            setattr(parent, leaf, new)
            replaced.add(index[id(mod.weight)])
        missing = [n for i, (n, _) in enumerate(named) if i not in replaced]
        if missing:
            raise NotImplementedError(f"no population module for trainable tensors: {missing[:4]}")

    @torch.inference_mode()
    def evaluate(self, tokens: torch.Tensor, pair_seeds: list[int]) -> torch.Tensor:
        """Next-token cross-entropy of every member on the shared batch ``tokens`` [S, T]
        (members 2j, 2j+1 from pair_seeds[j] with signs +1, -1). Returns [2*len(pair_seeds)]
        fp32 losses, each the mean over the member's S*(T-1) predicted tokens."""
        S, T = tokens.shape
        pop = self.pop
        pop.pair_seeds = list(pair_seeds)
        P = pop.members
        pop.rows_per_member = S * T
        pop.signs = torch.tensor([1.0, -1.0] * len(pair_seeds), device=tokens.device)
        ids = tokens.repeat(P, 1)                                   # [P*S, T]
        hidden = self.model.model(input_ids=ids).last_hidden_state   # [P*S, T, d]
        logits = self.model.lm_head(hidden)                          # [P*S, T, V] bf16
        V = logits.shape[-1]
        ce = F.cross_entropy(logits[:, :-1, :].reshape(-1, V).float(), ids[:, 1:].reshape(-1), reduction="none")
        return ce.view(P, -1).mean(dim=1)
