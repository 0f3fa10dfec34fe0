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
contiguous block of rows). ``zt_eggroll_factors`` draws A_i, B_i and c for every pair of
a chunk in one launch (||P Psi||_F^2 = sum((P^T P) * (Psi Psi^T)), a 4x4 product).
The rest of a decoder layer runs as fused bandwidth-bound kernels on the population rows:
RMSNorm with per-member weights (``zt_eggroll_rmsnorm``), the rotary embedding in place
(``zt_eggroll_rope``) and the SwiGLU product (``zt_eggroll_swiglu``); attention is the
model's own configured implementation. Embedding rows are perturbed per member directly.

The reference names EGGROLL (README.md:11) but has no implementation; this module is
the population forward the optimizer's fitness-shaping path (train_zo.py:474-508,
:568-578) scores.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn as nn

from . import kernels as K

RANK = 4


@dataclass
class EggrollConfig:
    sigma: float = 1e-3
    """Perturbation scale."""
    normalize: bool = True
    """Scale each low-rank direction to ||z||_F = sqrt(numel), as the reference's low_rank branch does."""
    cuda_graphs: bool = False
    """Capture the chunk forward once per (batch shape, pairs) in a CUDA graph and replay it for
    every later chunk: the pair seeds live in device memory and the kernels derive their keys
    there, so a chunk costs one seed copy, one token copy and one graph launch on the host
    (0.1 ms instead of ~180 ms of Python per 16-member chunk of the 8B shape). Off by
    default: on one B200 the eager enqueue already runs ahead of the GPU, and the replayed
    chunk measured 235 ms against 223-226 ms eager; it pays where host cores are scarce."""


def _key(seed: int, n: int, idx: int) -> int:
    return ((seed * n + idx) & 0xFFFFFFFFFFFFFFFF) & 0x7FFFFFFF


class _Population:
    """The member chunk being evaluated: its pair seeds and rows per member."""

    def __init__(self, n_params: int, cfg: EggrollConfig):
        self.n_params = n_params
        self.cfg = cfg
        self.pair_seeds: list[int] = []
        self.rows_per_member = 0
        self.seeds_dev: torch.Tensor | None = None   # int64 [ZT_EGGROLL_MAX_PAIRS]: the pairs' uint64 seeds
        self._seed_bufs: dict = {}                     # one per device; captured graphs keep their address

    def set_pairs(self, pair_seeds: list[int], device) -> None:
        """Make pair_seeds the current pairs, on the host and in device memory (a copy
        ordered on the current stream, so kernels and graph replays launched after it
        see the new seeds)."""
        from . import _lib as L
        if len(pair_seeds) > L.ZT_EGGROLL_MAX_PAIRS:
            raise ValueError(f"at most {L.ZT_EGGROLL_MAX_PAIRS} pairs at a time")
        device = torch.device(device)
        self.pair_seeds = list(pair_seeds)
        if device not in self._seed_bufs:
            with torch.inference_mode(False):   # a normal tensor: written by no-grad and inference code alike
                self._seed_bufs[device] = torch.zeros(L.ZT_EGGROLL_MAX_PAIRS, dtype=torch.int64, device=device)
        self.seeds_dev = self._seed_bufs[device]
        if pair_seeds:
            bits = [(int(v) & 0xFFFFFFFFFFFFFFFF) - (1 << 64) if (int(v) & (1 << 63)) else int(v) & 0xFFFFFFFFFFFFFFFF
                    for v in pair_seeds]
            host = torch.tensor(bits, dtype=torch.int64).pin_memory()
            self.seeds_dev[:len(bits)].copy_(host, non_blocking=True)

    def dev_seeds(self, *indices: int):
        """The (seeds, n_params, *indices) argument of the kernels' device-key form."""
        return (self.seeds_dev[:len(self.pair_seeds)], self.n_params, *indices)

    @property
    def members(self) -> int:
        return 2 * len(self.pair_seeds)

    def keys(self, idx: int) -> list[int]:
        return [_key(s, self.n_params, idx) for s in self.pair_seeds]

    def use_ext(self, rows: int) -> bool:
        """Whether the rank-4 terms run as a tensor-core K-slab: needs 256-row GEMM tiles
        that each lie inside one member."""
        return rows % 256 == 0 and self.rows_per_member % 256 == 0

    def low_rank(self, idx: int, out_f: int, in_f: int, device, dtype=torch.bfloat16, ext_slot=None, bt=None,
                 bt_row: int = 0):
        """A [members, out, 4], B [members, in, 4] (fp32 holding dtype-rounded values) and
        the signed scale [members] of tensor idx for the current chunk (zt_eggroll_factors:
        one launch for the factors of every pair plus one for the normalisation); with
        ext_slot also A's bf16 K-slab rows, with bt also B^T into rows bt_row.. of bt."""
        return K.eggroll_factors(None, None, out_f, in_f, self.cfg.sigma, device, dtype, self.cfg.normalize,
                                 ext_slot=ext_slot, b_ext=bt, b_ext_row=bt_row,
                                 dev_seeds=self.dev_seeds(idx + 2 * self.n_params, idx + self.n_params))


class PopLinear(nn.Module):
    def __init__(self, base: nn.Linear, idx: int, pop: _Population):
        super().__init__()
        if base.bias is not None:
            raise NotImplementedError("EGGROLL linear layers without bias only (Llama)")
        self.weight = base.weight
        self.idx, self.pop = idx, pop

    def factors(self, device, ext_slot=None, bt=None, bt_row: int = 0):
        out_f, in_f = self.weight.shape
        return self.pop.low_rank(self.idx, out_f, in_f, device, self.weight.dtype, ext_slot, bt, bt_row)

    def forward(self, x, fac=None, xb=None, xe=None):
        """fac = the factors and xb = X B (fp32) or xe = its K-slab rows, from a shared
        zt_eggroll_xb call over x; or None to compute them here."""
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).contiguous()
        out_f = self.weight.shape[0]
        rpm = self.pop.rows_per_member
        if fac is None:
            if self.pop.use_ext(x2.shape[0]):
                bt = torch.zeros((x2.shape[0] // rpm, 16, x2.shape[1]), dtype=torch.bfloat16, device=x.device)
                fac = self.factors(x.device, 0, bt, 0)
                xe = K.eggroll_xb_ext(x2, [fac[1]], [fac[2]], [0], rpm, bt=bt)[0]
            else:
                fac = self.factors(x.device)
        if xe is not None:
            y = K.eggroll_linear(x2, self.weight.data, fac[0], None, fac[2], rpm, x_ext=xe, w_ext=fac[3])
        else:
            y = K.eggroll_linear(x2, self.weight.data, fac[0], fac[1], fac[2], rpm, xb=xb, xb_ready=xb is not None)
        return y.view(*shp[:-1], out_f)


def _shared_input(x, linears, pop, slots=None):
    """Factors of every linear reading x and their X B in one pass over x: fp32 X B, or
    the K-slab rows when the tiles allow it (slots as eggroll_xb_ext takes them; slot 2,
    the second half of a shared row, pairs with A_ext slot 1)."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if pop.use_ext(x2.shape[0]):
        slots = slots or [0] * len(linears)
        rpm = pop.rows_per_member
        bt = torch.zeros((x2.shape[0] // rpm, 16, x2.shape[1]), dtype=torch.bfloat16, device=x.device)
        facs = [lin.factors(x.device, 1 if sl == 2 else 0, bt, 4 * i) for i, (lin, sl) in enumerate(zip(linears, slots))]
        xes = K.eggroll_xb_ext(x2, [f[1] for f in facs], [f[2] for f in facs], slots, rpm, bt=bt)
        return x2, facs, [None] * len(linears), xes
    facs = [lin.factors(x.device) for lin in linears]
    xbs = K.eggroll_xb(x2, [f[1] for f in facs], pop.rows_per_member)
    return x2, facs, xbs, [None] * len(linears)


class PopRMSNorm(nn.Module):
    """Llama RMSNorm with member i's weight w + sign_i sigma z_i on member i's rows
    (zt_eggroll_rmsnorm: the member weights and the normalisation in two launches)."""

    def __init__(self, base, idx: int, pop: _Population):
        super().__init__()
        self.weight = base.weight
        self.eps = getattr(base, "variance_epsilon", getattr(base, "eps", 1e-6))
        self.idx, self.pop = idx, pop

    def forward(self, x):
        return K.eggroll_rmsnorm(x.contiguous(), self.weight.data, None, self.pop.cfg.sigma, self.eps,
                                 self.pop.rows_per_member, dev_seeds=self.pop.dev_seeds(self.idx))


class PopAttention(nn.Module):
    """transformers' LlamaAttention with population projections and the rotary embedding
    applied in place by zt_eggroll_rope; the attention itself is the model's configured
    implementation, called exactly as LlamaAttention.forward calls it."""

    _ATTRS = ("config", "layer_idx", "head_dim", "num_key_value_groups", "scaling", "attention_dropout", "is_causal")

    def __init__(self, base, q_proj, k_proj, v_proj, o_proj):
        super().__init__()
        for a in self._ATTRS:
            setattr(self, a, getattr(base, a))
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = q_proj, k_proj, v_proj, o_proj

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None, **kwargs):
        from transformers.models.llama.modeling_llama import ALL_ATTENTION_FUNCTIONS, eager_attention_forward
        bsz, T, _ = hidden_states.shape
        hd = self.head_dim
        projs = (self.q_proj, self.k_proj, self.v_proj)
        if all(isinstance(p, PopLinear) for p in projs):
            x2, facs, xbs, xes = _shared_input(hidden_states, projs, projs[0].pop)
            q, k, v = (p(x2, f, xb, xe).view(bsz, T, -1) for p, f, xb, xe in zip(projs, facs, xbs, xes))
        else:
            q, k, v = (p(hidden_states) for p in projs)
        cos, sin = position_embeddings
        if cos.shape[0] != 1:
            raise NotImplementedError("per-sequence position ids")
        K.eggroll_rope_(q, k, cos[0].contiguous(), sin[0].contiguous(), T, hd)
        q = q.view(bsz, T, -1, hd).transpose(1, 2)
        k = k.view(bsz, T, -1, hd).transpose(1, 2)
        v = v.view(bsz, T, -1, hd).transpose(1, 2)
        if past_key_values is not None:
            k, v = past_key_values.update(k, v, self.layer_idx)
        attn = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation, eager_attention_forward)
        out, weights = attn(self, q, k, v, attention_mask, dropout=0.0, scaling=self.scaling, **kwargs)
        return self.o_proj(out.reshape(bsz, T, -1).contiguous()), weights


class PopMLP(nn.Module):
    """Llama MLP down(silu(gate(x)) * up(x)) with population projections. Gate, up and
    the SwiGLU product run as one GEMM (zt_eggroll_gated) when the rows split into
    256-row tiles, else as two EGGROLL linears and zt_eggroll_swiglu."""

    def __init__(self, gate_proj, up_proj, down_proj):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    def forward(self, x):
        projs = (self.gate_proj, self.up_proj)
        if all(isinstance(p, PopLinear) for p in projs):
            pop = projs[0].pop
            rows = x.numel() // x.shape[-1]
            if rows % 256 == 0:   # gate, up and SwiGLU in one GEMM (zt_eggroll_gated)
                x2, facs, xbs, xes = _shared_input(x, projs, pop, slots=[1, 2])
                h = K.eggroll_gated(x2, self.gate_proj.weight.data, self.up_proj.weight.data, facs[0], facs[1],
                                    xbs[0], xbs[1], pop.rows_per_member, x_ext=xes[0])
                return self.down_proj(h.view(*x.shape[:-1], -1))
            x2, facs, xbs, xes = _shared_input(x, projs, pop)
            g, u = (p(x2, f, xb, xe).view(*x.shape[:-1], -1) for p, f, xb, xe in zip(projs, facs, xbs, xes))
        else:
            g, u = (p(x) for p in projs)
        return self.down_proj(K.eggroll_swiglu(g, u))


class PopEmbedding(nn.Module):
    """Embedding rows of member i: E[t] + sign_i sigma c_i P_i[t] Psi_i, rounded to E's dtype."""

    def __init__(self, base: nn.Embedding, idx: int, pop: _Population):
        super().__init__()
        self.weight = base.weight
        self.idx, self.pop = idx, pop

    def forward(self, ids):
        V, d = self.weight.shape
        A, B, sig = self.pop.low_rank(self.idx, V, d, ids.device, self.weight.dtype)   # A [m, V, 4], B [m, d, 4]
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
        self.named = named
        self.pop = _Population(len(named), self.cfg)
        self._graphs: dict = {}
        from transformers.models.llama import modeling_llama as ml
        replaced = set()

        def lin(mod):
            replaced.add(index[id(mod.weight)])
            return PopLinear(mod, index[id(mod.weight)], self.pop)

        done_prefixes: list[str] = []
        for name, mod in list(model.named_modules()):
            if any(name.startswith(p) for p in done_prefixes):
                continue
            new = None
            if isinstance(mod, ml.LlamaAttention):
                new = PopAttention(mod, *(lin(getattr(mod, a)) for a in ("q_proj", "k_proj", "v_proj", "o_proj")))
            elif isinstance(mod, ml.LlamaMLP):
                if getattr(mod.config, "hidden_act", "silu") != "silu":
                    raise NotImplementedError("EGGROLL MLP: SiLU gating only")
                new = PopMLP(*(lin(getattr(mod, a)) for a in ("gate_proj", "up_proj", "down_proj")))
            elif isinstance(mod, nn.Linear) and id(mod.weight) in index:
                new = lin(mod)
            elif isinstance(mod, nn.Embedding) and id(mod.weight) in index:
                new = PopEmbedding(mod, index[id(mod.weight)], self.pop)
                replaced.add(index[id(mod.weight)])
            elif isinstance(mod, ml.LlamaRMSNorm) and id(mod.weight) in index:
                new = PopRMSNorm(mod, index[id(mod.weight)], self.pop)
                replaced.add(index[id(mod.weight)])
            if new is None:
                continue
            done_prefixes.append(name + ".")
            parent = model
            *path, leaf = name.split(".")
            for p in path:
                parent = getattr(parent, p)
            setattr(parent, leaf, new)
        missing = [n for i, (n, _) in enumerate(named) if i not in replaced]
        if missing:
            raise NotImplementedError(f"no population module for trainable tensors: {missing[:4]}")

    @torch.inference_mode()
    def evaluate(self, tokens: torch.Tensor, pair_seeds: list[int]) -> torch.Tensor:
        """Next-token cross-entropy of every member on the shared batch ``tokens`` [S, T]
        (members 2j, 2j+1 from pair_seeds[j] with signs +1, -1). Returns [2*len(pair_seeds)]
        fp32 losses, each the mean over the member's S*(T-1) predicted tokens. With
        cfg.cuda_graphs on a CUDA device, the first chunk of a shape is captured and every
        later one replays the graph."""
        S, T = tokens.shape
        pop = self.pop
        pop.set_pairs(pair_seeds, tokens.device)
        pop.rows_per_member = S * T
        if not (self.cfg.cuda_graphs and tokens.is_cuda):
            return self._forward(tokens)
        key = (S, T, pop.members, tokens.device)
        entry = self._graphs.get(key)
        if entry is None:
            static_tokens = tokens.clone()
            side = torch.cuda.Stream(tokens.device)
            side.wait_stream(torch.cuda.current_stream(tokens.device))
            with torch.cuda.stream(side):       # warm-up outside the capture (one-time setup calls)
                self._forward(static_tokens)
            torch.cuda.current_stream(tokens.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = self._forward(static_tokens)
            entry = self._graphs[key] = (graph, static_tokens, out)
        graph, static_tokens, out = entry
        static_tokens.copy_(tokens)
        graph.replay()
        return out.clone()

    def _forward(self, tokens: torch.Tensor) -> torch.Tensor:
        S, T = tokens.shape
        P = self.pop.members
        ids = tokens.repeat(P, 1)                                   # [P*S, T]
        hidden = self.model.model(input_ids=ids, use_cache=False).last_hidden_state   # [P*S, T, d]
        logits = self.model.lm_head(hidden)                          # [P*S, T, V] bf16
        V = logits.shape[-1]
        tgt = torch.full_like(ids, -100)
        tgt[:, :-1] = ids[:, 1:]
        ce, _, _ = K.xent_rows(logits.view(-1, V), tgt.view(-1), want_lse=False, want_correct=False)
        return ce.view(P, -1).sum(dim=1) / (S * (T - 1))

    # -- the evolution-strategies step ------------------------------------------------

    def evaluate_all(self, tokens: torch.Tensor, pair_seeds: list[int], chunk_pairs: int = 8) -> torch.Tensor:
        """evaluate() over pair_seeds in chunks of chunk_pairs pairs: [2*len(pair_seeds)] losses."""
        out = [self.evaluate(tokens, pair_seeds[c:c + chunk_pairs]) for c in range(0, len(pair_seeds), chunk_pairs)]
        return torch.cat(out) if out else torch.empty(0, device=tokens.device)

    @torch.no_grad()
    def apply_update(self, pair_seeds: list[int], coefs: list[float], lr: float):
        """theta <- theta - lr * sum_j coefs[j] * z_j over every trainable tensor, z_j the
        pair's direction: c_j P_j Psi_j for 2-D tensors (the reference's normalised
        low_rank z, train_zo.py:304-320) and the Gaussian field for 1-D ones (:303).

        2-D tensors take the sum as one GEMM of rank 4 * pairs on the tensor cores:
        [A_hi | A_lo] [B | B]^T with A = (coef_j c_j P_j)_j split into two bf16 parts
        (~2^-16 relative) and B = (Psi_j^T)_j (bf16-exact), accumulated in fp32 and added to
        the weight in the GEMM's epilogue (zt_gemm_addto; torch's addmm for shapes it does
        not take), rounded to the parameter dtype once (the reference accumulates grad_est
        in that dtype pair by pair)."""
        if len(pair_seeds) != len(coefs):
            raise ValueError("one coefficient per pair")
        if not pair_seeds:
            return
        pop = self.pop
        dev = self.named[0][1].device
        coef = torch.tensor(coefs, dtype=torch.float32, device=dev)
        saved = pop.pair_seeds
        pop.set_pairs(pair_seeds, dev)
        sigma = float(np.float32(self.cfg.sigma))
        # fp32 accumulation end to end in the update GEMMs (no bf16 split-K partial sums)
        matmul_flags = torch.backends.cuda.matmul
        reduced = matmul_flags.allow_bf16_reduced_precision_reduction
        matmul_flags.allow_bf16_reduced_precision_reduction = False
        try:
            self._apply(pair_seeds, coef, lr, sigma, dev)
        finally:
            pop.set_pairs(saved, dev)
            matmul_flags.allow_bf16_reduced_precision_reduction = reduced

    def _apply(self, pair_seeds, coef, lr, sigma, dev):
        pop = self.pop
        alpha = -float(np.float32(lr))
        for i, (_, p) in enumerate(self.named):
            w = p.data
            if w.dim() == 2:
                a, b, scale, *_ = pop.low_rank(i, w.shape[0], w.shape[1], dev, w.dtype)
                a_cat, b_cat = K.eggroll_update_operands(a, b, scale, coef, sigma)
                # W <- round(W - lr * a_cat b_cat^T): one tensor-core GEMM whose epilogue reads W,
                # adds the fp32 product scaled by -lr and rounds once (zt_gemm_addto)
                if K.gemm_addto_supported(w, a_cat.shape[1]):
                    K.gemm_addto(w, a_cat, b_cat, alpha)
                else:
                    w.addmm_(a_cat, b_cat.T, beta=1.0, alpha=alpha)
            elif w.dim() == 1:
                z = K.randn_keys(pop.keys(i), w.numel(), dev)                    # [P, numel]
                w.copy_((w.float() + alpha * (coef @ z)).to(w.dtype))
            else:
                raise NotImplementedError("EGGROLL updates 1-D and 2-D tensors")

    def step(self, tokens: torch.Tensor, pair_seeds: list[int], lr: float, strategy: str = "centered_rank",
             normalize_std: bool = True, chunk_pairs: int = 8, group=None) -> dict:
        """One evolution-strategies step: every rank scores its share of the antithetic
        pairs (pairs r, r+W, ...), one all-gather of the member losses, fitness shaping by
        the reference's rules (train_zo.py:475-508: centered ranks, GRPO advantages, or the
        plain (L+ - L-) / (2 sigma)), then the same rank-(4 * pairs) update on every rank."""
        from .distributed import gather_pair_values, local_pairs, world_info
        from .train_zo import StepPlanner, f32, f32_recip
        rank, world = world_info(group)
        Z = len(pair_seeds)
        mine = local_pairs(Z, rank, world)
        local = self.evaluate_all(tokens, [pair_seeds[j] for j in mine], chunk_pairs).view(-1, 2)
        rows = gather_pair_values(local, Z, rank, world, group) if world > 1 else local
        vals = rows.flatten().tolist()
        if strategy == "centered_rank":
            u = StepPlanner._centered_ranks([-v for v in vals])
            g = [u[2 * j + 1] - u[2 * j] for j in range(Z)]
        elif strategy == "grpo":
            mean = sum(vals) / len(vals)
            adv = [mean - v for v in vals]
            if normalize_std:
                std = (sum(a_ * a_ for a_ in adv) / len(adv)) ** 0.5
                adv = [a_ / (std + 1e-8) for a_ in adv]
            g = [adv[2 * j + 1] - adv[2 * j] for j in range(Z)]
        elif strategy == "none":
            inv = f32_recip(2 * self.cfg.sigma)
            g = [float(np.float32(np.float32(np.float32(vals[2 * j]) - np.float32(vals[2 * j + 1])) * np.float32(inv)))
                 for j in range(Z)]
        else:
            raise ValueError(f"unknown fitness strategy {strategy!r}")
        coefs = [f32(gj / Z) for gj in g]
        self.apply_update(pair_seeds, coefs, lr)
        return {"loss": sum(vals) / len(vals), "fit_rms": (sum(x * x for x in g) / Z) ** 0.5,
                "members": 2 * Z}
