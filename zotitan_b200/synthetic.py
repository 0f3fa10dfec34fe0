"""Synthetic Llama-shaped parameter sets for the benchmark workloads.

Names, shapes and order follow ``LlamaForCausalLM.named_parameters()`` so the
per-tensor noise keys (position i in the trainable list) are those a real model
of that shape would get. Weights are N(0, 0.02) from a seeded generator.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LlamaShape:
    vocab: int
    d_model: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    tied: bool

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads


# Benchmark workloads: Llama-3.2-1B shape (tied embeddings) and Llama-3-8B shape (untied)
LLAMA_1B = LlamaShape(vocab=128256, d_model=2048, layers=16, heads=32, kv_heads=8, ffn=8192, tied=True)
LLAMA_8B = LlamaShape(vocab=128256, d_model=4096, layers=32, heads=32, kv_heads=8, ffn=14336, tied=False)

LORA_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def llama_param_shapes(s: LlamaShape) -> list[tuple[str, tuple[int, ...]]]:
    d, kv = s.d_model, s.kv_heads * s.head_dim
    out = [("model.embed_tokens.weight", (s.vocab, d))]
    for i in range(s.layers):
        p = f"model.layers.{i}."
        out += [(p + "self_attn.q_proj.weight", (d, d)), (p + "self_attn.k_proj.weight", (kv, d)),
                (p + "self_attn.v_proj.weight", (kv, d)), (p + "self_attn.o_proj.weight", (d, d)),
                (p + "mlp.gate_proj.weight", (s.ffn, d)), (p + "mlp.up_proj.weight", (s.ffn, d)),
                (p + "mlp.down_proj.weight", (d, s.ffn)),
                (p + "input_layernorm.weight", (d,)), (p + "post_attention_layernorm.weight", (d,))]
    out.append(("model.norm.weight", (d,)))
    if not s.tied:
        out.append(("lm_head.weight", (s.vocab, d)))
    return out


def build_llama(s: LlamaShape, device="cuda", dtype=None, seed: int = 0, max_positions: int = 2048):
    """A transformers LlamaForCausalLM of this shape built directly on `device` in `dtype`
    (bf16 default), every parameter re-drawn N(0, 0.02) from a seeded generator."""
    from transformers import LlamaConfig, LlamaForCausalLM
    dtype = dtype or torch.bfloat16
    cfg = LlamaConfig(vocab_size=s.vocab, hidden_size=s.d_model, intermediate_size=s.ffn, num_hidden_layers=s.layers,
                      num_attention_heads=s.heads, num_key_value_heads=s.kv_heads, tie_word_embeddings=s.tied,
                      max_position_embeddings=max_positions, attn_implementation="sdpa")
    with torch.device(device):
        model = LlamaForCausalLM._from_config(cfg, dtype=dtype)
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for _, p in model.named_parameters():
            p.normal_(0.0, 0.02, generator=g)
    return model.eval()


def linear_flops_per_token(s: LlamaShape) -> float:
    """2 * (sum of in*out over the linear layers, lm_head included): base GEMM FLOPs per token."""
    d, kv = s.d_model, s.kv_heads * s.head_dim
    per_layer = d * d * 2 + d * kv * 2 + 3 * d * s.ffn
    return 2.0 * (s.layers * per_layer + s.vocab * d)


def lora_param_shapes(s: LlamaShape, r: int = 16) -> list[tuple[str, tuple[int, ...]]]:
    """Trainable LoRA adapters (A: [r, in], B: [out, r]) on every q/k/v/o/gate/up/down."""
    out = []
    for name, shape in llama_param_shapes(s):
        mod = name.rsplit(".", 2)[-2] if name.endswith(".weight") else ""
        if mod in LORA_TARGETS:
            base = name[: -len(".weight")]
            out += [(base + ".lora_A.weight", (r, shape[1])), (base + ".lora_B.weight", (shape[0], r))]
    return out


def make_params(shapes, dtype=torch.bfloat16, device="cuda", seed: int = 0, std: float = 0.02):
    """Seeded N(0, std) tensors for a shape list (generated on the device)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for name, shape in shapes:
        t = torch.empty(shape, dtype=dtype, device=device)
        t.normal_(0.0, std, generator=g)
        out.append((name, torch.nn.Parameter(t, requires_grad=True)))
    return out


def numel(shapes) -> int:
    n = 0
    for _, s in shapes:
        k = 1
        for x in s:
            k *= x
        n += k
    return n
