"""Fused CUDA pieces for the no-grad forward of transformers' Llama decoder.

A zeroth-order step evaluates the model 2Z times without gradients (the two
perturbed losses of each pair run under `torch.inference_mode()`,
zotitan/train_zo.py:365-371), and eager transformers runs the decoder's elementwise
work as many separate kernels per layer.
`fuse_llama(model)` swaps the forward of every LlamaRMSNorm, LlamaAttention and
LlamaMLP instance of a model for one that calls this package's kernels:

- RMSNorm: `zt_rmsnorm`, one pass per row (fp32 sum of squares, rsqrt, bf16 round,
  weight product): LlamaRMSNorm.forward with its rounding points; only the summation
  order of a row's squares differs.
- attention: the q/k/v projections (the modules themselves, so LoRA wrappers keep
  working), the rotary embedding applied in place on the projection outputs by
  `zt_eggroll_rope` (bit-exact with apply_rotary_pos_emb), the configured attention
  implementation called as LlamaAttention.forward calls it, then o_proj.
- MLP: for plain bias-free bf16 linears and rows in 256-row tiles, gate, up and the
  SwiGLU as one tcgen05 GEMM (`zt_gemm_swiglu`, the SwiGLU in its epilogue); otherwise
  (LoRA wrappers, ragged rows) the projections as modules and `zt_eggroll_swiglu`
  (bf16(bf16(silu(g)) * u), torch's rounding points). Then the down projection.

Each fused forward defers to the module's own forward when gradients are enabled,
the activations are not bf16 on a CUDA device, the layout does not fit (head_dim not a
multiple of 16, per-sequence position ids), or the MLP's activation is not SiLU.
`unfuse_llama(model)` restores the original forwards.
"""
from __future__ import annotations

import contextlib
import types

import torch
import torch.nn as nn

from . import kernels as K


_ASSUME_CAUSAL = False


@contextlib.contextmanager
def assume_causal():
    """Within this context the fused attention forward ignores the attention mask it is
    given and lets SDPA apply the causal mask itself (`is_causal`). For batches whose
    sequences have no padding, where transformers' mask is purely causal; used while a
    forward is captured into a CUDA graph, when transformers materialises that mask."""
    global _ASSUME_CAUSAL
    prev, _ASSUME_CAUSAL = _ASSUME_CAUSAL, True
    try:
        yield
    finally:
        _ASSUME_CAUSAL = prev


def _fast(x: torch.Tensor) -> bool:
    return (not torch.is_grad_enabled()) and x.is_cuda and x.dtype == torch.bfloat16


def _rmsnorm_forward(self, hidden_states):
    w = self.weight
    if (not _fast(hidden_states) or w.dtype != torch.bfloat16 or hidden_states.shape[-1] % 8
            or not hidden_states.is_contiguous()):
        return self._zt_orig_forward(hidden_states)
    return K.rmsnorm(hidden_states, w.detach(), self.variance_epsilon)


def _attention_forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None,
                       **kwargs):
    cos, sin = position_embeddings if position_embeddings is not None else (None, None)
    hd = self.head_dim
    if (not _fast(hidden_states) or cos is None or cos.shape[0] != 1 or hd % 16 or cos.dtype != torch.bfloat16
            or hidden_states.dim() != 3):
        return self._zt_orig_forward(hidden_states, position_embeddings, attention_mask, past_key_values, **kwargs)
    from transformers.models.llama.modeling_llama import ALL_ATTENTION_FUNCTIONS, eager_attention_forward
    bsz, T, _ = hidden_states.shape
    q = self.q_proj(hidden_states)
    k = self.k_proj(hidden_states)
    v = self.v_proj(hidden_states)
    q = q if q.is_contiguous() else q.contiguous()
    k = k if k.is_contiguous() else k.contiguous()
    # rows of q / k are tokens at positions 0..T-1 of each sequence (cos[0] is shared)
    K.eggroll_rope_(q, k, cos[0].contiguous(), sin[0].contiguous(), T, hd)
    q = q.view(bsz, T, -1, hd).transpose(1, 2)
    k = k.view(bsz, T, -1, hd).transpose(1, 2)
    v = v.view(bsz, T, -1, hd).transpose(1, 2)
    if past_key_values is not None:
        k, v = past_key_values.update(k, v, self.layer_idx)
    if _ASSUME_CAUSAL and past_key_values is None:
        attention_mask = None   # purely causal: SDPA's is_causal (see assume_causal)
    attn = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation, eager_attention_forward)
    out, weights = attn(self, q, k, v, attention_mask, dropout=0.0 if not self.training else self.attention_dropout,
                        scaling=self.scaling, **kwargs)
    return self.o_proj(out.reshape(bsz, T, -1).contiguous()), weights


def is_silu(act) -> bool:
    """torch's SiLU module or transformers' SiLUActivation (both F.silu)."""
    return isinstance(act, nn.SiLU) or type(act).__name__ == "SiLUActivation"


def _plain_linear(m, k: int) -> bool:
    w = getattr(m, "weight", None)
    return (type(m) is nn.Linear and m.bias is None and w is not None and w.dtype == torch.bfloat16
            and w.is_contiguous() and w.shape[1] == k)


def _mlp_forward(self, x):
    if not _fast(x) or not is_silu(self.act_fn):
        return self._zt_orig_forward(x)
    k = x.shape[-1]
    rows = x.numel() // k
    if (_plain_linear(self.gate_proj, k) and _plain_linear(self.up_proj, k) and rows % 256 == 0 and k % 64 == 0
            and self.gate_proj.weight.shape[0] % 128 == 0 and self.gate_proj.weight.shape == self.up_proj.weight.shape):
        # gate, up and SwiGLU in one tcgen05 GEMM (zt_gemm_swiglu)
        x2 = x.reshape(rows, k)
        x2 = x2 if x2.is_contiguous() else x2.contiguous()
        h = K.gemm_swiglu(x2, self.gate_proj.weight.detach(), self.up_proj.weight.detach())
        return self.down_proj(h.view(*x.shape[:-1], -1))
    g = self.gate_proj(x)
    u = self.up_proj(x)
    if g.dtype != torch.bfloat16 or u.dtype != torch.bfloat16 or g.numel() % 8:
        return self.down_proj(self.act_fn(g) * u)
    g = g if g.is_contiguous() else g.contiguous()
    u = u if u.is_contiguous() else u.contiguous()
    return self.down_proj(K.eggroll_swiglu(g, u))


_FORWARDS = {"LlamaRMSNorm": _rmsnorm_forward, "LlamaAttention": _attention_forward, "LlamaMLP": _mlp_forward}


def fuse_llama(model: nn.Module) -> int:
    """Install the fused forwards on every Llama RMSNorm / attention / MLP module of
    `model`; returns how many modules were changed. Idempotent."""
    n = 0
    for m in model.modules():
        fn = _FORWARDS.get(type(m).__name__)
        if fn is None or hasattr(m, "_zt_orig_forward"):
            continue
        m._zt_orig_forward = m.forward
        m.forward = types.MethodType(fn, m)
        n += 1
    return n


def unfuse_llama(model: nn.Module) -> int:
    """Restore the forwards fuse_llama replaced; returns how many modules were restored."""
    n = 0
    for m in model.modules():
        if hasattr(m, "_zt_orig_forward"):
            m.forward = m._zt_orig_forward
            del m._zt_orig_forward
            n += 1
    return n
