"""Cross-entropy scorers over the model's LM head (zotitan/losses.py).

``get_xentropy(fused)`` picks the scorer as the reference does (zotitan/losses.py:7-15):
``fused=True`` -> ``fused_xentropy``: the decoder's hidden states and ``zt_linear_xent``, the
lm_head GEMM on the tensor cores with the per-row loss, logsumexp and first argmax kept in
its epilogue so no logit reaches HBM, in place of the Liger fused linear cross-entropy
(zotitan/losses.py:17-52); heads it cannot take (a bias, other dtypes, an inner dimension
that is not a multiple of 64) go through the lm_head GEMM in row chunks and
``zt_xent_rows`` (one CUDA read of each logits row). ``fused=False`` -> ``torch_xentropy``,
the reference's torch path (zotitan/losses.py:55-79), run eagerly. Both return
(ce, z_loss | None, extra | None) with ce and z_loss kept apart, as the reference's
contract does.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import kernels as K

IGNORE_INDEX = -100
CHUNK_ROWS = 8192


def torch_xentropy(model, batch, z_loss_weight: float, compute_accuracy: bool):
    """Full forward, CE from materialised logits, optional z-loss and accuracy
    (zotitan/losses.py:55-79). Returns (loss, z_loss | None, extra | None)."""
    out = model(**batch)
    loss = out.loss
    extra = None
    if compute_accuracy:
        logits = out.logits[:, :-1, :]
        labels = batch["labels"][:, 1:]
        mask = labels != IGNORE_INDEX
        correct = (logits.argmax(-1) == labels) & mask
        extra = {"acc": correct.sum() / mask.sum().clamp_min(1)}
    if z_loss_weight == 0.0:
        return loss, None, extra
    logits = out.logits[:, :-1, :].float()
    labels = batch["labels"][:, 1:]
    mask = labels != IGNORE_INDEX
    lse = torch.logsumexp(logits, dim=-1)
    z_loss = z_loss_weight * (lse.square() * mask).sum() / mask.sum().clamp_min(1)
    return loss, z_loss, extra


def head_xentropy(hidden: torch.Tensor, targets: torch.Tensor, weight: torch.Tensor, bias=None,
                  want_lse: bool = True, want_correct: bool = True, chunk_rows: int = CHUNK_ROWS):
    """Per-row (loss, lse, correct) of next-token CE for hidden rows [R, d] against
    targets [R] (negative = ignored), logits = bf16(hidden @ weight^T (+ bias)): the fused
    kernel (zt_linear_xent) when it takes the operands, else one chunk of rows at a time
    through the GEMM and zt_xent_rows."""
    if bias is None and K.linear_xent_supported(hidden, weight):
        return K.linear_xent(hidden, weight, targets, want_lse, want_correct)
    R = hidden.shape[0]
    dev = hidden.device
    loss = torch.empty(R, dtype=torch.float32, device=dev)
    lse = torch.empty(R, dtype=torch.float32, device=dev) if want_lse else None
    correct = torch.empty(R, dtype=torch.int32, device=dev) if want_correct else None
    for r0 in range(0, R, chunk_rows):
        r1 = min(R, r0 + chunk_rows)
        logits = F.linear(hidden[r0:r1], weight, bias)
        lo, ls, co = K.xent_rows(logits, targets[r0:r1], want_lse, want_correct)
        loss[r0:r1] = lo
        if want_lse:
            lse[r0:r1] = ls
        if want_correct:
            correct[r0:r1] = co
        del logits
    return loss, lse, correct


def fused_xentropy(model, batch, z_loss_weight: float, compute_accuracy: bool):
    """The fused scorer: decoder forward, causal shift (hidden[:, :-1] predicts
    labels[:, 1:], -100 ignored), head_xentropy. Every position is scored against the next
    label, the last one of each sequence against -100 (ignored), so the hidden states are
    read in place. Same return contract and reductions as the reference's paths:
    ce = mean CE over the unmasked positions, z_loss = z_loss_weight * mean(lse^2),
    acc = mean(argmax == label)."""
    m = getattr(model, "_orig_mod", model)
    hidden = m.get_decoder()(input_ids=batch["input_ids"], attention_mask=batch.get("attention_mask"),
                             use_cache=False).last_hidden_state
    head = m.get_output_embeddings()
    B, S, d = hidden.shape
    shift_h = hidden.reshape(-1, d)
    labels = batch["labels"]
    shift_t = torch.full((B, S), IGNORE_INDEX, dtype=torch.int64, device=labels.device)
    shift_t[:, :-1] = labels[:, 1:]
    shift_t = shift_t.reshape(-1)
    if shift_h.dtype != torch.bfloat16:
        raise NotImplementedError("the fused scorer reads bf16 logits; use fused=False for other dtypes")
    has_z = z_loss_weight != 0.0
    loss, lse, correct = head_xentropy(shift_h, shift_t, head.weight, getattr(head, "bias", None),
                                       want_lse=has_z, want_correct=compute_accuracy)
    mask = shift_t != IGNORE_INDEX
    n = mask.sum().clamp_min(1)
    ce = loss.sum() / n
    extra = {"acc": correct.sum() / n} if compute_accuracy else None
    if not has_z:
        return ce, None, extra
    z_loss = z_loss_weight * (lse.square() * mask).sum() / n
    return ce, z_loss, extra


def get_xentropy(fused: bool, compile_mode: str | None = None):
    """The scorer for (fused, compile_mode) (zotitan/losses.py:7-15). compile_mode is
    accepted for signature compatibility; nothing on this path is compiled."""
    del compile_mode
    return fused_xentropy if fused else torch_xentropy
