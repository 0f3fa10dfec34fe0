"""Small Llama-shaped models and token batches shared by the golden-vector
generator and the tests. Weights: ``torch.manual_seed(seed)`` then every
parameter ``normal_(0, 0.02)`` in ``named_parameters`` order (the benchmark
initialisation for synthetic Llama models)."""
from __future__ import annotations

import torch

TOY = dict(vocab_size=64, hidden_size=16, intermediate_size=32, num_hidden_layers=2,
           num_attention_heads=2, num_key_value_heads=1, max_position_embeddings=64,
           tie_word_embeddings=False)

# The reference's CPU MeZO workload: Llama 4L/d256/4H/FFN1024/V4096, fp32, untied.
C1 = dict(vocab_size=4096, hidden_size=256, intermediate_size=1024, num_hidden_layers=4,
          num_attention_heads=4, num_key_value_heads=4, max_position_embeddings=256,
          tie_word_embeddings=False)


def build_llama(shape: dict, dtype=torch.float32, seed: int = 0, device="cpu"):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(**shape, attn_implementation="sdpa")
    torch.manual_seed(seed)
    model = LlamaForCausalLM(cfg)
    torch.manual_seed(seed)
    with torch.no_grad():
        for _, p in model.named_parameters():
            p.normal_(0.0, 0.02)
    return model.to(device=device, dtype=dtype).eval()


def token_batch(vocab: int, batch: int, seq: int, seed: int, device="cpu") -> dict:
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq), generator=g)
    return {"input_ids": ids.to(device), "labels": ids.clone().to(device)}


def torch_xentropy_score(model, batch, z_loss_weight: float = 0.0):
    """Cross-entropy + z-loss + accuracy over the LM head, same arithmetic as the
    reference's torch path (zotitan/losses.py:55-79, zotitan/objective.py:87-95).
    Returns (value, metrics) with 0-dim tensors."""
    out = model(**batch)
    loss = out.loss
    logits = out.logits[:, :-1, :]
    labels = batch["labels"][:, 1:]
    mask = labels != -100
    correct = (logits.argmax(-1) == labels) & mask
    metrics = {"ce": loss, "acc": correct.sum() / mask.sum().clamp_min(1)}
    if z_loss_weight == 0.0:
        return loss, metrics
    lse = torch.logsumexp(logits.float(), dim=-1)
    z_loss = z_loss_weight * (lse.square() * mask).sum() / mask.sum().clamp_min(1)
    metrics["z_loss"] = z_loss
    return loss + z_loss, metrics
