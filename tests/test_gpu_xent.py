"""GPU parity of the fused cross-entropy scorer.

zt_xent_rows against torch on the fp32 upcast of the same bf16 logits (cross_entropy with
reduction="none", logsumexp, first-occurrence argmax): loss and lse within 2e-5
relative + 2e-5 absolute (the row sums are reduced in a different order), argmax hits
exact, ignored rows zero. losses.fused_xentropy against the reference's torch path
(losses.torch_xentropy) on a bf16 toy Llama: ce and z_loss within 1e-3 relative.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from zotitan_b200 import kernels as K  # noqa: E402


def _torch_rows(logits, tgt):
    x = logits.float()
    mask = tgt >= 0
    safe = tgt.clamp_min(0)
    loss = F.cross_entropy(x, safe, reduction="none") * mask
    lse = torch.logsumexp(x, dim=-1) * mask
    correct = ((x.argmax(-1) == safe) & mask).int()
    return loss, lse, correct


@pytest.mark.parametrize("rows,vocab,ld", [(64, 128256, 128256), (300, 1003, 1008), (7, 8, 8), (1, 4096, 4096)])
def test_xent_rows_match_torch(rows, vocab, ld):
    g = torch.Generator(device="cuda").manual_seed(rows + vocab)
    full = (torch.randn(rows, ld, device="cuda", generator=g) * 4).bfloat16()
    logits = full[:, :vocab]
    tgt = torch.randint(0, vocab, (rows,), device="cuda", generator=g)
    tgt[::5] = -100
    # ties at the maximum: first occurrence must win
    if vocab >= 16:
        logits[1::3, vocab // 2] = 60.0
        logits[1::3, vocab - 1] = 60.0
        tgt[1::6] = vocab // 2
        tgt[4::6] = vocab - 1
    loss, lse, correct = K.xent_rows(logits, tgt)
    want_loss, want_lse, want_correct = _torch_rows(logits, tgt)
    torch.testing.assert_close(loss, want_loss, rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(lse, want_lse, rtol=2e-5, atol=2e-5)
    assert torch.equal(correct, want_correct)
    only_loss, no_lse, no_corr = K.xent_rows(logits, tgt, want_lse=False, want_correct=False)
    assert no_lse is None and no_corr is None and torch.equal(only_loss, loss)


def test_fused_scorer_matches_torch_path():
    from toy_models import build_llama, token_batch
    from zotitan_b200.losses import fused_xentropy, torch_xentropy
    shape = dict(vocab_size=4096, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=4, max_position_embeddings=256, tie_word_embeddings=False)
    model = build_llama(shape, dtype=torch.bfloat16, seed=0, device="cuda")
    batch = token_batch(4096, 8, 128, seed=3, device="cuda")
    batch["labels"][0, :10] = -100
    with torch.inference_mode():
        ce, z, extra = fused_xentropy(model, batch, 1e-4, True)
        ce_t, z_t, extra_t = torch_xentropy(model, batch, 1e-4, True)
    assert abs(float(ce) - float(ce_t)) <= 1e-3 * abs(float(ce_t))
    assert abs(float(z) - float(z_t)) <= 1e-3 * abs(float(z_t))
    n = int((batch["labels"][:, 1:] != -100).sum())
    assert abs(float(extra["acc"]) - float(extra_t["acc"])) <= 2.0 / n
    with torch.inference_mode():
        ce2, z2, extra2 = fused_xentropy(model, batch, 0.0, False)
    assert z2 is None and extra2 is None and abs(float(ce2) - float(ce)) <= 1e-6 * abs(float(ce))
