"""GPU tests of the fused linear cross-entropy (zt_linear_xent).

Against torch on the same operands: logits = F.linear(x, w) in bf16 (the reference's
bf16 lm_head), then loss / logsumexp / first argmax on their fp32 upcast, as
zotitan/losses.py:55-79 computes them. The kernel accumulates the dot products on the
tensor cores in another order than cuBLAS, so a logit can round to the neighbouring
bf16 value: loss and lse agree within 1e-3 relative (the losses' tolerance of the parity bar),
and the argmax flag agrees on all but a handful of near-tied rows. Shapes cover ragged
row and vocabulary counts (partial 256-row tiles, a partial last vocabulary tile), the
config-3 scorer shape (16 x 512 rows, vocabulary 128,256, d 2048), ignored rows and an
out-of-range target (NaN, as zt_xent_rows).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def reference(x, w, t, chunk=4096):
    loss, lse, correct = [], [], []
    for r0 in range(0, x.shape[0], chunk):
        logits = F.linear(x[r0:r0 + chunk], w).float()
        tt = t[r0:r0 + chunk]
        ls = torch.logsumexp(logits, dim=-1)
        valid = (tt >= 0) & (tt < w.shape[0])
        tgt = logits.gather(1, tt.clamp(0, w.shape[0] - 1)[:, None])[:, 0]
        lo = torch.where(valid, ls - tgt, torch.zeros_like(ls))
        lo = torch.where(tt >= w.shape[0], torch.full_like(ls, float("nan")), lo)
        co = ((logits.argmax(-1) == tt) & (tt >= 0)).int()
        loss.append(lo)
        lse.append(torch.where(tt >= 0, ls, torch.zeros_like(ls)))
        correct.append(co)
    return torch.cat(loss), torch.cat(lse), torch.cat(correct)


def operands(rows, vocab, k, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(rows, k, generator=g, device="cuda") * scale).bfloat16()
    w = (torch.randn(vocab, k, generator=g, device="cuda") * 0.02).bfloat16()
    t = torch.randint(0, vocab, (rows,), generator=g, device="cuda")
    return x, w, t


@pytest.mark.parametrize("rows,vocab,k", [(300, 1000, 128), (256, 512, 64), (1, 257, 64), (700, 4096, 256),
                                          (8192, 128256, 2048)])
def test_linear_xent_matches_torch(rows, vocab, k):
    from zotitan_b200 import kernels as K
    x, w, t = operands(rows, vocab, k, seed=rows + vocab)
    if rows > 4:
        t[3] = -100                    # ignored
        t[4] = vocab - 1               # the last column (in the partial last tile when vocab % 256)
    loss, lse, correct = K.linear_xent(x, w, t)
    rl, rs, rc = reference(x, w, t)
    torch.cuda.synchronize()
    assert K.linear_xent_take_error() == 0
    ok = t >= 0
    assert torch.all(loss[~ok] == 0) and torch.all(lse[~ok] == 0) and torch.all(correct[~ok] == 0)
    torch.testing.assert_close(loss[ok], rl[ok], rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(lse[ok], rs[ok], rtol=1e-3, atol=1e-3)
    agree = (correct == rc).float().mean().item()
    assert agree >= 0.999 if rows >= 1000 else int((correct != rc).sum()) <= 1


def test_linear_xent_argmax_first_index_and_outliers():
    """Planted winners: each row's target column gets a large logit, so correct = 1 on
    every row; a tie between two columns resolves to the first; a target >= vocab is NaN."""
    from zotitan_b200 import kernels as K
    rows, vocab, k = 512, 3000, 128
    x, w, t = operands(rows, vocab, k, seed=5)
    # row r's hidden state aligned with w[t_r]: its logit dominates
    x = (w[t].float() * 40.0).bfloat16()
    t2 = t.clone()
    t2[7] = vocab + 3
    loss, lse, correct = K.linear_xent(x, w, t2)
    rl, rs, rc = reference(x, w, t2)
    torch.cuda.synchronize()
    assert torch.isnan(loss[7])
    keep = torch.ones(rows, dtype=torch.bool, device="cuda")
    keep[7] = False
    assert int(correct[keep].sum()) == rows - 1 == int(rc[keep].sum())
    torch.testing.assert_close(loss[keep], rl[keep], rtol=1e-3, atol=1e-3)
    # ties: two identical weight rows, the earlier column wins
    w2 = w.clone()
    w2[2000] = w2[1500]
    x2 = (w2[1500].float()[None, :].expand(8, -1) * 40.0).bfloat16().contiguous()
    t3 = torch.full((8,), 1500, dtype=torch.int64, device="cuda")
    _, _, c3 = K.linear_xent(x2, w2, t3)
    assert torch.all(c3 == 1)
    t3.fill_(2000)
    _, _, c4 = K.linear_xent(x2, w2, t3)
    assert torch.all(c4 == 0)


def test_fused_scorer_uses_the_kernel_and_matches_torch_path():
    """The fused scorer on a bf16 Llama whose head the kernel takes (d 256, vocab 4096)
    against the reference's torch path (zotitan/losses.py:55-79): ce, z-loss and accuracy
    within 1e-3."""
    from toy_models import C1, build_llama, token_batch
    from zotitan_b200 import kernels as K
    from zotitan_b200.losses import fused_xentropy, torch_xentropy
    model = build_llama(C1, dtype=torch.bfloat16, seed=0, device="cuda")
    batch = token_batch(C1["vocab_size"], 4, 128, seed=3, device="cuda")
    calls = {"n": 0}
    orig = K.linear_xent

    def counting(*a, **kw):
        calls["n"] += 1
        return orig(*a, **kw)

    K.linear_xent = counting
    try:
        with torch.inference_mode():
            ce, zl, ex = fused_xentropy(model, batch, 1e-4, True)
            ce_r, zl_r, ex_r = torch_xentropy(model, batch, 1e-4, True)
    finally:
        K.linear_xent = orig
    assert calls["n"] == 1
    assert abs(ce.item() - ce_r.item()) <= 1e-3 * abs(ce_r.item())
    assert abs(zl.item() - zl_r.item()) <= 1e-3 * abs(zl_r.item())
    assert abs(ex["acc"].item() - ex_r["acc"].item()) <= 1e-3
    assert np.isfinite(ce.item())
