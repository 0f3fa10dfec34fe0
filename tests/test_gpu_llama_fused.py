"""Fused no-grad forward of transformers' Llama (zotitan_b200/llama_fused.py) against the
modules' own forwards on the same inputs, bf16 on the GPU.

- attention (projections, in-place RoPE, sdpa, o_proj): bit-identical;
- RMSNorm (zt_rmsnorm): >= 99.9% bit-identical, the rest within two bf16 steps (the
  row's sum of squares is added in another order, which can move the rsqrt by an ulp
  and the result across one rounding boundary before the weight product and one after);
- MLP (zt_eggroll_swiglu inside): >= 99% bit-identical, all within a bf16 step of
  |output| plus 2^-7 of the largest partial product magnitude;
- the whole model: next-token cross-entropy within 1e-3 relative of the unfused model,
  logits within a few bf16 steps of their scale.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(layers=2, d=256, heads=4, kv=2, ffn=512, vocab=1000, seed=0):
    from zotitan_b200.synthetic import LlamaShape, build_llama
    return build_llama(LlamaShape(vocab=vocab, d_model=d, layers=layers, heads=heads, kv_heads=kv, ffn=ffn, tied=False),
                       device="cuda", seed=seed, max_positions=512)


def _steps(a, b):
    """|a - b| in bf16 steps at max(|a|, |b|)."""
    a, b = a.float(), b.float()
    scale = torch.maximum(a.abs(), b.abs()).clamp_min(2.0 ** -126)
    ulp = torch.ldexp(torch.ones_like(scale), torch.frexp(scale)[1] - 8)
    return (a - b).abs() / ulp


def test_fuse_counts_and_unfuse():
    from zotitan_b200.llama_fused import fuse_llama, unfuse_llama
    m = _model(layers=3)
    assert fuse_llama(m) == 3 * 2 + 1 + 3 + 3
    assert fuse_llama(m) == 0
    assert unfuse_llama(m) == 13


def test_attention_bit_identical():
    from zotitan_b200.llama_fused import fuse_llama
    m = _model()
    attn = m.model.layers[1].self_attn
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(3, 128, 256, device="cuda", generator=g).bfloat16()
    pos = torch.arange(128, device="cuda")[None]
    cos, sin = m.model.rotary_emb(x, pos)
    with torch.inference_mode():
        want, _ = attn(x, (cos, sin), None)
        fuse_llama(m)
        got, _ = attn(x, (cos, sin), None)
    assert torch.equal(got, want)


def test_rmsnorm_close():
    from zotitan_b200.llama_fused import fuse_llama
    m = _model(d=2048, heads=16, kv=4, ffn=1024)
    norm = m.model.layers[0].input_layernorm
    with torch.no_grad():
        norm.weight.normal_(1.0, 0.1)
    g = torch.Generator(device="cuda").manual_seed(2)
    x = (torch.randn(4096, 2048, device="cuda", generator=g) * 3).bfloat16()
    with torch.inference_mode():
        want = norm(x)
        fuse_llama(m)
        got = norm(x)
    st = _steps(got, want)
    assert float(st.max()) <= 2.0
    assert float((st == 0).float().mean()) >= 0.999


def test_mlp_close():
    from zotitan_b200.llama_fused import fuse_llama
    m = _model()
    mlp = m.model.layers[0].mlp
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(2, 64, 256, device="cuda", generator=g).bfloat16()
    with torch.inference_mode():
        want = mlp(x)
        h = mlp.act_fn(mlp.gate_proj(x)) * mlp.up_proj(x)
        bound = h.float().abs() @ mlp.down_proj.weight.float().abs().T
        fuse_llama(m)
        got = mlp(x)
    d = (got.float() - want.float()).abs()
    ulp = torch.ldexp(torch.ones_like(d), torch.frexp(want.float().abs().clamp_min(2.0 ** -126))[1] - 8)
    assert bool((d <= ulp + 2.0 ** -7 * bound).all())
    assert float((d == 0).float().mean()) >= 0.99


def test_grad_enabled_falls_back():
    from zotitan_b200.llama_fused import fuse_llama
    m = _model()
    toks = torch.randint(0, 1000, (2, 64), device="cuda")
    want = m(toks, use_cache=False).logits
    fuse_llama(m)
    got = m(toks, use_cache=False).logits   # gradients enabled: every module takes its own forward
    assert torch.equal(got, want)


def test_model_loss_close(monkeypatch):
    from zotitan_b200 import kernels as K
    from zotitan_b200.llama_fused import fuse_llama
    calls = {"rmsnorm": 0, "eggroll_rope_": 0, "eggroll_swiglu": 0, "gemm_swiglu": 0}
    for name in calls:
        fn = getattr(K, name)

        def counted(*a, _fn=fn, _name=name, **kw):
            calls[_name] += 1
            return _fn(*a, **kw)
        monkeypatch.setattr(K, name, counted)
    m = _model(layers=4, d=512, heads=8, kv=2, ffn=1024, vocab=4096)
    toks = torch.randint(0, 4096, (4, 256), device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))

    def loss_and_logits():
        with torch.inference_mode():
            lg = m(toks[:, :-1], use_cache=False).logits
            return torch.nn.functional.cross_entropy(lg.float().reshape(-1, 4096), toks[:, 1:].reshape(-1)), lg
    want, lw = loss_and_logits()
    fuse_llama(m)
    got, lg = loss_and_logits()
    # 4 x 255 rows: not whole 256-row tiles, so the MLP takes the two projections and zt_eggroll_swiglu
    assert calls == {"rmsnorm": 2 * 4 + 1, "eggroll_rope_": 4, "eggroll_swiglu": 4, "gemm_swiglu": 0}
    assert abs(float(got) - float(want)) <= 1e-3 * abs(float(want))
    scale = float(lw.float().abs().max())
    assert float((lg.float() - lw.float()).abs().max()) <= 2.0 ** -5 * scale


def test_mlp_gated_gemm_path(monkeypatch):
    """Rows in whole 256-row tiles and plain bf16 linears: gate, up and SwiGLU run as one
    zt_gemm_swiglu; the output is within a bf16 step of |output| plus 2^-6 of the
    partial-product bound of the module's own forward (the GEMM accumulates in another
    order, which can move g or u by one bf16 step)."""
    from zotitan_b200 import kernels as K
    from zotitan_b200.llama_fused import fuse_llama
    calls = {"n": 0}
    fn = K.gemm_swiglu

    def counted(*a, **kw):
        calls["n"] += 1
        return fn(*a, **kw)
    monkeypatch.setattr(K, "gemm_swiglu", counted)
    m = _model()
    mlp = m.model.layers[0].mlp
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(4, 128, 256, device="cuda", generator=g).bfloat16()
    with torch.inference_mode():
        want = mlp(x)
        h = mlp.act_fn(mlp.gate_proj(x)) * mlp.up_proj(x)
        bound = h.float().abs() @ mlp.down_proj.weight.float().abs().T
        fuse_llama(m)
        got = mlp(x)
    assert calls["n"] == 1
    d = (got.float() - want.float()).abs()
    ulp = torch.ldexp(torch.ones_like(d), torch.frexp(want.float().abs().clamp_min(2.0 ** -126))[1] - 8)
    assert bool((d <= ulp + 2.0 ** -6 * bound).all())
