"""Fused LoRA forward (x A^T from bf16 x against A split exactly into three bf16 parts on
the tensor cores, then zt_lora_add) against the reference's LoRALinear arithmetic
(zotitan/lora.py:77-86): base(x) + (lora_B(lora_A(x.float())) * scaling).to(bf16).
Bar: >= 99.9% of outputs bit-exact; the rest within one bf16 step of |out| + |delta|
(the fp32 sums are ordered differently from cuBLAS's, which can move the delta's bf16
rounding by one step; where base and delta cancel that step is large against |out|)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("r,n_in,n_out,rows", [(16, 512, 1024, 300), (4, 256, 128, 8), (64, 128, 256, 1000),
                                               (16, 4096, 14336, 64)])
def test_lora_tail_matches_reference(r, n_in, n_out, rows):
    from zotitan_b200.lora import LoRALinear
    g = torch.Generator(device="cuda").manual_seed(r + n_in)
    base = torch.nn.Linear(n_in, n_out, bias=False, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        base.weight.normal_(0, 0.02, generator=g)
    m = LoRALinear(base, r, 2 * r)
    with torch.no_grad():
        m.lora_B.weight.normal_(0, 0.05, generator=g)
    x = torch.randn(2, rows, n_in, device="cuda", generator=g).bfloat16()
    with torch.inference_mode():
        got = m(x)
        want = base(x) + (m.lora_B(m.lora_A(x.float())) * m.scaling).to(torch.bfloat16)
        delta = (m.lora_B(m.lora_A(x.float())) * m.scaling).to(torch.bfloat16)
    d = (got.float() - want.float()).abs()
    bound = 2.0 ** -7 * (want.float().abs() + delta.float().abs()) + 1e-30
    assert bool((d <= bound).all()), float((d / bound).max())
    assert float((d == 0).float().mean()) >= 0.999
    with torch.enable_grad():   # gradients on: the reference's torch path, identical values
        x2 = x.clone().requires_grad_(False)
        assert torch.equal(m(x2), want)
