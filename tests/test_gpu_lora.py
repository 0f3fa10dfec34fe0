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


def test_lora_split_parts_sum_exactly():
    """zt_lora_split: the three bf16 parts equal torch's cast-and-subtract chain and sum to
    the fp32 input exactly (checked in fp64)."""
    from zotitan_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(16, 4096, device="cuda", generator=g) * torch.logspace(-6, 2, 4096, device="cuda")
    parts = K.lora_split(a)
    a0 = a.bfloat16()
    rest = a - a0.float()
    a1 = rest.bfloat16()
    a2 = (rest - a1.float()).bfloat16()
    assert torch.equal(parts[0], a0) and torch.equal(parts[1], a1) and torch.equal(parts[2], a2)
    assert torch.equal(parts.double().sum(0), a.double())


@pytest.mark.parametrize("r", [4, 16, 64])
def test_lora_add3_equals_summed_lora_add(r):
    """zt_lora_add3 on three partial products = zt_lora_add on their fp32 sum ((p0+p1)+p2)."""
    from zotitan_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(r)
    rows, n = 300, 1000
    xa3 = torch.randn(rows, 3 * r, device="cuda", generator=g)
    b = torch.randn(n, r, device="cuda", generator=g) * 0.1
    base = torch.randn(rows, n, device="cuda", generator=g).bfloat16()
    want = base.clone()
    K.lora_add_(want, ((xa3[:, :r] + xa3[:, r:2 * r]) + xa3[:, 2 * r:]).contiguous(), b, 2.0)
    got = base.clone()
    K.lora_add3_(got, xa3, b, 2.0)
    assert torch.equal(got, want)
