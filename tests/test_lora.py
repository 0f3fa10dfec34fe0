"""LoRA adapter surface (mirror of zotitan/lora.py) on a toy Llama, CPU only."""
import torch

from zotitan_b200.lora import LoRAConfig, LoRALinear, make_lora, merge_and_unload, merged_state_dict, trainable_params
from zotitan_b200.synthetic import LlamaShape, lora_param_shapes, numel


SHAPE = dict(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, max_position_embeddings=64, tie_word_embeddings=False)


def _model():
    from toy_models import build_llama
    return build_llama(SHAPE, dtype=torch.float32, seed=0, device="cpu")


def test_make_lora_wraps_targets_and_freezes_base():
    model = make_lora(_model(), LoRAConfig(r=4, alpha=8))
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    shape = LlamaShape(vocab=256, d_model=64, layers=2, heads=4, kv_heads=2, ffn=128, tied=False)
    want = lora_param_shapes(shape, r=4)
    assert [n for n, _ in named] == [n.replace(".lora_", ".lora_") for n, _ in want]
    assert [tuple(p.shape) for _, p in named] == [s for _, s in want]
    assert trainable_params(model)[0] == numel(want)
    assert all(p.dtype == torch.float32 for _, p in named)
    assert sum(isinstance(m, LoRALinear) for m in model.modules()) == 7 * 2


def test_adapter_forward_and_merge():
    torch.manual_seed(3)
    model = make_lora(_model(), LoRAConfig(r=4, alpha=8))
    with torch.no_grad():
        for n, p in model.named_parameters():
            if "lora_B" in n:
                p.normal_(0, 0.05)
    ids = torch.randint(0, 256, (2, 16))
    m = model.model.layers[0].self_attn.q_proj
    x = torch.randn(3, 64)
    want = m.base_linear(x) + (x @ m.lora_A.weight.T @ m.lora_B.weight.T) * 2.0
    torch.testing.assert_close(m(x), want, rtol=1e-5, atol=1e-5)
    with torch.no_grad():
        out = model(input_ids=ids).logits
        sd = merged_state_dict(model)
        merged = merge_and_unload(model)
        out2 = merged(input_ids=ids).logits
    torch.testing.assert_close(out, out2, rtol=1e-4, atol=1e-4)
    assert "model.layers.0.self_attn.q_proj.weight" in sd and not any("lora_" in k for k in sd)
    assert not any(isinstance(x_, LoRALinear) for x_ in merged.modules())
