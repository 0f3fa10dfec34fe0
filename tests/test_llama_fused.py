"""Host logic of zotitan_b200/llama_fused.py on the CPU: the fused forwards are installed
on the right modules, defer to the modules' own forwards off the GPU (so outputs are
unchanged), and unfuse_llama restores the originals."""
import torch


def _tiny():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def test_fuse_off_gpu_is_transparent():
    from zotitan_b200.llama_fused import fuse_llama, unfuse_llama
    m = _tiny()
    toks = torch.randint(0, 128, (2, 16), generator=torch.Generator().manual_seed(1))
    with torch.inference_mode():
        want = m(toks, use_cache=False).logits
    assert fuse_llama(m) == 2 * 2 + 1 + 2 + 2
    kinds = sorted({type(x).__name__ for x in m.modules() if hasattr(x, "_zt_orig_forward")})
    assert kinds == ["LlamaAttention", "LlamaMLP", "LlamaRMSNorm"]
    with torch.inference_mode():
        got = m(toks, use_cache=False).logits
    assert torch.equal(got, want)
    assert unfuse_llama(m) == 9
    assert not any(hasattr(x, "_zt_orig_forward") for x in m.modules())


def test_llama_activation_is_recognised_as_silu():
    from zotitan_b200.llama_fused import is_silu
    m = _tiny()
    assert is_silu(m.model.layers[0].mlp.act_fn)
    assert is_silu(torch.nn.SiLU()) and not is_silu(torch.nn.GELU())
