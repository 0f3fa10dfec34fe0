"""Host-side pieces of the CUDA-graph score replay, on CPU: the capture key and the
causal-mask switch of the fused attention (zotitan_b200.graphs, zotitan_b200.llama_fused)."""
import torch

from zotitan_b200 import llama_fused
from zotitan_b200.graphs import GraphedScore, _key


def test_capture_key_follows_shapes_not_values():
    m = object()
    a = {"input_ids": torch.zeros(2, 8, dtype=torch.long), "labels": torch.ones(2, 8, dtype=torch.long)}
    b = {"labels": torch.full((2, 8), 5), "input_ids": torch.full((2, 8), 3)}
    c = {"input_ids": torch.zeros(2, 9, dtype=torch.long), "labels": torch.zeros(2, 9, dtype=torch.long)}
    assert _key(m, a) == _key(m, b)            # same shapes and dtypes, any order or values
    assert _key(m, a) != _key(m, c)            # a new sequence length needs a new graph
    assert _key(m, a) != _key(object(), a)     # graphs hold one model's parameter addresses


def test_assume_causal_is_scoped():
    assert not llama_fused._ASSUME_CAUSAL
    with llama_fused.assume_causal():
        assert llama_fused._ASSUME_CAUSAL
        with llama_fused.assume_causal():
            assert llama_fused._ASSUME_CAUSAL
        assert llama_fused._ASSUME_CAUSAL
    assert not llama_fused._ASSUME_CAUSAL
    try:
        with llama_fused.assume_causal():
            raise RuntimeError("capture failed")
    except RuntimeError:
        pass
    assert not llama_fused._ASSUME_CAUSAL


def test_reset_drops_graphs():
    g = GraphedScore(lambda model, batch: None)
    g._graphs[("k",)] = object()
    g.reset()
    assert g._graphs == {}
