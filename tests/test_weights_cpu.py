"""Seeded synthetic weights: layout of the upstream load_weights dict,
determinism, the layer-prefix property, and the RoPE tables."""
import torch

from qwen_weights import LAYER_FIELDS, rope_tables, synthetic_weights


def test_layout_and_prefix(weights_28l):
    w2 = synthetic_weights(seed=1234, num_layers=2)
    assert w2["embed_weight"].shape == (151936, 1024) and w2["embed_weight"].dtype == torch.float16
    assert w2["lm_head_weight"] is w2["embed_weight"]
    assert len(weights_28l["layer_weights"]) == 28 * 11
    for j, (name, shape) in enumerate(LAYER_FIELDS):
        assert tuple(w2["layer_weights"][j].shape) == shape, name
    assert torch.equal(w2["embed_weight"], weights_28l["embed_weight"])
    for a, b in zip(w2["layer_weights"], weights_28l["layer_weights"][:22]):
        assert torch.equal(a, b)
    assert float(weights_28l["layer_weights"][1].float().std()) == pytest_approx(0.02, 0.002)


def pytest_approx(v, tol):
    import pytest
    return pytest.approx(v, abs=tol)


def test_rope_tables_follow_upstream_construction():
    cos, sin = rope_tables(2048)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    freqs = torch.outer(torch.arange(2048, dtype=torch.float32), inv_freq)
    assert torch.equal(cos, torch.cos(freqs).repeat(1, 2).half())
    assert torch.equal(sin, torch.sin(freqs).repeat(1, 2).half())
    assert torch.equal(cos[:, :64], cos[:, 64:])
