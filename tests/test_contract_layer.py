"""Contract of the MoE layer seam and the HF decoder-layer swap.

Follows the reference's ``tests/test_moe_layer.py`` and the router checks of
``tests/test_engine.py``: ``MoELayer.forward`` takes ``[tokens, hidden]`` or
``[batch, seq, hidden]`` and keeps token order, refuses other ranks and hidden
sizes with ``ValueError``; ``MoEInfraDecoderLayer.set_moe`` installs the layer
behind ``MoELayerAdapter`` and the HF decoder layer runs with it; the
``_ensure_expert_on_gpu`` seam (``model/moe_layer.py:39-115``) lets test
experts replace the NF4 experts while the real router, dispatch and ordered
fp16 combine run (GPU), matching the oracle of ``model/moe_layer.py:147-191``.
"""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from moeinfra_b200.engine.decoder_layer import MoEInfraDecoderLayer, MoELayerAdapter
from moeinfra_b200.model.moe_layer import MoELayer


def _small_mixtral_config(hidden=64, heads=4, kv=2):
    from transformers import MixtralConfig

    return MixtralConfig(hidden_size=hidden, intermediate_size=2 * hidden, num_hidden_layers=2,
                         num_attention_heads=heads, num_key_value_heads=kv, num_local_experts=4,
                         num_experts_per_tok=2, vocab_size=32)


def test_forward_keeps_token_order_for_3d_input(monkeypatch):
    moe = MoELayer(0, None, None, None, None)
    monkeypatch.setattr(moe, "_forward_tokens", lambda h: h * 3.0 - 1.0)
    h = torch.arange(2 * 5 * 4, dtype=torch.float32).reshape(2, 5, 4)
    torch.testing.assert_close(moe.forward(h), (h.reshape(-1, 4) * 3.0 - 1.0).reshape(2, 5, 4))
    torch.testing.assert_close(moe.forward(h[0]), h[0] * 3.0 - 1.0)


def test_forward_rejects_bad_ranks_and_hidden_sizes():
    router = types.SimpleNamespace(hidden_size=8, num_experts=4, num_experts_per_tok=2)
    moe = MoELayer(0, router, None, None, None)
    with pytest.raises(ValueError):
        moe.forward(torch.zeros(8))
    with pytest.raises(ValueError):
        moe.forward(torch.zeros(1, 2, 3, 8))
    with pytest.raises(ValueError, match="hidden size"):
        moe._forward_tokens(torch.zeros(3, 7))
    assert moe._forward_tokens(torch.zeros(0, 8)).shape == (0, 8)


def test_set_moe_installs_the_adapter():
    layer = MoEInfraDecoderLayer(_small_mixtral_config(), layer_idx=0)
    moe = MoELayer(0, None, None, None, None)
    layer.set_moe(moe)
    assert isinstance(layer.mlp, MoELayerAdapter)
    assert layer.mlp.moe_layer is moe
    with pytest.raises(ValueError):
        layer.mlp(torch.zeros(4, 64))


def test_decoder_layer_runs_with_an_injected_moe():
    from transformers.models.mixtral.modeling_mixtral import MixtralRotaryEmbedding

    cfg = _small_mixtral_config()
    layer = MoEInfraDecoderLayer(cfg, layer_idx=0)

    class Doubling(torch.nn.Module):
        def forward(self, h):
            return 2.0 * h

    layer.set_moe(Doubling())
    h = torch.randn(1, 4, 64)
    pos = torch.arange(4).unsqueeze(0)
    pe = MixtralRotaryEmbedding(cfg)(h, position_ids=pos)
    out = layer(h, position_embeddings=pe, attention_mask=None, position_ids=pos,
                cache_position=torch.arange(4))
    out = out[0] if isinstance(out, tuple) else out
    assert out.shape == h.shape and torch.isfinite(out).all()


def test_predict_next_layer_experts_is_sorted_and_unique():
    from moeinfra_b200.engine.router import ExpertRouter

    r = ExpertRouter(torch.zeros(8, 16), num_experts_per_tok=2)
    assert r.predict_next_layer_experts(torch.tensor([[5, 1], [1, 7], [3, 5]])) == [1, 3, 5, 7]
    with pytest.raises(ValueError):
        ExpertRouter(torch.zeros(8), 2)
    with pytest.raises(ValueError):
        ExpertRouter(torch.zeros(4, 16), 5)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 5, 40])
def test_seam_experts_run_behind_the_real_router_and_combine(monkeypatch, T):
    """Stand-in experts through ``_ensure_expert_on_gpu``; dispatch and combine as the reference."""
    from moeinfra_b200.engine.router import ExpertRouter
    from oracle import moe as omoe

    H, E, k = 256, 8, 2
    g = torch.Generator(device="cuda").manual_seed(11 + T)
    gate = (torch.randn(E, H, generator=g, device="cuda") * 0.05).half()
    router = ExpertRouter(gate, num_experts_per_tok=k)
    moe = MoELayer(0, router, None, None, None)
    scales = [0.5 + 0.25 * e for e in range(E)]

    class Scale:
        def __init__(self, s):
            self.s = s

        def __call__(self, x):
            return (x.float() * self.s).half()

    calls = []

    def ensure(e):
        calls.append(e)
        return Scale(scales[e])

    monkeypatch.setattr(moe, "_ensure_expert_on_gpu", ensure)
    h = torch.randn(T, H, generator=g, device="cuda").half()
    out = moe.forward(h.reshape(1, T, H)).reshape(T, H)
    assert calls == sorted(set(calls))  # ascending expert ids, each once
    hn, wn = h.cpu().numpy(), gate.cpu().numpy()
    y, idx, _, _ = omoe.moe_layer_forward(
        hn, wn, [], H, 0, k=k,
        expert_fn=lambda x, e: (x.astype(np.float32) * scales[e]).astype(np.float16))
    assert calls == sorted(set(int(v) for v in idx.reshape(-1)))
    assert np.array_equal(out.cpu().numpy().view(np.uint16), y.view(np.uint16))
