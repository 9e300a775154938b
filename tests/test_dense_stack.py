"""CPU (fp32): the engine's dense decoder against Hugging Face's Mixtral modules.

``DenseStack`` (fused q/k/v, static KV cache, device-side decode position) and
HF's ``MixtralForCausalLM`` get the same dense weights and the same stand-in
MoE block; prefill logits and the logits of several decode steps (one token
at a time through the static cache, with the position as a tensor as in the
captured graph) must match HF's full-sequence forward.
"""
from __future__ import annotations

import pytest
import torch

from moeinfra_b200.engine.dense import DenseConfig, DenseStack
from moeinfra_b200.model.types import LayerWeights

H, L, E, V, HEADS, KV = 64, 2, 4, 48, 4, 2


class LinearMoE(torch.nn.Module):
    """Stand-in MoE: a fixed linear map of the tokens (the same on both sides)."""

    def __init__(self, w):
        super().__init__()
        self.w = w

    def forward(self, x):
        shape = x.shape
        return (x.reshape(-1, shape[-1]) @ self.w.t()).reshape(shape)


def _models(seed=0):
    from transformers import MixtralConfig
    from transformers.models.mixtral.modeling_mixtral import MixtralForCausalLM

    cfg = MixtralConfig(hidden_size=H, intermediate_size=2 * H, num_hidden_layers=L,
                        num_attention_heads=HEADS, num_key_value_heads=KV, num_local_experts=E,
                        num_experts_per_tok=2, vocab_size=V, rope_theta=1e6, rms_norm_eps=1e-5)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    hf = MixtralForCausalLM(cfg).eval()
    moes = []
    with torch.no_grad():
        for p in hf.parameters():
            p.normal_(0, 0.05)
        for layer in hf.model.layers:
            layer.input_layernorm.weight.add_(1.0)
            layer.post_attention_layernorm.weight.add_(1.0)
            m = LinearMoE(torch.randn(H, H) * 0.05)
            layer.mlp = m
            moes.append(m)
        hf.model.norm.weight.add_(1.0)
    weights = [LayerWeights(input_layernorm=l.input_layernorm.weight.data,
                            q_proj=l.self_attn.q_proj.weight.data,
                            k_proj=l.self_attn.k_proj.weight.data,
                            v_proj=l.self_attn.v_proj.weight.data,
                            o_proj=l.self_attn.o_proj.weight.data,
                            post_attention_layernorm=l.post_attention_layernorm.weight.data,
                            moe_gate=torch.zeros(E, H)) for l in hf.model.layers]
    stack = DenseStack(DenseConfig.from_mixtral(cfg), weights, hf.model.embed_tokens.weight.data,
                       hf.model.norm.weight.data, hf.lm_head.weight.data, moes, "cpu",
                       max_batch=2, max_len=32, dtype=torch.float32)
    return hf, stack


@pytest.mark.parametrize("B", [1, 2])
def test_prefill_and_decode_match_hf(B):
    hf, stack = _models()
    g = torch.Generator().manual_seed(B)
    S, steps = 7, 4
    ids = torch.randint(0, V, (B, S + steps), generator=g)
    with torch.no_grad():
        want = hf(ids).logits  # [B, S + steps, V]
        got = stack.forward(ids[:, :S], pos0=0)
        torch.testing.assert_close(got, want[:, S - 1], rtol=1e-4, atol=1e-5)
        pos = torch.tensor([S])
        for i in range(steps):
            got = stack.forward(ids[:, S + i:S + i + 1], decode_pos=pos)
            torch.testing.assert_close(got, want[:, S + i], rtol=1e-4, atol=1e-5)
            pos += 1


def test_chunked_prefill_continues_the_cache():
    hf, stack = _models(seed=1)
    ids = torch.randint(0, V, (1, 10), generator=torch.Generator().manual_seed(9))
    with torch.no_grad():
        want = hf(ids).logits
        stack.forward(ids[:, :6], pos0=0)
        got = stack.forward(ids[:, 6:], pos0=6)
    torch.testing.assert_close(got, want[:, -1], rtol=1e-4, atol=1e-5)


def test_limits_are_checked():
    _, stack = _models()
    with pytest.raises(ValueError):
        stack.forward(torch.zeros(3, 4, dtype=torch.long))
    with pytest.raises(ValueError):
        stack.forward(torch.zeros(1, 40, dtype=torch.long))
