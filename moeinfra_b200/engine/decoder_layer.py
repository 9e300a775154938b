"""HF Mixtral decoder-layer seam (API of the reference's ``engine/decoder_layer.py``).

``MoEInfraDecoderLayer.set_moe`` swaps Hugging Face's sparse-MoE block for a
:class:`~moeinfra_b200.model.moe_layer.MoELayer` through
:class:`MoELayerAdapter`, which flattens ``[batch, seq, hidden]`` to
``[tokens, hidden]`` and back (``:7-42``).
"""
from __future__ import annotations

import torch
from transformers.models.mixtral.modeling_mixtral import MixtralDecoderLayer


class MoELayerAdapter(torch.nn.Module):
    """Adapt the token-level MoELayer to HF's 3-D interface."""

    def __init__(self, moe_layer):
        super().__init__()
        self.moe_layer = moe_layer

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if hidden_states.ndim != 3:
            raise ValueError("hidden_states must have shape (batch, sequence, hidden)")
        b, s, h = hidden_states.shape
        out = self.moe_layer.forward(hidden_states.reshape(b * s, h))
        return out.reshape(b, s, h)


class MoEInfraDecoderLayer(MixtralDecoderLayer):
    """Mixtral decoder layer using the B200 MoE layer for expert execution."""

    def set_moe(self, moe_layer) -> None:
        self.mlp = MoELayerAdapter(moe_layer)
