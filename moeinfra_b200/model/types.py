"""Dense per-layer weights (API of the reference's ``model/types.py``)."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LayerWeights:
    input_layernorm: torch.Tensor
    q_proj: torch.Tensor
    k_proj: torch.Tensor
    v_proj: torch.Tensor
    o_proj: torch.Tensor
    post_attention_layernorm: torch.Tensor
    moe_gate: torch.Tensor
