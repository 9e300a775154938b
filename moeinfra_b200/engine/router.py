"""Top-k router for a Mixtral MoE layer (API of the reference's ``engine/router.py``).

``route_with_logits`` runs one fused B200 kernel: fp16 gate GEMV with fp32
accumulation, fp32 softmax in torch's CUDA operation order, top-k (exact ties
toward the lower expert index) and renormalisation over the chosen k
(``engine/router.py:65-94``).  Inputs must be CUDA fp16 tensors (the
reference engine casts the gate to the model dtype, ``engine/engine.py:230-234``);
there is no CPU path.
"""
from __future__ import annotations

import logging
from typing import Optional

import torch

from moeinfra_b200 import kernels


class ExpertRouter:
    """Top-k router for a Mixtral MoE layer."""

    def __init__(self, gate_weight: torch.Tensor, num_experts_per_tok: int = 2,
                 logger: Optional[logging.Logger] = None) -> None:
        if gate_weight.ndim != 2:
            raise ValueError(f"gate_weight must be 2D, got shape {tuple(gate_weight.shape)}")
        self.num_experts = gate_weight.shape[0]
        self.hidden_size = gate_weight.shape[1]
        self.num_experts_per_tok = num_experts_per_tok
        self._logger = logger or logging.getLogger(__name__)
        if num_experts_per_tok <= 0:
            raise ValueError("num_experts_per_tok must be positive")
        if num_experts_per_tok > self.num_experts:
            raise ValueError(
                f"num_experts_per_tok ({num_experts_per_tok}) must be <= "
                f"num_experts ({self.num_experts})")
        self.gate_weight = gate_weight
        self._gate_f16: Optional[torch.Tensor] = None

    @property
    def device(self) -> torch.device:
        return self.gate_weight.device

    def _check(self, hidden_states: torch.Tensor) -> None:
        if hidden_states.shape[-1] != self.hidden_size:
            raise ValueError(
                f"hidden_states last dim {hidden_states.shape[-1]} != hidden_size {self.hidden_size}")
        if hidden_states.device != self.gate_weight.device:
            raise ValueError(
                f"hidden_states device {hidden_states.device} != gate device {self.gate_weight.device}")

    def gate_f16(self) -> torch.Tensor:
        """The gate in the fp16 compute dtype, contiguous (cached)."""
        g = self._gate_f16
        if g is None or g.device != self.gate_weight.device:
            g = self.gate_weight.to(torch.float16).contiguous()
            self._gate_f16 = g
        return g

    def _flat(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if hidden_states.dtype != torch.float16:
            raise ValueError(
                f"the B200 router computes in fp16 (the model dtype); got {hidden_states.dtype}")
        return hidden_states.reshape(-1, self.hidden_size).contiguous()

    def logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """Mixtral router logits ``h . Wg^T`` in fp16."""
        self._check(hidden_states)
        lg, _, _ = kernels.router_topk(self._flat(hidden_states), self.gate_f16(),
                                       self.num_experts_per_tok, with_logits=True)
        return lg.reshape(*hidden_states.shape[:-1], self.num_experts)

    def route(self, hidden_states):
        _, expert_weights, expert_indices = self.route_with_logits(hidden_states)
        return expert_indices, expert_weights

    def route_with_logits(self, hidden_states: torch.Tensor):
        self._check(hidden_states)
        lead = hidden_states.shape[:-1]
        lg, w, idx = kernels.router_topk(self._flat(hidden_states), self.gate_f16(),
                                         self.num_experts_per_tok, with_logits=True)
        k = self.num_experts_per_tok
        return lg.reshape(*lead, self.num_experts), w.reshape(*lead, k), idx.reshape(*lead, k)

    def predict_next_layer_experts(self, current_expert_indices: torch.Tensor) -> list[int]:
        """Predict next-layer experts using current-layer selections."""
        flat = current_expert_indices.reshape(-1)
        return sorted(int(x) for x in flat.unique().tolist())
