"""MoE-layer oracle (numpy) — TEST INFRASTRUCTURE ONLY, never imported by the product.

Restates ``MoELayer._forward_tokens`` (``model/moe_layer.py:117-211``):

* route once for all tokens (``:143``);
* ``output = zeros_like(h)`` in fp16 (``:147``);
* for each routed expert in ascending id (``:150-153``, ``:172``):
  ``token_w = sum_k w[:, k] * (idx[:, k] == e)`` in fp32 (``:180-183``),
  ``y = expert(h[mask])`` in fp16 (``:185-186``),
  ``output[mask] += y * token_w[mask, None]`` (``:187-191``): the product is
  fp32, the in-place add on the fp16 output computes in fp32 and rounds to
  fp16 once per expert.
"""
from __future__ import annotations

import numpy as np

from oracle import nf4 as onf4
from oracle import router as orouter


def combine_expert_outputs(T: int, H: int, idx: np.ndarray, w: np.ndarray,
                           expert_out: dict) -> np.ndarray:
    """Weighted combine in ascending expert order.

    ``expert_out[e]`` is the fp16 output [n_e, H] of expert ``e`` on the tokens
    routed to it, in ascending token order.
    """
    out = np.zeros((T, H), np.float16)
    for e in sorted(expert_out):
        match = idx == e
        mask = match.any(-1)
        tw = (w * match.astype(np.float32)).sum(-1, dtype=np.float32).astype(np.float32)
        prod = expert_out[e].astype(np.float32) * tw[mask][:, None]
        out[mask] = (out[mask].astype(np.float32) + prod.astype(np.float32)).astype(np.float16)
    return out


def moe_layer_forward(h16: np.ndarray, wg16: np.ndarray, experts: list, hidden: int,
                      inter: int, k: int = 2, expert_fn=None):
    """Full layer: returns ``(out fp16 [T,H], idx, w, logits)``."""
    lg, w, idx = orouter.route_with_logits(h16, wg16, k)
    fn = expert_fn or (lambda x, e: onf4.expert_forward(x, experts[e], hidden, inter))
    outs = {}
    for e in sorted(set(int(v) for v in idx.reshape(-1))):
        mask = (idx == e).any(-1)
        outs[e] = fn(h16[mask], e)
    return combine_expert_outputs(h16.shape[0], h16.shape[1], idx, w, outs), idx, w, lg
