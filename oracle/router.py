"""Router oracle (numpy) — TEST INFRASTRUCTURE ONLY, never imported by the product.

Restates ``ExpertRouter.route_with_logits`` (``engine/router.py:65-94``):

1. ``logits = F.linear(h, Wg)`` in fp16 (``router.py:66-69``; the gate is cast
   to the model dtype at ``engine/engine.py:231-234``): fp32-or-wider
   accumulation of exact fp16 products, one rounding to fp16.  The oracle
   accumulates in fp64, i.e. returns the correctly rounded logit.
2. ``softmax(logits.float(), -1)`` (``router.py:81-84``) in the operation
   order of torch's CUDA warp softmax for a last dim of 8: max, ``exp(l - max)``,
   a butterfly sum over lane offsets 4, 2, 1, then ``e / sum``.
3. ``topk(p, k)`` (``router.py:86-90``): descending probability.  Exact ties
   follow torch's CUDA topk (the reference router runs on the GPU): the lower
   expert indices are selected, and equal values are listed in descending
   index order.  (torch's CPU topk differs on ties; tests compare tied
   selections against CPU goldens by value.)
4. ``w /= w.sum(-1)`` (``router.py:92``).
"""
from __future__ import annotations

import numpy as np


def logits_f16(h16: np.ndarray, wg16: np.ndarray) -> np.ndarray:
    acc = np.asarray(h16, np.float16).astype(np.float64) @ np.asarray(wg16, np.float16).astype(np.float64).T
    return acc.astype(np.float16)


def _butterfly_sum(e: np.ndarray) -> np.ndarray:
    """Sum over the last axis in xor-butterfly order (width = next pow2)."""
    n = e.shape[-1]
    width = 1
    while width < n:
        width *= 2
    v = np.zeros(e.shape[:-1] + (width,), np.float32)
    v[..., :n] = e
    off = width // 2
    lanes = np.arange(width)
    while off > 0:
        v = (v + v[..., lanes ^ off]).astype(np.float32)
        off //= 2
    return v[..., 0]


def softmax_f32(logits16: np.ndarray) -> np.ndarray:
    lg = np.asarray(logits16, np.float16).astype(np.float32)
    m = lg.max(axis=-1, keepdims=True)
    e = np.exp((lg - m).astype(np.float32)).astype(np.float32)
    s = _butterfly_sum(e)[..., None]
    return (e / s).astype(np.float32)


def topk_cuda_order(p: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Top-k per row: lower indices win ties for selection; output in
    descending value, equal values in descending index."""
    ar = np.broadcast_to(np.arange(p.shape[-1]), p.shape)
    sel = np.lexsort((ar, -p), axis=-1)[..., :k]
    vals = np.take_along_axis(p, sel, -1)
    order = np.lexsort((-sel, -vals), axis=-1)
    sel = np.take_along_axis(sel, order, -1)
    return np.take_along_axis(p, sel, -1), sel.astype(np.int64)


def route_with_logits(h16: np.ndarray, wg16: np.ndarray, k: int = 2):
    """Returns ``(logits fp16 [T,E], weights fp32 [T,k], indices int64 [T,k])``."""
    lg = logits_f16(h16, wg16)
    return (lg,) + route_from_logits(lg, k)


def route_from_logits(lg16: np.ndarray, k: int = 2):
    p = softmax_f32(lg16)
    w, idx = topk_cuda_order(p, k)
    s = w[..., 0].copy()
    for j in range(1, k):
        s = (s + w[..., j]).astype(np.float32)
    return (w / s[..., None]).astype(np.float32), idx
