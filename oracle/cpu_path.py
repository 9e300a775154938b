"""Multi-threaded CPU restatement of one MoE layer step (torch on the host cores).

TEST AND BENCH INFRASTRUCTURE ONLY: this is the timed CPU baseline of
``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) and is
checked against the numpy oracle in ``tests/``.  The product never imports it.

It computes what ``oracle.moe.moe_layer_forward`` computes -- the reference's
``MoELayer._forward_tokens`` (``model/moe_layer.py:117-211``) over NF4 experts
(``transfer/nf4_reconstruct.py:152-155``) -- with torch CPU kernels so that all
host threads take part, as the reference's CPU path (bitsandbytes' CPU backend
behind the same modules) would:

* router: fp16 logits of an fp32-accumulated ``h . Wg^T``, fp32 softmax,
  top-k, renormalised (``engine/router.py:65-94``);
* an expert with one token: fp16 weights ``fp16(fp16(code) * fp16(absmax))``
  (the 4-bit GEMV branch), fp32 accumulation;
* an expert with more tokens: ``bf16(code * absmax)`` weights cast to fp16,
  fp32 accumulation (dequantise-then-GEMM);
* ``silu(w1 x) * (w3 x)`` rounded to fp16 as the modules do, then ``w2``;
* combine in ascending expert id with one fp16 rounding per expert
  (``model/moe_layer.py:187-191``).

Summation order differs from the numpy oracle (torch's blocked kernels), so
outputs agree within fp16 rounding, not bit for bit.
"""
from __future__ import annotations

import torch

BLOCK = 64


def dequant_store(q: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, rows: int,
                  cols: int, gemv: bool) -> torch.Tensor:
    """fp16 weight [rows, cols] from a store-layout NF4 projection (element 2j = high nibble)."""
    hi = (q >> 4).long()
    lo = (q & 15).long()
    nib = torch.stack((hi, lo), dim=1).reshape(rows, cols // BLOCK, BLOCK)
    a = absmax.reshape(rows, cols // BLOCK, 1)
    if gemv:
        c16 = code.to(torch.float16).float()
        a16 = a.to(torch.float16).float()
        w = (c16[nib] * a16).to(torch.float16)       # fp32 product of two fp16 is exact
    else:
        w = (code[nib] * a).to(torch.bfloat16).to(torch.float16)
    return w.reshape(rows, cols)


def linear(x16: torch.Tensor, proj: dict, code: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    w = dequant_store(proj["q"], proj["absmax"], code, rows, cols, gemv=x16.shape[0] == 1)
    return (x16.float() @ w.float().t()).to(torch.float16)


def expert_forward(x16: torch.Tensor, ex: dict, code: torch.Tensor, hidden: int,
                   inter: int) -> torch.Tensor:
    g = linear(x16, ex["w1"], code, inter, hidden).float()
    u = linear(x16, ex["w3"], code, inter, hidden)
    s = (g / (1.0 + torch.exp(-g))).to(torch.float16)
    a = (s.float() * u.float()).to(torch.float16)
    return linear(a, ex["w2"], code, hidden, inter)


def route(h16: torch.Tensor, wg16: torch.Tensor, k: int):
    logits = (h16.float() @ wg16.float().t()).to(torch.float16)
    p = torch.softmax(logits.float(), dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return logits, w, idx


def layer_forward(h16: torch.Tensor, wg16: torch.Tensor, experts, code: torch.Tensor,
                  hidden: int, inter: int, k: int = 2):
    """``experts[e]`` is ``{"w1": {"q", "absmax"}, "w3": ..., "w2": ...}`` or None when unrouted."""
    _, w, idx = route(h16, wg16, k)
    out = torch.zeros_like(h16)
    for e in sorted(set(idx.reshape(-1).tolist())):
        match = idx == e
        mask = match.any(-1)
        tw = (w * match.float()).sum(-1)
        y = expert_forward(h16[mask], experts[e], code, hidden, inter)
        out[mask] = (out[mask].float() + y.float() * tw[mask, None]).to(torch.float16)
    return out, idx, w
