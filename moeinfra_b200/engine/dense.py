"""Dense (non-expert) part of the Mixtral decoder, laid out for batched decode on B200.

The reference runs Hugging Face's ``MixtralDecoderLayer`` with a growing
``DynamicCache`` (``engine/engine.py:326-378``), which rules out CUDA graphs
and reallocates the cache every token.  Here the same arithmetic is laid out
for fixed shapes so a whole decode step (32 layers, MoE included) can be
captured once and replayed:

* per layer: input RMSNorm, ONE fused q/k/v projection (the three weights
  concatenated row-wise, one fp16 GEMM instead of three), RoPE, a write of
  the new keys / values into a preallocated cache ``[B, kv_heads, max_len,
  head_dim]`` at the step's position, grouped-query attention over the cache
  (positions past the current one masked), o_proj, residual add,
  post-attention RMSNorm, the MoE layer (``MoELayer.forward``), residual add;
* final RMSNorm and lm_head on each sequence's last position.

Numerics follow the HF modules the reference uses: RMSNorm in fp32 and cast
back (``weight * x.to(fp16)``), RoPE ``x*cos + rotate_half(x)*sin`` in fp16
with HF's default frequencies (``theta ** (-2i/d)``), attention with fp32
softmax, everything else fp16 with fp32 accumulation (cuBLAS / SDPA).  The
position of a decode step lives in a device tensor, so a captured graph
advances it itself.  Sequences of one batch share their length (equal-length
prompts, as in the benchmark configurations).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F


@dataclass
class DenseConfig:
    hidden_size: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    vocab_size: int
    rope_theta: float
    rms_norm_eps: float

    @classmethod
    def from_mixtral(cls, cfg) -> "DenseConfig":
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        theta = getattr(cfg, "rope_theta", None)
        if theta is None:
            rp = getattr(cfg, "rope_parameters", None) or {}
            theta = rp.get("rope_theta", 1e6)
        return cls(hidden_size=cfg.hidden_size, num_heads=cfg.num_attention_heads,
                   num_kv_heads=cfg.num_key_value_heads, head_dim=head_dim,
                   vocab_size=cfg.vocab_size, rope_theta=float(theta),
                   rms_norm_eps=float(cfg.rms_norm_eps))


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """HF ``MixtralRMSNorm``: fp32 statistics, cast back before the weight."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return weight * xf.to(x.dtype)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class DenseLayer:
    """Weights of one decoder layer's dense part on the device (fp16)."""

    def __init__(self, weights, cfg: DenseConfig, device, dtype=torch.float16) -> None:
        def t(x):
            return x.to(device=device, dtype=dtype).contiguous()

        self.in_norm = t(weights.input_layernorm)
        self.post_norm = t(weights.post_attention_layernorm)
        self.w_qkv = torch.cat([t(weights.q_proj), t(weights.k_proj), t(weights.v_proj)], 0)
        self.w_o = t(weights.o_proj)
        self.q_dim = cfg.num_heads * cfg.head_dim
        self.kv_dim = cfg.num_kv_heads * cfg.head_dim


class DenseStack:
    """The dense decoder stack with a static KV cache; the MoE layers plug in per layer."""

    def __init__(self, cfg: DenseConfig, layers: list, embed: torch.Tensor, final_norm: torch.Tensor,
                 lm_head: torch.Tensor, moe_layers: list, device, max_batch: int, max_len: int,
                 dtype=torch.float16) -> None:
        if len(layers) != len(moe_layers):
            raise ValueError("one MoE layer per decoder layer is required")
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.layers = [DenseLayer(w, cfg, self.device, dtype) for w in layers]
        self.moe = list(moe_layers)
        self.embed = embed.to(device=self.device, dtype=dtype).contiguous()
        self.final_norm = final_norm.to(device=self.device, dtype=dtype).contiguous()
        self.lm_head = lm_head.to(device=self.device, dtype=dtype).contiguous()
        self.max_batch, self.max_len = max_batch, max_len
        L, B, kv, hd = len(layers), max_batch, cfg.num_kv_heads, cfg.head_dim
        self.k_cache = torch.zeros(L, B, kv, max_len, hd, device=self.device, dtype=dtype)
        self.v_cache = torch.zeros_like(self.k_cache)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.int64,
                                                      device=self.device).float() / hd))
        pos = torch.arange(max_len, device=self.device, dtype=torch.float32)
        freqs = torch.outer(pos, inv)
        emb = torch.cat((freqs, freqs), dim=-1)
        self.cos = emb.cos().to(dtype)
        self.sin = emb.sin().to(dtype)
        self.scale = 1.0 / math.sqrt(hd)
        self.layer_hook = None  # called as hook(layer_id, moe_layer) after each MoE layer

    # -- attention --------------------------------------------------------------------
    def _attention(self, li: int, x: torch.Tensor, pos0, T: int, decode_pos: Optional[torch.Tensor]):
        """x [B, T, H] normed -> attention output [B, T, H]; writes the cache."""
        cfg, lay = self.cfg, self.layers[li]
        B = x.shape[0]
        qkv = F.linear(x, lay.w_qkv)
        q, k, v = qkv.split([lay.q_dim, lay.kv_dim, lay.kv_dim], dim=-1)
        q = q.view(B, T, cfg.num_heads, cfg.head_dim).transpose(1, 2)
        k = k.view(B, T, cfg.num_kv_heads, cfg.head_dim).transpose(1, 2)
        v = v.view(B, T, cfg.num_kv_heads, cfg.head_dim).transpose(1, 2)
        if decode_pos is not None:  # one token per sequence at a device-side position
            cos = self.cos.index_select(0, decode_pos)[None, None]
            sin = self.sin.index_select(0, decode_pos)[None, None]
        else:
            cos = self.cos[pos0:pos0 + T][None, None]
            sin = self.sin[pos0:pos0 + T][None, None]
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        kc, vc = self.k_cache[li, :B], self.v_cache[li, :B]
        if decode_pos is not None:
            kc.index_copy_(2, decode_pos, k)
            vc.index_copy_(2, decode_pos, v)
            ar = torch.arange(self.max_len, device=self.device)
            mask = torch.where(ar <= decode_pos, 0.0, float("-inf")).to(q.dtype)[None, None, None]
            o = F.scaled_dot_product_attention(q, kc, vc, attn_mask=mask, scale=self.scale,
                                               enable_gqa=True)
        else:
            kc[:, :, pos0:pos0 + T] = k
            vc[:, :, pos0:pos0 + T] = v
            keys, vals = kc[:, :, :pos0 + T], vc[:, :, :pos0 + T]
            if pos0 == 0:
                o = F.scaled_dot_product_attention(q, keys, vals, is_causal=True, scale=self.scale,
                                                   enable_gqa=True)
            else:
                qpos = torch.arange(pos0, pos0 + T, device=self.device)[:, None]
                kpos = torch.arange(pos0 + T, device=self.device)[None, :]
                mask = torch.where(kpos <= qpos, 0.0, float("-inf")).to(q.dtype)[None, None]
                o = F.scaled_dot_product_attention(q, keys, vals, attn_mask=mask,
                                                   scale=self.scale, enable_gqa=True)
        o = o.transpose(1, 2).reshape(B, T, cfg.num_heads * cfg.head_dim)
        return F.linear(o, lay.w_o)

    # -- forward ------------------------------------------------------------------------
    def forward(self, ids: torch.Tensor, pos0: int = 0,
                decode_pos: Optional[torch.Tensor] = None) -> torch.Tensor:
        """ids [B, T] (T == 1 with ``decode_pos``) -> fp16 logits of the last position [B, vocab]."""
        B, T = ids.shape
        if B > self.max_batch:
            raise ValueError(f"batch {B} exceeds max_batch {self.max_batch}")
        if decode_pos is None and pos0 + T > self.max_len:
            raise ValueError(f"{pos0 + T} positions exceed max_len {self.max_len}")
        eps = self.cfg.rms_norm_eps
        h = F.embedding(ids, self.embed)
        for li, lay in enumerate(self.layers):
            a = self._attention(li, rms_norm(h, lay.in_norm, eps), pos0, T, decode_pos)
            h = h + a
            x = rms_norm(h, lay.post_norm, eps)
            y = self.moe[li].forward(x.reshape(B * T, -1)).reshape(B, T, -1)
            if self.layer_hook is not None:
                self.layer_hook(li, self.moe[li])
            h = h + y
        h = rms_norm(h[:, -1], self.final_norm, eps)
        return F.linear(h, self.lm_head)
