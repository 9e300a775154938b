"""NF4 Mixtral expert representations (API of the reference's ``model/expert.py``).

* :class:`PrequantizedNF4Expert` — CPU-resident serialized NF4 state exactly as
  stored (``model/expert.py:176-241``); no quantization or reconstruction.
* :class:`QuantizedMixtralExpert` — bf16 weights in, NF4 out
  (``model/expert.py:8-174``).  The reference wraps bitsandbytes
  ``Linear4bit``; here the weights are quantized by this package's own
  quantizer at construction (``compress_statistics=False`` as at
  ``model/expert.py:52``) and the forward pass runs the B200 expert kernel.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from moeinfra_b200.model.nf4_format import (
    BLOB_KEY, REQUIRED_SERIALIZED_KEYS, canonical_state, parse_blob, quantize_nf4,
)


class NF4Linear(nn.Module):
    """One NF4 projection in serialized store form (stand-in for ``Linear4bit``).

    ``state`` holds the ``Linear4bit.state_dict()`` tensors; ``weight`` is the
    packed uint8 tensor so ``size_bytes`` counts packed bytes like the
    reference (``model/expert.py:82-87``).
    """

    def __init__(self, state: dict, in_features: int, out_features: int) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.compute_dtype = torch.float16
        self.state = dict(state)

    @property
    def weight(self) -> torch.Tensor:
        return self.state["weight"]

    def canonical(self) -> dict:
        return canonical_state(self.state)

    def state_dict(self, *args, **kwargs):  # noqa: D401 - mirrors Linear4bit.state_dict keys
        return dict(self.state)

    def _apply(self, fn, recurse=True):
        # Device moves only: packed codes, absmax and codebooks keep their dtypes
        # (Module.half()/float() must not rewrite quantization state).
        moved = {}
        for k, v in self.state.items():
            if isinstance(v, torch.Tensor) and k != BLOB_KEY:
                r = fn(v)
                moved[k] = r if r.dtype == v.dtype else v.to(r.device)
            else:
                moved[k] = v
        self.state = moved
        return self


class QuantizedMixtralExpert(nn.Module):
    """A Mixtral SwiGLU expert ``w2(silu(w1 x) * w3 x)`` with NF4 weights."""

    def __init__(self, w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor) -> None:
        super().__init__()
        self.w1 = self._quantize_linear(w1)
        self.w2 = self._quantize_linear(w2)
        self.w3 = self._quantize_linear(w3)
        self._gpu = None

    @staticmethod
    def _quantize_linear(weight: torch.Tensor) -> NF4Linear:
        if weight.ndim != 2:
            raise ValueError(f"Expected a 2D weight tensor, got shape {weight.shape}")
        if weight.dtype != torch.bfloat16:
            raise ValueError(f"Expected BF16 weights, got {weight.dtype}")
        return NF4Linear(quantize_nf4(weight, compress_statistics=False),
                         in_features=weight.shape[1], out_features=weight.shape[0])

    @property
    def hidden_size(self) -> int:
        return self.w1.in_features

    @property
    def intermediate_size(self) -> int:
        return self.w1.out_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.device.type != "cuda":
            raise RuntimeError("QuantizedMixtralExpert.forward runs on CUDA only; call .cuda() first")
        if self._gpu is None or self._gpu.device != self.device:
            from moeinfra_b200.transfer.nf4_reconstruct import ReconstructedNF4Expert

            self._gpu = ReconstructedNF4Expert(
                self, {n: getattr(self, n).canonical() for n in ("w1", "w2", "w3")})
        return self._gpu(x)

    def _apply(self, fn, recurse=True):
        self._gpu = None
        return super()._apply(fn, recurse)

    @property
    def device(self) -> torch.device:
        return self.w1.weight.device

    @property
    def size_bytes(self) -> int:
        return sum(l.weight.numel() * l.weight.element_size() for l in (self.w1, self.w2, self.w3))

    @classmethod
    def from_prequantized(cls, w1_state: dict, w2_state: dict, w3_state: dict,
                          hidden_size: int, intermediate_size: int) -> "QuantizedMixtralExpert":
        expert = cls.__new__(cls)
        nn.Module.__init__(expert)
        expert._gpu = None
        expert.w1 = cls._linear_from_prequantized(w1_state, hidden_size, intermediate_size)
        expert.w2 = cls._linear_from_prequantized(w2_state, intermediate_size, hidden_size)
        expert.w3 = cls._linear_from_prequantized(w3_state, hidden_size, intermediate_size)
        return expert

    @staticmethod
    def _linear_from_prequantized(state: dict, in_features: int, out_features: int) -> NF4Linear:
        missing = REQUIRED_SERIALIZED_KEYS - state.keys()
        if missing:
            raise ValueError(f"Missing prequantized NF4 state tensors: {sorted(missing)}")
        meta = parse_blob(state[BLOB_KEY])
        if meta is not None and "shape" in meta:
            if list(meta["shape"]) != [out_features, in_features]:
                raise ValueError(
                    f"NF4 state shape {meta['shape']} != expected {[out_features, in_features]}")
        return NF4Linear({k: v.cpu() if isinstance(v, torch.Tensor) else v for k, v in state.items()},
                         in_features=in_features, out_features=out_features)


@dataclass
class PrequantizedNF4Expert:
    """CPU-resident representation of an already-quantized NF4 Mixtral expert."""

    w1: dict
    w2: dict
    w3: dict
    hidden_size: int
    intermediate_size: int

    _REQUIRED_KEYS = REQUIRED_SERIALIZED_KEYS

    @classmethod
    def from_serialized(cls, w1: dict, w2: dict, w3: dict, hidden_size: int,
                        intermediate_size: int) -> "PrequantizedNF4Expert":
        for name, state in (("w1", w1), ("w2", w2), ("w3", w3)):
            missing = cls._REQUIRED_KEYS - state.keys()
            if missing:
                raise ValueError(f"Missing serialized NF4 state for {name}: {sorted(missing)}")
        return cls(w1=dict(w1), w2=dict(w2), w3=dict(w3), hidden_size=hidden_size,
                   intermediate_size=intermediate_size)

    @property
    def device(self) -> torch.device:
        return self.w1["weight"].device

    @property
    def size_bytes(self) -> int:
        return sum(t.numel() * t.element_size()
                   for st in (self.w1, self.w2, self.w3) for t in st.values()
                   if isinstance(t, torch.Tensor))
