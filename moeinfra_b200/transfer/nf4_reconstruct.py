"""GPU-resident NF4 expert over transferred packed tensors.

API of the reference's ``transfer/nf4_reconstruct.py`` (``ReconstructedNF4Expert``,
``:117-166``).  The reference wraps the device tensors in bitsandbytes
``Linear4bit`` shells and runs three library matmuls; here construction only
re-lays each projection out once into the tile16 device layout (16-row x
64-element tiles contiguous, an exact permutation; a double-quantized absmax is
first rebuilt exactly, ``:17-38``) and ``forward`` is one call of the fused
B200 SwiGLU expert kernel on the packed weights (``:152-155``).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from moeinfra_b200 import kernels
from moeinfra_b200._native import NF4Expert
from moeinfra_b200.model.nf4_format import NESTED_BLOCKSIZE, NF4_BLOCKSIZE

_NF4_BLOCKSIZE = NF4_BLOCKSIZE        # reference :9
_NF4_QUANT_STORAGE = torch.uint8       # reference :11
_NF4_DTYPE = torch.bfloat16            # reference :12 (dequant dtype)
_NESTED_BLOCKSIZE = NESTED_BLOCKSIZE   # reference :13
_NESTED_DTYPE = torch.float32          # reference :14


class GPUNF4Linear(nn.Module):
    """Device view of one NF4 projection (stand-in for the reference's Linear4bit)."""

    def __init__(self, state: dict, *, in_features: int, out_features: int) -> None:
        super().__init__()
        weight = state.get("weight")
        if weight is None:
            raise ValueError("NF4 state is missing packed weight")
        if weight.dtype != _NF4_QUANT_STORAGE:
            raise ValueError(f"Expected packed NF4 weight dtype {_NF4_QUANT_STORAGE}, got {weight.dtype}")
        if weight.device.type != "cuda":
            raise RuntimeError("ReconstructedNF4Expert needs CUDA-resident NF4 tensors")
        numel = in_features * out_features
        if weight.numel() * 2 != numel:
            raise ValueError(f"packed weight has {weight.numel()} bytes, expected {numel // 2}")
        if numel % _NF4_BLOCKSIZE:
            raise ValueError(f"in*out = {numel} is not a multiple of {_NF4_BLOCKSIZE}")
        code = state.get("code")
        if code is None or code.numel() != 16 or code.dtype != torch.float32:
            raise ValueError("NF4 state needs a fp32 codebook of 16 entries")
        s2a, s2c = state.get("state2_absmax"), state.get("state2_code")
        if s2a is not None or s2c is not None:
            if s2a is None or s2c is None:
                raise ValueError("Incomplete nested NF4 quantization state")
            off = state.get("offset")
            off = 0.0 if off is None else float(off)
            absmax = kernels.nested_absmax(state["absmax"].reshape(-1).contiguous(),
                                           s2a.reshape(-1).contiguous().float(),
                                           s2c.reshape(-1).contiguous().float(), off,
                                           _NESTED_BLOCKSIZE)
        else:
            absmax = state["absmax"]
            if absmax.dtype != torch.float32:
                raise ValueError(f"absmax must be fp32 when not nested, got {absmax.dtype}")
        if absmax.numel() * _NF4_BLOCKSIZE != numel:
            raise ValueError("absmax length does not match the weight shape")
        if out_features % 16 or in_features % 64:
            raise ValueError("NF4 expert kernels need out_features % 16 == 0 and in_features % 64 == 0")
        self.in_features = in_features
        self.out_features = out_features
        self.compute_dtype = torch.float16
        # tile16 device layout: every kernel reads 16-row x 64-element tiles.
        self.packed, self.absmax = kernels.nf4_tile16(
            weight.reshape(-1).contiguous(), absmax.reshape(-1).contiguous().float(),
            out_features, in_features)
        self.code = code.reshape(-1).contiguous()

    @property
    def weight(self) -> torch.Tensor:
        return self.packed

    def dequantize(self) -> torch.Tensor:
        """bf16 weight [out, in], bit-exact with bitsandbytes' dequantize_4bit."""
        return kernels.nf4_dequant_tile16(self.packed, self.absmax, self.code,
                                          self.out_features, self.in_features)

    def descriptor(self):
        return kernels.matrix_desc(self.packed, self.absmax, self.code)


def _code_signature(state: dict, original, name: str) -> tuple:
    """16 codebook values, read from the CPU copy when one exists (no device sync)."""
    src = None
    proj = getattr(original, name, None)
    if isinstance(proj, dict):
        src = proj.get("weight.quant_map", proj.get("quant_map", proj.get("code")))
    elif proj is not None and hasattr(proj, "state"):
        src = proj.state.get("weight.quant_map")
    if src is None or src.device.type != "cpu":
        src = state["code"]
    return tuple(float(v) for v in src.detach().float().cpu().reshape(-1).tolist())


class ReconstructedNF4Expert(nn.Module):
    """GPU-resident Mixtral expert reconstructed from transferred NF4 state."""

    def __init__(self, original_expert, gpu_state) -> None:
        super().__init__()
        hidden_size = getattr(original_expert, "hidden_size", None)
        intermediate_size = getattr(original_expert, "intermediate_size", None)
        if hidden_size is None or intermediate_size is None:
            raise ValueError("Prequantized expert must expose hidden_size and intermediate_size")
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.w1 = GPUNF4Linear(gpu_state["w1"], in_features=hidden_size, out_features=intermediate_size)
        self.w2 = GPUNF4Linear(gpu_state["w2"], in_features=intermediate_size, out_features=hidden_size)
        self.w3 = GPUNF4Linear(gpu_state["w3"], in_features=hidden_size, out_features=intermediate_size)
        sigs = {n: _code_signature(gpu_state[n], original_expert, n) for n in ("w1", "w2", "w3")}
        if len(set(sigs.values())) != 1:
            raise NotImplementedError(
                "w1/w2/w3 carry different NF4 codebooks; the fused kernels need one codebook per expert")
        self.code_signature = sigs["w1"]
        self._desc = NF4Expert(self.w1.descriptor(), self.w3.descriptor(), self.w2.descriptor())

    @property
    def nf4_descriptor(self) -> NF4Expert:
        return self._desc

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.ndim != 2:
            raise ValueError(f"expected [tokens, hidden] input, got {tuple(x.shape)}")
        inp_dtype = x.dtype
        # Linear4bit computes in fp16 (reference :94) and returns the input dtype.
        y = kernels.expert_forward(self._desc, x.to(torch.float16).contiguous(), self.hidden_size,
                                   self.intermediate_size)
        return y if inp_dtype == torch.float16 else y.to(inp_dtype)

    @property
    def device(self) -> torch.device:
        return self.w1.weight.device

    @property
    def size_bytes(self) -> int:
        return sum(l.weight.numel() * l.weight.element_size() for l in (self.w1, self.w2, self.w3))


def resident_expert(cpu_expert, device) -> ReconstructedNF4Expert:
    """A GPU-resident copy of a CPU expert (its canonical NF4 state copied to ``device``)."""
    from moeinfra_b200.model.nf4_format import canonical_state

    state = {}
    for name in ("w1", "w2", "w3"):
        proj = getattr(cpu_expert, name)
        raw = proj if isinstance(proj, dict) else proj.state
        c = canonical_state(raw, name)
        state[name] = {k: (None if v is None else
                           v if k == "offset" else v.to(device, non_blocking=True))
                       for k, v in c.items()}
    return ReconstructedNF4Expert(cpu_expert, state)

