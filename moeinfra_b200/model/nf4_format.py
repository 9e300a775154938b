"""NF4 expert-store format: serialized state <-> canonical state, and a quantizer.

The store (one safetensors file per expert, ``model/loader.py:303-316`` of the
reference) keeps each projection ``w1``/``w2``/``w3`` in the bitsandbytes
``Linear4bit.state_dict()`` layout:

* ``weight``                               uint8, packed codes (2 per byte; element
  2j in the high nibble of byte j), row-major over [out, in];
* ``weight.absmax``                        fp32 [numel/64] (uint8 when nested);
* ``weight.quant_map``                     fp32 [16] codebook;
* ``weight.nested_absmax`` / ``weight.nested_quant_map``   (nested only);
* ``weight.quant_state.bitsandbytes__nf4`` uint8 bytes of a UTF-8 JSON object with
  ``quant_type``, ``blocksize``, ``dtype``, ``shape`` and, when nested,
  ``nested_blocksize``, ``nested_dtype``, ``nested_offset``.

The canonical in-memory form (``transfer/reusable_staging.py:126-222``) is
``{weight, absmax, code, offset[, state2_absmax, state2_code, state2_offset]}``.
Blobs that are not valid JSON (the reference's own loader fixture uses eight
arbitrary bytes, ``tests/test_model_loader_fast_path.py:93-96``) are tolerated:
defaults (nf4, blocksize 64, not nested) apply.
"""
from __future__ import annotations

import json
from typing import Optional

import torch

BLOB_KEY = "weight.quant_state.bitsandbytes__nf4"
NF4_BLOCKSIZE = 64
NESTED_BLOCKSIZE = 256

# The NF4 data type (QLoRA, Dettmers et al. 2023): 16 normal-distribution
# quantiles normalised to [-1, 1], exactly representable in fp32.
NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
    0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
    0.7229568362236023, 1.0,
)

REQUIRED_SERIALIZED_KEYS = {"weight", "weight.absmax", "weight.quant_map", BLOB_KEY}
PROJECTIONS = ("w1", "w2", "w3")


def nf4_code_tensor(device: torch.device | str = "cpu") -> torch.Tensor:
    return torch.tensor(NF4_CODE, dtype=torch.float32, device=device)


def pack_blob(meta: dict) -> torch.Tensor:
    return torch.tensor(list(json.dumps(meta).encode("utf-8")), dtype=torch.uint8)


def parse_blob(blob: Optional[torch.Tensor]) -> Optional[dict]:
    """Decode the JSON metadata blob; ``None`` when it is absent or not JSON."""
    if blob is None:
        return None
    try:
        raw = bytes(blob.detach().to("cpu", torch.uint8).reshape(-1).tolist())
        meta = json.loads(raw.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError, ValueError):
        return None
    return meta if isinstance(meta, dict) else None


def canonical_state(raw: dict, name: str = "projection") -> dict:
    """Canonical staging form of one projection (serialized or canonical input)."""
    if "weight" not in raw:
        raise ValueError(f"Projection {name!r} is missing 'weight'")
    if "absmax" in raw and ("code" in raw or "quant_map" in raw):
        st = {
            "weight": raw["weight"],
            "absmax": raw["absmax"],
            "code": raw.get("code", raw.get("quant_map")),
            "offset": raw.get("offset"),
        }
        for key in ("state2_absmax", "state2_code", "state2_offset"):
            if key in raw:
                st[key] = raw[key]
        if st["code"] is None:
            raise ValueError(f"Projection {name!r} is missing NF4 code/quant_map")
        return st
    missing = {"weight.absmax", "weight.quant_map", BLOB_KEY} - raw.keys()
    if missing:
        raise ValueError(
            f"Projection {name!r} is missing serialized NF4 state tensors: {sorted(missing)}")
    meta = parse_blob(raw[BLOB_KEY]) or {}
    if meta.get("quant_type", "nf4") != "nf4":
        raise ValueError(f"Projection {name!r}: unsupported quant_type {meta.get('quant_type')!r}")
    if int(meta.get("blocksize", NF4_BLOCKSIZE)) != NF4_BLOCKSIZE:
        raise ValueError(f"Projection {name!r}: only blocksize {NF4_BLOCKSIZE} is supported")
    st = {
        "weight": raw["weight"],
        "absmax": raw["weight.absmax"],
        "code": raw["weight.quant_map"],
        "offset": None,
    }
    if "weight.nested_absmax" in raw or "nested_offset" in meta:
        if "weight.nested_absmax" not in raw or "weight.nested_quant_map" not in raw:
            raise ValueError(f"Projection {name!r}: incomplete nested NF4 state")
        st["offset"] = torch.tensor(float(meta.get("nested_offset", 0.0)), dtype=torch.float32)
        st["state2_absmax"] = raw["weight.nested_absmax"]
        st["state2_code"] = raw["weight.nested_quant_map"]
        st["state2_offset"] = None
    return st


def is_nested(state: dict) -> bool:
    return state.get("state2_absmax") is not None or state.get("state2_code") is not None


def check_projection_sizes(state: dict, in_features: int, out_features: int,
                           name: str = "projection") -> None:
    """Raise ``ValueError`` when a canonical projection's tensors do not cover [out, in].

    A store file cut short, or a blob that lies about the shape, is caught on
    the host before any byte is staged or copied to the GPU.
    """
    numel = in_features * out_features
    w = state.get("weight")
    if w is None or w.numel() * 2 != numel:
        got = None if w is None else w.numel()
        raise ValueError(f"{name}: packed weight has {got} bytes, expected {numel // 2} "
                         f"for [{out_features}, {in_features}]")
    a = state.get("absmax")
    if a is None or a.numel() * NF4_BLOCKSIZE != numel:
        got = None if a is None else a.numel()
        raise ValueError(f"{name}: absmax has {got} entries, expected {numel // NF4_BLOCKSIZE}")
    c = state.get("code")
    if c is None or c.numel() != 16:
        raise ValueError(f"{name}: NF4 codebook must have 16 entries")
    if is_nested(state):
        a2 = state.get("state2_absmax")
        need = -(-a.numel() // NESTED_BLOCKSIZE)
        if a2 is None or a2.numel() < need or state.get("state2_code") is None:
            raise ValueError(f"{name}: nested absmax state is incomplete")


# ---------------------------------------------------------------------------
# Store files (one safetensors file per expert)
# ---------------------------------------------------------------------------

def store_file_name(layer_id: int, expert_id: int) -> str:
    """``layer_LL_expert_EE.safetensors`` (the reference's ``model/loader.py:305``)."""
    return f"layer_{layer_id:02d}_expert_{expert_id:02d}.safetensors"


def expert_store_tensors(expert) -> dict:
    """Flat store dict ``{"w1.weight": ..., "w1.weight.absmax": ..., ...}`` of an expert.

    ``expert`` exposes ``w1``/``w2``/``w3`` as serialized state dicts
    (``PrequantizedNF4Expert``) or as modules with a ``.state`` dict
    (``QuantizedMixtralExpert``'s projections).
    """
    out = {}
    for proj in PROJECTIONS:
        st = getattr(expert, proj)
        st = st if isinstance(st, dict) else st.state
        for key, t in st.items():
            if isinstance(t, torch.Tensor):
                out[f"{proj}.{key}"] = t.detach().to("cpu").contiguous()
    return out


def save_expert_store(store_dir, layer_id: int, expert_id: int, expert):
    """Write one expert to ``store_dir`` in the store format; returns the file path."""
    from pathlib import Path

    from safetensors.torch import save_file

    path = Path(store_dir) / store_file_name(layer_id, expert_id)
    path.parent.mkdir(parents=True, exist_ok=True)
    save_file(expert_store_tensors(expert), str(path))
    return path


# ---------------------------------------------------------------------------
# Quantizer (store writer; not on the inference path)
# ---------------------------------------------------------------------------

def _dynamic_map_signed() -> torch.Tensor:
    """Signed 8-bit dynamic ("tree") map used for double-quantized absmax."""
    data: list[float] = []
    for i in range(7):
        bounds = torch.linspace(0.1, 1.0, 2 ** i + 1, dtype=torch.float32)
        means = (bounds[:-1] + bounds[1:]) / 2.0
        scale = 10.0 ** (i - 6)
        data += (scale * means.double()).tolist()
        data += (-scale * means.double()).tolist()
    data += [0.0, 1.0]
    return torch.tensor(sorted(data), dtype=torch.float32)


def quantize_nf4_packed(weight: torch.Tensor, blocksize: int = NF4_BLOCKSIZE):
    """Blockwise NF4 quantization on the weight's own device.

    Returns ``(packed uint8 [numel/2], absmax fp32 [numel/blocksize], code fp32 [16])``
    in the store layout: nearest code (a value exactly on a midpoint takes the
    lower code), element 2j in the high nibble of byte j.
    """
    flat = weight.detach().to(torch.float32).reshape(-1)
    if flat.numel() % blocksize:
        raise ValueError(f"weight numel {flat.numel()} is not a multiple of {blocksize}")
    code = nf4_code_tensor(flat.device)
    blocks = flat.view(-1, blocksize)
    absmax = blocks.abs().amax(dim=1)
    safe = torch.where(absmax == 0, torch.ones_like(absmax), absmax)
    normed = (blocks / safe[:, None]).reshape(-1)
    mids = (code[:-1] + code[1:]) / 2.0
    idx = torch.bucketize(normed, mids, right=False, out_int32=True).to(torch.uint8)
    packed = ((idx[0::2] << 4) | idx[1::2]).contiguous()
    return packed, absmax, code


def quantize_linear_state(weight: torch.Tensor, compress_statistics: bool = False) -> dict:
    """Serialized NF4 state of one [out, in] weight (alias of :func:`quantize_nf4`)."""
    return quantize_nf4(weight, compress_statistics=compress_statistics)


def quantize_nf4(weight: torch.Tensor, compress_statistics: bool = False,
                 blocksize: int = NF4_BLOCKSIZE) -> dict:
    """Quantize a 2-D weight [out, in] to a serialized NF4 projection state.

    Blockwise absmax scaling, nearest NF4 code (a value exactly on a midpoint
    takes the lower code), two codes per byte, high nibble first.  With
    ``compress_statistics`` the absmax vector is double-quantized (mean offset,
    256-blocks, signed dynamic 8-bit map) as bitsandbytes does.
    """
    if weight.ndim != 2:
        raise ValueError(f"Expected a 2D weight tensor, got shape {tuple(weight.shape)}")
    out_f, in_f = weight.shape
    packed, absmax, code = quantize_nf4_packed(weight, blocksize)
    meta = {"quant_type": "nf4", "blocksize": blocksize, "dtype": "bfloat16",
            "shape": [out_f, in_f]}
    st = {"weight": packed.cpu(), "weight.quant_map": code.cpu()}
    if compress_statistics:
        offset = absmax.double().mean().float()
        centred = (absmax - offset).float()
        n = centred.numel()
        nb = (n + NESTED_BLOCKSIZE - 1) // NESTED_BLOCKSIZE
        pad = torch.zeros(nb * NESTED_BLOCKSIZE, dtype=torch.float32, device=centred.device)
        pad[:n] = centred
        a2 = pad.view(nb, NESTED_BLOCKSIZE).abs().amax(dim=1)
        safe2 = torch.where(a2 == 0, torch.ones_like(a2), a2)
        normed2 = (pad.view(nb, NESTED_BLOCKSIZE) / safe2[:, None]).reshape(-1)[:n]
        code2 = _dynamic_map_signed().to(centred.device)
        pos = torch.bucketize(normed2, code2).clamp(1, 255)
        lo, hi = code2[pos - 1], code2[pos]
        q2 = torch.where((normed2 - lo).abs() <= (hi - normed2).abs(), pos - 1, pos).to(torch.uint8)
        st["weight.absmax"] = q2.cpu()
        st["weight.nested_absmax"] = a2.cpu()
        st["weight.nested_quant_map"] = code2.cpu()
        meta.update({"nested_blocksize": NESTED_BLOCKSIZE, "nested_dtype": "float32",
                     "nested_offset": float(offset)})
    else:
        st["weight.absmax"] = absmax.float().cpu()
    st[BLOB_KEY] = pack_blob(meta)
    return st
