"""NF4 oracle (numpy) — TEST INFRASTRUCTURE ONLY, never imported by the product.

Restates the arithmetic the reference reaches through bitsandbytes 0.50.2
``Linear4bit`` (pinned in the reference's ``requirements.txt:3``; the package
is not vendored in the reference and is not installed here).

Reference call sites this follows:

* ``transfer/nf4_reconstruct.py:9-14``  blocksize 64, dequant dtype bf16,
  nested blocksize 256, nested dtype fp32.
* ``transfer/nf4_reconstruct.py:45-54`` QuantState(absmax, shape=(out,in),
  code, offset, state2).
* ``transfer/nf4_reconstruct.py:94``    compute dtype fp16.
* ``transfer/nf4_reconstruct.py:152-155`` ``w2(silu(w1(x)) * w3(x))``.
* ``model/expert.py:49-55``             store built with
  ``compress_statistics=False`` (fp32 absmax).

bitsandbytes' published algorithm, restated:

* Packing: byte ``j`` of the packed weight holds element ``2j`` in its HIGH
  nibble and element ``2j+1`` in its LOW nibble, row-major over [out, in].
* Dequant (``dequantize_4bit``): ``w[i] = dtype(code[nib(i)] * absmax[i // 64])``
  with the product formed in fp32 and rounded once to bf16
  (round-to-nearest-even).  With double quantization the fp32 absmax is
  first rebuilt as ``code2[qabs[b]] * absmax2[b // 256]`` (fp32) ``+ offset``
  (fp32), two separately rounded operations.
* ``Linear4bit.forward`` with fp16 input takes one of two paths
  (``bnb.matmul_4bit``):

  - single-row input (``x.numel() == x.shape[-1]``, no grad): the 4-bit
    inference GEMV.  Each weight is ``fp16(fp16(code[n]) * fp16(absmax))``;
    the row dot product accumulates ``fp32(x) * fp32(w)`` in fp32 and is
    rounded once to fp16.  (This is the kernel's sm_75 branch, which is what
    the reference's published T4 numbers ran on.  The sm_80+ branch rounds
    each product to fp16 before accumulating; the two differ by ~1e-4
    relative, far inside the expert tolerance.)
  - otherwise: dequantize to bf16, cast to fp16 (``.to(A.dtype)``), then an
    fp16 GEMM with fp32 accumulation (cuBLAS), output rounded to fp16.

Parity status: the codebook is pinned to the published QLoRA NF4 table
(Dettmers et al. 2023, appendix) and the dequant to hand-computed
known-answer vectors in ``tests/test_oracle.py``.  bitsandbytes' own kernels
could not be run here: "parity unpinned" against bitsandbytes itself.
"""
from __future__ import annotations

import numpy as np

NF4_BLOCKSIZE = 64          # transfer/nf4_reconstruct.py:9
NESTED_BLOCKSIZE = 256      # transfer/nf4_reconstruct.py:13

# Published QLoRA NF4 table (fp32), used only to pin nf4_codebook().
PUBLISHED_NF4 = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
    0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
    0.7229568362236023, 1.0,
)


# ---------------------------------------------------------------------------
# Codebooks
# ---------------------------------------------------------------------------

def nf4_codebook() -> np.ndarray:
    """The 16-entry NF4 codebook from its published construction.

    NF4 (QLoRA): 8 positive normal quantiles over linspace(0.9677083, 0.5, 9)
    minus its last point, 7 negative ones over linspace(0.9677083, 0.5, 8)
    minus its last point, plus an exact zero; sorted and normalised by the
    maximum.  The linspace is torch's fp32 linspace (as in the published
    construction), the quantiles fp64, the normalisation fp32.
    """
    import torch
    from scipy.stats import norm

    offset = 0.9677083
    pos = norm.ppf(torch.linspace(offset, 0.5, 9)[:-1].numpy().astype(np.float64))
    neg = -norm.ppf(torch.linspace(offset, 0.5, 8)[:-1].numpy().astype(np.float64))
    vals = np.sort(np.concatenate([pos, [0.0], neg]).astype(np.float32))
    return (vals / vals.max()).astype(np.float32)


def dynamic_map_signed() -> np.ndarray:
    """256-entry signed dynamic ("tree") 8-bit map used for nested absmax.

    Published construction (Dettmers et al., 8-bit optimizers): for each
    exponent i in 0..6, 2**i fraction means of linspace(0.1, 1, 2**i + 1),
    scaled by 10**(i - 6), with both signs; plus 0 and 1.0; sorted.
    """
    import torch

    data: list[float] = []
    for i in range(7):
        bounds = torch.linspace(0.1, 1.0, 2 ** i + 1).numpy()
        means = (bounds[:-1] + bounds[1:]) / np.float32(2.0)
        scale = 10.0 ** (i - 6)
        data += (scale * means.astype(np.float64)).tolist()
        data += (-scale * means.astype(np.float64)).tolist()
    data += [0.0, 1.0]
    assert len(data) == 256
    return np.sort(np.asarray(data, dtype=np.float32))


# ---------------------------------------------------------------------------
# Rounding helpers (bit-level, no platform float16 tricks for bf16)
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern, round to nearest even; NaN stays quiet NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32)
    lsb = (b >> np.uint32(16)) & np.uint32(1)
    r = ((b + np.uint32(0x7FFF) + lsb) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = r.copy()
        r[nan] = ((b[nan] >> np.uint32(16)) | np.uint32(0x0040)).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_bits_to_f16(b: np.ndarray) -> np.ndarray:
    """bf16 -> fp16 as torch's ``.to(torch.float16)`` does (one RN rounding)."""
    return bf16_bits_to_f32(b).astype(np.float16)


# ---------------------------------------------------------------------------
# Packing / dequant
# ---------------------------------------------------------------------------

def unpack_nf4(q: np.ndarray) -> np.ndarray:
    """Packed bytes -> nibble indices; element 2j = high nibble of byte j."""
    q = np.asarray(q, dtype=np.uint8).reshape(-1)
    out = np.empty(q.size * 2, dtype=np.uint8)
    out[0::2] = q >> 4
    out[1::2] = q & 0x0F
    return out


def pack_nf4(idx: np.ndarray) -> np.ndarray:
    idx = np.asarray(idx, dtype=np.uint8).reshape(-1)
    assert idx.size % 2 == 0
    return ((idx[0::2] << 4) | (idx[1::2] & 0x0F)).astype(np.uint8)


def nested_absmax(qabs: np.ndarray, absmax2: np.ndarray, code2: np.ndarray,
                  offset: float, blocksize2: int = NESTED_BLOCKSIZE) -> np.ndarray:
    """Rebuild fp32 absmax from its 8-bit double quantization.

    ``absmax[b] = fp32(fp32(code2[qabs[b]] * absmax2[b // 256]) + offset)``.
    """
    qabs = np.asarray(qabs, dtype=np.uint8).reshape(-1)
    blk = np.arange(qabs.size) // blocksize2
    prod = (np.asarray(code2, np.float32)[qabs] * np.asarray(absmax2, np.float32)[blk]).astype(np.float32)
    return (prod + np.float32(offset)).astype(np.float32)


def dequant_nf4_bf16(q: np.ndarray, absmax: np.ndarray, code: np.ndarray,
                     numel: int, blocksize: int = NF4_BLOCKSIZE) -> np.ndarray:
    """bf16 bit patterns of ``code[nib(i)] * absmax[i // blocksize]``."""
    nib = unpack_nf4(q)[:numel]
    blk = np.arange(numel, dtype=np.int64) // blocksize
    prod = (np.asarray(code, np.float32)[nib] * np.asarray(absmax, np.float32)[blk]).astype(np.float32)
    return f32_to_bf16_bits(prod)


def dequant_weight_f16(state: dict, shape: tuple[int, int]) -> np.ndarray:
    """Weight as the reference's multi-row path sees it: bf16 dequant -> fp16."""
    numel = shape[0] * shape[1]
    bits = dequant_nf4_bf16(state["weight"], resolve_absmax(state), state["code"], numel)
    return bf16_bits_to_f16(bits).reshape(shape)


def resolve_absmax(state: dict) -> np.ndarray:
    if state.get("state2_absmax") is not None:
        off = state.get("offset")
        off = 0.0 if off is None else float(np.asarray(off, np.float32).reshape(-1)[0])
        return nested_absmax(state["absmax"], state["state2_absmax"], state["state2_code"], off)
    return np.asarray(state["absmax"], dtype=np.float32).reshape(-1)


# ---------------------------------------------------------------------------
# Quantizer (synthetic stores only; parity with bitsandbytes' quantizer is
# not claimed: bnb's nearest-code thresholds are decimal literals)
# ---------------------------------------------------------------------------

def quantize_nf4(w: np.ndarray, code: np.ndarray | None = None,
                 blocksize: int = NF4_BLOCKSIZE) -> tuple[np.ndarray, np.ndarray]:
    """Blockwise absmax NF4 quantization of a fp32 view of bf16 weights.

    Returns ``(packed uint8 [numel/2], absmax fp32 [numel/blocksize])``.
    Nearest code by midpoints; a value exactly on a midpoint takes the lower
    code (strict ``>`` comparisons).
    """
    code = nf4_codebook() if code is None else np.asarray(code, np.float32)
    flat = np.asarray(w, dtype=np.float32).reshape(-1)
    assert flat.size % blocksize == 0
    blocks = flat.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax == 0, np.float32(1.0), absmax).astype(np.float32)
    norm = (blocks / safe[:, None]).astype(np.float32)
    mids = ((code[:-1] + code[1:]) / np.float32(2.0)).astype(np.float32)
    idx = np.searchsorted(mids, norm.reshape(-1), side="left").astype(np.uint8)
    return pack_nf4(idx), absmax


def quantize_absmax_nested(absmax: np.ndarray, blocksize2: int = NESTED_BLOCKSIZE):
    """Double quantization of an fp32 absmax vector (8-bit dynamic map)."""
    code2 = dynamic_map_signed()
    a = np.asarray(absmax, np.float32).reshape(-1)
    offset = np.float32(a.mean(dtype=np.float64))
    centred = (a - offset).astype(np.float32)
    n = centred.size
    nb = (n + blocksize2 - 1) // blocksize2
    pad = np.zeros(nb * blocksize2, np.float32)
    pad[:n] = centred
    blocks = pad.reshape(nb, blocksize2)
    absmax2 = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax2 == 0, np.float32(1.0), absmax2)
    normed = (blocks / safe[:, None]).reshape(-1)[:n].astype(np.float32)
    pos = np.clip(np.searchsorted(code2, normed), 1, 255)
    lo, hi = code2[pos - 1], code2[pos]
    q = np.where(np.abs(normed - lo) <= np.abs(hi - normed), pos - 1, pos).astype(np.uint8)
    return q, absmax2, code2, offset


# ---------------------------------------------------------------------------
# Linear layers in the two bitsandbytes semantics, SwiGLU, expert
# ---------------------------------------------------------------------------

def linear_multirow(x16: np.ndarray, w16: np.ndarray) -> np.ndarray:
    """fp16 GEMM with wide accumulation: ``fp16(sum_k x[k] * w[n,k])``."""
    acc = np.asarray(x16, np.float64) @ np.asarray(w16, np.float64).T
    return acc.astype(np.float16)


def gemv_weight_f16(state: dict, shape: tuple[int, int]) -> np.ndarray:
    """Per-weight value of the single-row path: fp16(fp16(code) * fp16(absmax))."""
    numel = shape[0] * shape[1]
    nib = unpack_nf4(state["weight"])[:numel]
    absmax = resolve_absmax(state)
    blk = np.arange(numel, dtype=np.int64) // NF4_BLOCKSIZE
    c16 = np.asarray(state["code"], np.float32).astype(np.float16).astype(np.float32)
    a16 = absmax.astype(np.float16).astype(np.float32)
    return (c16[nib] * a16[blk]).astype(np.float16).reshape(shape)


def linear_nf4(x16: np.ndarray, state: dict, shape: tuple[int, int]) -> np.ndarray:
    """``Linear4bit(x)`` for fp16 ``x`` of shape [n, in]; picks bnb's path by n."""
    x16 = np.asarray(x16, np.float16)
    if x16.shape[0] == 1:
        return linear_multirow(x16, gemv_weight_f16(state, shape))
    return linear_multirow(x16, dequant_weight_f16(state, shape))


def silu_f16(g16: np.ndarray) -> np.ndarray:
    """torch ``F.silu`` on fp16: ``x / (1 + exp(-x))`` in fp32, rounded to fp16."""
    g = np.asarray(g16, np.float16).astype(np.float32)
    with np.errstate(over="ignore"):
        s = g / (np.float32(1.0) + np.exp(-g))
    return s.astype(np.float16)


def swiglu_f16(g16: np.ndarray, u16: np.ndarray) -> np.ndarray:
    """``F.silu(gate) * up`` on fp16 tensors (fp32 product, one fp16 rounding)."""
    s = silu_f16(g16).astype(np.float32)
    return (s * np.asarray(u16, np.float16).astype(np.float32)).astype(np.float16)


def expert_forward(x16: np.ndarray, expert: dict, hidden: int, inter: int) -> np.ndarray:
    """SwiGLU expert ``w2(silu(w1 x) * w3 x)`` (``nf4_reconstruct.py:152-155``).

    ``expert`` maps ``w1``/``w2``/``w3`` to canonical states
    ``{weight, absmax, code, offset, [state2_absmax, state2_code]}``.
    """
    g = linear_nf4(x16, expert["w1"], (inter, hidden))
    u = linear_nf4(x16, expert["w3"], (inter, hidden))
    h = swiglu_f16(g, u)
    return linear_nf4(h, expert["w2"], (hidden, inter))


def make_expert(rng: np.random.Generator, hidden: int, inter: int,
                std: float = 0.02, nested: bool = False) -> dict:
    """Seeded synthetic NF4 expert: N(0, std) weights rounded to bf16, quantized."""
    code = nf4_codebook()
    out = {}
    for name, shape in (("w1", (inter, hidden)), ("w3", (inter, hidden)), ("w2", (hidden, inter))):
        w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        w = bf16_bits_to_f32(f32_to_bf16_bits(w))  # the reference quantizes bf16 weights
        q, absmax = quantize_nf4(w, code)
        st = {"weight": q, "absmax": absmax, "code": code.copy(), "offset": None}
        if nested:
            qa, a2, c2, off = quantize_absmax_nested(absmax)
            st = {"weight": q, "absmax": qa, "code": code.copy(), "offset": np.float32(off),
                  "state2_absmax": a2, "state2_code": c2, "state2_offset": None}
        out[name] = st
    return out


# ---------------------------------------------------------------------------
# tile16 device layout (this build's resident layout; an exact permutation)
# ---------------------------------------------------------------------------

def tile16(q: np.ndarray, absmax: np.ndarray, rows: int, cols: int):
    """Store layout -> tile16: (16-row tile, 64-element block, row, 32 bytes)."""
    nblk = cols // 64
    qb = np.asarray(q, np.uint8).reshape(rows // 16, 16, nblk, 32)
    ab = np.asarray(absmax, np.float32).reshape(rows // 16, 16, nblk)
    return (np.ascontiguousarray(qb.transpose(0, 2, 1, 3)).reshape(-1),
            np.ascontiguousarray(ab.transpose(0, 2, 1)).reshape(-1))
