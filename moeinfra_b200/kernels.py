"""Torch-facing wrappers of the C ABI (device memory and streams come from torch).

Every function validates dtype, device and contiguity the way the reference's
Python layer does, allocates outputs and workspace with the torch caching
allocator, enqueues on the current CUDA stream and raises ``RuntimeError``
with the library's status text on failure.  There is no CPU path.
"""
from __future__ import annotations

import ctypes
import functools
from typing import Sequence

import torch

from moeinfra_b200 import _native
from moeinfra_b200._native import NF4Expert, NF4Matrix, check

NF4_BLOCKSIZE = 64
NESTED_BLOCKSIZE = 256


def _p(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _on_device(fn):
    """Run a wrapper with the device of its first CUDA tensor (or device) argument current.

    The library launches on the stream it is given, and CUDA requires that stream to belong
    to the current device (torch's default stream is the null handle: the current device's
    own).  A call on another GPU's tensors than the current one switches devices for its
    duration, and only then."""
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        dev = None
        for a in (*args, *kwargs.values()):
            if isinstance(a, torch.Tensor) and a.is_cuda:
                dev = a.device.index
                break
            if isinstance(a, torch.device) and a.type == "cuda" and a.index is not None:
                dev = a.index
                break
        if dev is None or dev == torch.cuda.current_device():
            return fn(*args, **kwargs)
        with torch.cuda.device(dev):
            return fn(*args, **kwargs)
    return wrapper


def _need_cuda(what: str, **tensors: torch.Tensor) -> torch.device:
    dev = None
    for name, t in tensors.items():
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{what}: {name} must be a torch.Tensor")
        if t.device.type != "cuda":
            raise RuntimeError(
                f"{what}: {name} is on {t.device}; the B200 kernels run on CUDA tensors only "
                "(there is no CPU path)")
        if not t.is_contiguous():
            raise ValueError(f"{what}: {name} must be contiguous")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{what}: {name} is on {t.device}, expected {dev}")
    assert dev is not None
    return dev


def _need_dtype(what: str, t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype:
        raise ValueError(f"{what}: {name} must be {dtype}, got {t.dtype}")


# Rows an expert stage call may have on the decode kernels (MOE_DECODE_MAX_ROWS).
DECODE_MAX_ROWS = 8


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def check_device(device: torch.device | int | None = None) -> None:
    """Synchronise the current stream of ``device`` and raise if a kernel flagged an error.

    Kernels never trap: a bounded wait that ran out, or experts of one launch
    with different codebooks, leave a bit in the device error word and the
    launch's outputs invalid.  Call this where the caller synchronises anyway
    (the end of a step, before reading results back).
    """
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    with torch.cuda.device(dev):
        status = _native.stream_check(torch.cuda.current_stream(dev).cuda_stream)
    if status != 0:
        raise RuntimeError(f"device check failed: {_native.status_string(status)} (status {status})")


@_on_device
def probe_wait(flag: torch.Tensor, target: int = 1) -> torch.Tensor:
    """One bounded device wait until ``flag[0] >= target``; returns the device-side wait time (ns)."""
    dev = _need_cuda("probe_wait", flag=flag)
    _need_dtype("probe_wait", flag, torch.int32, "flag")
    waited = torch.zeros(1, dtype=torch.int32, device=dev)
    check(_native.lib().moe_probe_wait(_p(flag), int(target), _p(waited), _stream(dev)),
          "moe_probe_wait")
    return waited


# ---------------------------------------------------------------------------
# NF4 dequant
# ---------------------------------------------------------------------------

@_on_device
def nf4_dequant(q: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, numel: int,
                blocksize: int = NF4_BLOCKSIZE) -> torch.Tensor:
    """bf16 ``code[nib(i)] * absmax[i // blocksize]`` (bit-exact), flat [numel]."""
    dev = _need_cuda("nf4_dequant", q=q, absmax=absmax, code=code)
    _need_dtype("nf4_dequant", q, torch.uint8, "q")
    _need_dtype("nf4_dequant", absmax, torch.float32, "absmax")
    _need_dtype("nf4_dequant", code, torch.float32, "code")
    if q.numel() * 2 < numel or absmax.numel() * blocksize < numel or code.numel() < 16:
        raise ValueError("nf4_dequant: buffers too small for numel")
    out = torch.empty(numel, dtype=torch.bfloat16, device=dev)
    check(_native.lib().moe_nf4_dequant(_p(q), _p(absmax), _p(code), numel, blocksize, _p(out),
                                        _stream(dev)), "moe_nf4_dequant")
    return out


@_on_device
def nf4_tile16(q: torch.Tensor, absmax: torch.Tensor, rows: int, cols: int):
    """Store layout -> tile16 device layout (exact permutation); returns (q_t, absmax_t)."""
    dev = _need_cuda("nf4_tile16", q=q, absmax=absmax)
    _need_dtype("nf4_tile16", q, torch.uint8, "q")
    _need_dtype("nf4_tile16", absmax, torch.float32, "absmax")
    if q.numel() * 2 != rows * cols or absmax.numel() * NF4_BLOCKSIZE != rows * cols:
        raise ValueError("nf4_tile16: tensor sizes do not match rows x cols")
    q_out = torch.empty_like(q.reshape(-1))
    a_out = torch.empty_like(absmax.reshape(-1))
    check(_native.lib().moe_nf4_tile16(_p(q), _p(absmax), rows, cols, _p(q_out), _p(a_out),
                                       _stream(dev)), "moe_nf4_tile16")
    return q_out, a_out


@_on_device
def nf4_dequant_tile16(q: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, rows: int,
                       cols: int) -> torch.Tensor:
    """bf16 [rows, cols] of a tile16 matrix (bit-exact with the store-layout dequant)."""
    dev = _need_cuda("nf4_dequant_tile16", q=q, absmax=absmax, code=code)
    out = torch.empty(rows, cols, dtype=torch.bfloat16, device=dev)
    check(_native.lib().moe_nf4_dequant_tile16(_p(q), _p(absmax), _p(code), rows, cols, _p(out),
                                               _stream(dev)), "moe_nf4_dequant_tile16")
    return out


@_on_device
def nested_absmax(qabs: torch.Tensor, absmax2: torch.Tensor, code2: torch.Tensor,
                  offset: float, blocksize2: int = NESTED_BLOCKSIZE) -> torch.Tensor:
    dev = _need_cuda("nested_absmax", qabs=qabs, absmax2=absmax2, code2=code2)
    _need_dtype("nested_absmax", qabs, torch.uint8, "qabs")
    _need_dtype("nested_absmax", absmax2, torch.float32, "absmax2")
    _need_dtype("nested_absmax", code2, torch.float32, "code2")
    n = qabs.numel()
    if absmax2.numel() * blocksize2 < n or code2.numel() < 256:
        raise ValueError("nested_absmax: nested state too small")
    out = torch.empty(n, dtype=torch.float32, device=dev)
    check(_native.lib().moe_nf4_nested_absmax(_p(qabs), _p(absmax2), _p(code2), float(offset), n,
                                              blocksize2, _p(out), _stream(dev)),
          "moe_nf4_nested_absmax")
    return out


# ---------------------------------------------------------------------------
# Router
# ---------------------------------------------------------------------------

@_on_device
def router_topk(h: torch.Tensor, wg: torch.Tensor, k: int, with_logits: bool = True):
    """``(logits fp16 [T,E] | None, weights fp32 [T,k], indices int64 [T,k])``."""
    dev = _need_cuda("router_topk", h=h, wg=wg)
    _need_dtype("router_topk", h, torch.float16, "hidden_states")
    _need_dtype("router_topk", wg, torch.float16, "gate_weight")
    T, H = h.shape
    E = wg.shape[0]
    logits = torch.empty(T, E, dtype=torch.float16, device=dev) if with_logits else None
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    idx = torch.empty(T, k, dtype=torch.int64, device=dev)
    check(_native.lib().moe_router_topk(_p(h), _p(wg), T, H, E, k, _p(logits), _p(w), _p(idx),
                                        _stream(dev)), "moe_router_topk")
    return logits, w, idx


@_on_device
def router_topk_from_logits(logits: torch.Tensor, k: int):
    dev = _need_cuda("router_topk_from_logits", logits=logits)
    _need_dtype("router_topk_from_logits", logits, torch.float16, "logits")
    T, E = logits.shape
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    idx = torch.empty(T, k, dtype=torch.int64, device=dev)
    check(_native.lib().moe_router_topk_from_logits(_p(logits), T, E, k, _p(w), _p(idx),
                                                    _stream(dev)), "moe_router_topk_from_logits")
    return w, idx


# ---------------------------------------------------------------------------
# Experts and the fused layer
# ---------------------------------------------------------------------------

def matrix_desc(q: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor) -> NF4Matrix:
    return NF4Matrix(q.data_ptr(), absmax.data_ptr(), code.data_ptr())


@_on_device
def expert_forward(desc: NF4Expert, x: torch.Tensor, hidden: int, inter: int) -> torch.Tensor:
    dev = _need_cuda("expert_forward", x=x)
    _need_dtype("expert_forward", x, torch.float16, "x")
    if x.ndim != 2 or x.shape[1] != hidden:
        raise ValueError(f"expert_forward: x must be [n, {hidden}], got {tuple(x.shape)}")
    n = x.shape[0]
    y = torch.empty(n, hidden, dtype=torch.float16, device=dev)
    lib = _native.lib()
    ws_bytes = lib.moe_expert_workspace_size(n, hidden, inter)
    ws = _workspace(ws_bytes, dev)
    check(lib.moe_expert_forward(ctypes.byref(desc), _p(x), n, hidden, inter, _p(y), _p(ws),
                                 ws_bytes, _stream(dev)), "moe_expert_forward")
    return y


def expert_array(descs: Sequence[NF4Expert]):
    arr = (NF4Expert * len(descs))()
    for i, d in enumerate(descs):
        arr[i] = d
    return arr


# Decode-sized layer calls reuse one workspace (and routing scratch) per
# (device, stream, shape): calls on one stream are ordered, and every kernel
# of the layer waits for its predecessor before it touches the workspace.
_DECODE_WS_MAX_TOKENS = 8
_layer_ws: dict = {}


def _layer_scratch(dev: torch.device, stream: int, T: int, hidden: int, inter: int, E: int, k: int):
    key = (dev.index, stream, T, hidden, inter, E, k)
    ent = _layer_ws.get(key)
    if ent is None:
        ws_bytes = _native.lib().moe_layer_workspace_size(T, hidden, inter, E, k)
        ent = (_workspace(ws_bytes, dev), ws_bytes,
               torch.empty(T, k, dtype=torch.int64, device=dev),
               torch.empty(T, k, dtype=torch.float32, device=dev))
        if T <= _DECODE_WS_MAX_TOKENS:
            _layer_ws[key] = ent
    return ent


@_on_device
def layer_forward(h: torch.Tensor, wg: torch.Tensor, experts, k: int, hidden: int, inter: int,
                  out: torch.Tensor | None = None, routing: bool = True):
    """Fused MoE layer: returns ``(out fp16 [T,H], indices int64 [T,k], weights fp32 [T,k])``.

    ``experts`` is a ctypes array of ``NF4Expert`` (see :func:`expert_array`).
    ``routing=False``: the caller discards indices and weights (returned as
    None; the kernels write them to reused scratch).
    """
    dev = _need_cuda("layer_forward", h=h, wg=wg)
    _need_dtype("layer_forward", h, torch.float16, "hidden_states")
    _need_dtype("layer_forward", wg, torch.float16, "gate_weight")
    T = h.shape[0]
    E = len(experts)
    if out is None:
        out = torch.empty(T, hidden, dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws, ws_bytes, idx, w = _layer_scratch(dev, stream, T, hidden, inter, E, k)
    if routing:
        idx = torch.empty(T, k, dtype=torch.int64, device=dev)
        w = torch.empty(T, k, dtype=torch.float32, device=dev)
    check(_native.lib().moe_layer_forward(_p(h), _p(wg), experts, E, k, T, hidden, inter, _p(out),
                                          _p(idx), _p(w), _p(ws), ws_bytes,
                                          ctypes.c_void_p(stream)), "moe_layer_forward")
    return (out, idx, w) if routing else (out, None, None)


@_on_device
def layer_forward_noalloc(h: torch.Tensor, wg: torch.Tensor, experts, k: int, hidden: int,
                          inter: int, out: torch.Tensor | None = None):
    """:func:`layer_forward` with the library's own static device scratch (no workspace).

    At most ``MOE_NOALLOC_SCRATCH_BYTES`` of scratch; calls overlapping on one
    device must be serialised.
    """
    dev = _need_cuda("layer_forward_noalloc", h=h, wg=wg)
    _need_dtype("layer_forward_noalloc", h, torch.float16, "hidden_states")
    _need_dtype("layer_forward_noalloc", wg, torch.float16, "gate_weight")
    T = h.shape[0]
    if out is None:
        out = torch.empty(T, hidden, dtype=torch.float16, device=dev)
    idx = torch.empty(T, k, dtype=torch.int64, device=dev)
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    # The library takes the scratch of the CURRENT device: make it h's.
    with torch.cuda.device(dev):
        check(_native.lib().moe_layer_forward_noalloc(_p(h), _p(wg), experts, len(experts), k, T,
                                                      hidden, inter, _p(out), _p(idx), _p(w),
                                                      _stream(dev)), "moe_layer_forward_noalloc")
    return out, idx, w


@_on_device
def routed_layer_forward(h: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor, experts,
                         hidden: int, inter: int) -> torch.Tensor:
    """The MoE layer on routing the caller already has (indices int64 / weights fp32 [T, k]).

    permute -> gather -> experts -> ordered fp16 combine, with no second
    routing pass; every expert slot without tokens in ``indices`` is never read.
    """
    E = len(experts)
    offsets, pair_token, _, pair_slot = permute(indices.contiguous(), weights.contiguous(), E)
    x_sorted = gather_rows(h.contiguous(), pair_token)
    y_sorted = experts_forward(experts, offsets, x_sorted, hidden, inter)
    return combine(y_sorted, pair_slot, indices.contiguous(), weights.contiguous())


@_on_device
def experts_forward(experts, expert_offsets: torch.Tensor, x_sorted: torch.Tensor, hidden: int,
                    inter: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Expert stage on rows grouped by expert (``expert_offsets`` int32 [E+1] on device)."""
    dev = _need_cuda("experts_forward", expert_offsets=expert_offsets, x_sorted=x_sorted)
    _need_dtype("experts_forward", x_sorted, torch.float16, "x_sorted")
    _need_dtype("experts_forward", expert_offsets, torch.int32, "expert_offsets")
    P = x_sorted.shape[0]
    if out is None:
        out = torch.empty(P, hidden, dtype=torch.float16, device=dev)
    lib = _native.lib()
    ws_bytes = lib.moe_experts_workspace_size(P, hidden, inter)
    ws = _workspace(ws_bytes, dev)
    check(lib.moe_experts_forward(experts, len(experts), _p(expert_offsets), _p(x_sorted), P,
                                  hidden, inter, _p(out), _p(ws), ws_bytes, _stream(dev)),
          "moe_experts_forward")
    return out


@_on_device
def permute(indices: torch.Tensor, weights: torch.Tensor, num_experts: int):
    dev = _need_cuda("permute", indices=indices, weights=weights)
    _need_dtype("permute", indices, torch.int64, "indices")
    _need_dtype("permute", weights, torch.float32, "weights")
    T, k = indices.shape
    P = T * k
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    pair_token = torch.empty(P, dtype=torch.int32, device=dev)
    pair_weight = torch.empty(P, dtype=torch.float32, device=dev)
    pair_slot = torch.empty(P, dtype=torch.int32, device=dev)
    check(_native.lib().moe_permute(_p(indices), _p(weights), T, k, num_experts, _p(offsets),
                                    _p(pair_token), _p(pair_weight), _p(pair_slot), _stream(dev)),
          "moe_permute")
    return offsets, pair_token, pair_weight, pair_slot


@_on_device
def gather_rows(rows: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    dev = _need_cuda("gather_rows", rows=rows, index=index)
    _need_dtype("gather_rows", rows, torch.float16, "rows")
    _need_dtype("gather_rows", index, torch.int32, "index")
    out = torch.empty(index.numel(), rows.shape[1], dtype=torch.float16, device=dev)
    check(_native.lib().moe_gather_rows(_p(rows), _p(index), index.numel(), rows.shape[1], _p(out),
                                        _stream(dev)), "moe_gather_rows")
    return out


@_on_device
def combine(y_sorted: torch.Tensor, pair_slot: torch.Tensor, indices: torch.Tensor,
            weights: torch.Tensor) -> torch.Tensor:
    dev = _need_cuda("combine", y_sorted=y_sorted, pair_slot=pair_slot, indices=indices,
                     weights=weights)
    _need_dtype("combine", y_sorted, torch.float16, "y_sorted")
    T, k = indices.shape
    width = y_sorted.shape[1]
    out = torch.empty(T, width, dtype=torch.float16, device=dev)
    check(_native.lib().moe_combine(_p(y_sorted), _p(pair_slot), _p(indices), _p(weights), T, k,
                                    width, _p(out), _stream(dev)), "moe_combine")
    return out


# ---------------------------------------------------------------------------
# Expert-parallel exchange (pack / receive / return around two all-to-alls)
# ---------------------------------------------------------------------------

@_on_device
def ep_dispatch(h: torch.Tensor, offsets: torch.Tensor, pair_token: torch.Tensor,
                pair_slot: torch.Tensor, k: int, num_experts: int, world: int, cap: int):
    """``(send_rows fp16 [world*(cap+1), H], pair_slot_ep int32 [T*k])``.

    Chunk r of ``send_rows`` is cap token rows for rank r followed by a header
    row holding rank r's expert counts (int32).
    """
    dev = _need_cuda("ep_dispatch", h=h, offsets=offsets)
    _need_dtype("ep_dispatch", h, torch.float16, "hidden_states")
    T, H = h.shape
    send = torch.empty(world * (cap + 1), H, dtype=torch.float16, device=dev)
    slot_ep = torch.empty(T * k, dtype=torch.int32, device=dev)
    check(_native.lib().moe_ep_dispatch(_p(h), _p(offsets), _p(pair_token), _p(pair_slot), T, k,
                                        num_experts, world, cap, H, _p(send), None,
                                        _p(slot_ep), _stream(dev)), "moe_ep_dispatch")
    return send, slot_ep


@_on_device
def ep_receive(recv_rows: torch.Tensor, num_experts: int, world: int, cap: int):
    """``(x_sorted fp16 [world*cap, H], local_offsets int32 [E/world + 1], recv_counts int32 [E])``."""
    dev = _need_cuda("ep_receive", recv_rows=recv_rows)
    H = recv_rows.shape[1]
    x = torch.empty(world * cap, H, dtype=torch.float16, device=dev)
    off = torch.empty(num_experts // world + 1, dtype=torch.int32, device=dev)
    counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
    check(_native.lib().moe_ep_receive(_p(recv_rows), _p(counts), num_experts, world, cap, H,
                                       _p(x), _p(off), _stream(dev)), "moe_ep_receive")
    return x, off, counts


@_on_device
def ep_return(y_sorted: torch.Tensor, recv_counts: torch.Tensor, num_experts: int, world: int,
              cap: int) -> torch.Tensor:
    """``y_back fp16 [world*cap, H]`` in the exchanged (source rank, row) layout."""
    dev = _need_cuda("ep_return", y_sorted=y_sorted, recv_counts=recv_counts)
    H = y_sorted.shape[1]
    y_back = torch.empty(world * cap, H, dtype=torch.float16, device=dev)
    check(_native.lib().moe_ep_return(_p(y_sorted), _p(recv_counts), num_experts, world, cap, H,
                                      _p(y_back), _stream(dev)), "moe_ep_return")
    return y_back


# ---------------------------------------------------------------------------
# Expert-parallel exchange over peer memory (see moeinfra_b200.ep_p2p)
# ---------------------------------------------------------------------------

@_on_device
def ep_dispatch_p2p(h: torch.Tensor, offsets: torch.Tensor, pair_token: torch.Tensor,
                    pair_slot: torch.Tensor, k: int, num_experts: int, world: int, rank: int,
                    cap: int, peer_recv: int, peer_flags: int, seq: int, done: int) -> torch.Tensor:
    """Rows straight into the owners' receive regions, then signal; returns pair_slot_ep."""
    dev = _need_cuda("ep_dispatch_p2p", h=h, offsets=offsets)
    T, H = h.shape
    slot_ep = torch.empty(T * k, dtype=torch.int32, device=dev)
    check(_native.lib().moe_ep_dispatch_p2p(_p(h), _p(offsets), _p(pair_token), _p(pair_slot), T,
                                            k, num_experts, world, rank, cap, H,
                                            ctypes.c_void_p(peer_recv), ctypes.c_void_p(peer_flags),
                                            ctypes.c_void_p(seq), ctypes.c_void_p(done),
                                            _p(slot_ep), _stream(dev)), "moe_ep_dispatch_p2p")
    return slot_ep


@_on_device
def ep_return_p2p(y_sorted: torch.Tensor, recv_counts: torch.Tensor, num_experts: int, world: int,
                  rank: int, cap: int, peer_back: int, peer_flags: int, seq: int, done: int) -> None:
    dev = _need_cuda("ep_return_p2p", y_sorted=y_sorted, recv_counts=recv_counts)
    check(_native.lib().moe_ep_return_p2p(_p(y_sorted), _p(recv_counts), num_experts, world, rank,
                                          cap, y_sorted.shape[1], ctypes.c_void_p(peer_back),
                                          ctypes.c_void_p(peer_flags), ctypes.c_void_p(seq),
                                          ctypes.c_void_p(done), _stream(dev)), "moe_ep_return_p2p")


@_on_device
def ep_wait_p2p(flags: int, world: int, seq: int, device: torch.device) -> None:
    check(_native.lib().moe_ep_wait_p2p(ctypes.c_void_p(flags), world, ctypes.c_void_p(seq),
                                        _stream(device)), "moe_ep_wait_p2p")


@_on_device
def ep_receive_rows(recv_rows: torch.Tensor, num_experts: int, world: int, cap: int):
    """:func:`ep_receive` on a receive region that is a view (peer-memory exchange)."""
    return ep_receive(recv_rows, num_experts, world, cap)


@_on_device
def ep_receive_p2p(recv_rows: torch.Tensor, num_experts: int, world: int, cap: int, flags: int,
                   seq: int):
    """:func:`ep_receive` of a peer-memory receive region, waiting (bounded, in the kernel)
    for all ``world`` flags at ``flags`` to reach ``*seq`` first."""
    dev = _need_cuda("ep_receive_p2p", recv_rows=recv_rows)
    H = recv_rows.shape[1]
    x = torch.empty(world * cap, H, dtype=torch.float16, device=dev)
    off = torch.empty(num_experts // world + 1, dtype=torch.int32, device=dev)
    counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
    check(_native.lib().moe_ep_receive_p2p(_p(recv_rows), _p(counts), num_experts, world, cap, H,
                                           _p(x), _p(off), ctypes.c_void_p(flags),
                                           ctypes.c_void_p(seq), _stream(dev)),
          "moe_ep_receive_p2p")
    return x, off, counts


@_on_device
def combine_p2p(y_back: torch.Tensor, pair_slot: torch.Tensor, indices: torch.Tensor,
                weights: torch.Tensor, world: int, flags: int, seq: int) -> torch.Tensor:
    """:func:`combine` of a peer-memory return region, waiting (bounded, in the kernel) for all
    ``world`` flags at ``flags`` to reach ``*seq`` first."""
    dev = _need_cuda("combine_p2p", y_back=y_back, pair_slot=pair_slot, indices=indices,
                     weights=weights)
    _need_dtype("combine_p2p", y_back, torch.float16, "y_back")
    T, k = indices.shape
    width = y_back.shape[1]
    out = torch.empty(T, width, dtype=torch.float16, device=dev)
    check(_native.lib().moe_combine_p2p(_p(y_back), _p(pair_slot), _p(indices), _p(weights), T,
                                        k, width, _p(out), ctypes.c_void_p(flags), world,
                                        ctypes.c_void_p(seq), _stream(dev)), "moe_combine_p2p")
    return out


@_on_device
def ep_front_p2p(h: torch.Tensor, gate_f16: torch.Tensor, k: int, num_experts: int, world: int,
                 rank: int, cap: int, peer_recv: int, peer_flags: int, seq: int, done: int,
                 bar: int, zero: torch.Tensor | None = None):
    """Router, permute and the peer-memory dispatch in one launch (``T`` <= the SM count).

    Returns ``(weights fp32 [T, k], indices int64 [T, k], pair_slot_ep int32 [T*k])``, the
    values :func:`router_topk`, :func:`permute` and :func:`ep_dispatch_p2p` give.  ``zero``
    (int32, optional) is zeroed by the same launch: the counters of the expert stage that
    follows (:func:`experts_forward_partials` ``counters``)."""
    dev = _need_cuda("ep_front_p2p", h=h, gate_f16=gate_f16)
    _need_dtype("ep_front_p2p", h, torch.float16, "h")
    _need_dtype("ep_front_p2p", gate_f16, torch.float16, "gate_f16")
    T, H = h.shape
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    idx = torch.empty(T, k, dtype=torch.int64, device=dev)
    slot_ep = torch.empty(T * k, dtype=torch.int32, device=dev)
    check(_native.lib().moe_ep_front_p2p(_p(h), _p(gate_f16), T, num_experts, k, world, rank, cap,
                                         H, ctypes.c_void_p(peer_recv),
                                         ctypes.c_void_p(peer_flags), ctypes.c_void_p(seq),
                                         ctypes.c_void_p(done), ctypes.c_void_p(bar), _p(w),
                                         _p(idx), _p(slot_ep),
                                         None if zero is None else _p(zero),
                                         0 if zero is None else zero.numel(), _stream(dev)),
          "moe_ep_front_p2p")
    return w, idx, slot_ep


def expert_splits(inter: int) -> int:
    """K splits of the decode down projection (its fp32 partials per row)."""
    return int(_native.lib().moe_expert_splits(inter))


def expert_counter_words(inter: int) -> int:
    """int32 completion counters of the decode expert stage (zeroed before each call)."""
    return int(_native.lib().moe_experts_counter_words(inter))


@_on_device
def experts_forward_partials(experts, expert_offsets: torch.Tensor, x_sorted: torch.Tensor,
                             hidden: int, inter: int,
                             counters: torch.Tensor | None = None) -> torch.Tensor:
    """:func:`experts_forward` of a decode batch (<= 8 rows) up to the down projection's
    fp32 split partials ``[P, S, hidden]`` (their in-order fp16 sum is the output row).
    ``counters``: :func:`expert_counter_words` int32 already zeroed on the stream (by
    :func:`ep_front_p2p`), which spares the zeroing launch; None zeroes internal ones."""
    dev = _need_cuda("experts_forward_partials", expert_offsets=expert_offsets, x_sorted=x_sorted)
    _need_dtype("experts_forward_partials", x_sorted, torch.float16, "x_sorted")
    _need_dtype("experts_forward_partials", expert_offsets, torch.int32, "expert_offsets")
    P = x_sorted.shape[0]
    part = torch.empty(P, expert_splits(inter), hidden, dtype=torch.float32, device=dev)
    lib = _native.lib()
    ws_bytes = lib.moe_experts_workspace_size(P, hidden, inter)
    ws = _workspace(ws_bytes, dev)
    if counters is not None and counters.numel() < expert_counter_words(inter):
        raise ValueError("counters smaller than expert_counter_words(inter)")
    check(lib.moe_experts_forward_partials(experts, len(experts), _p(expert_offsets),
                                           _p(x_sorted), P, hidden, inter, _p(part),
                                           None if counters is None else _p(counters), _p(ws),
                                           ws_bytes, _stream(dev)),
          "moe_experts_forward_partials")
    return part


@_on_device
def ep_return_partials_p2p(y_part: torch.Tensor, recv_counts: torch.Tensor, num_experts: int,
                           world: int, rank: int, cap: int, peer_back: int, peer_flags: int,
                           seq: int, done: int) -> None:
    """:func:`ep_return_p2p` from :func:`experts_forward_partials`' fp32 partials."""
    dev = _need_cuda("ep_return_partials_p2p", y_part=y_part, recv_counts=recv_counts)
    _need_dtype("ep_return_partials_p2p", y_part, torch.float32, "y_part")
    check(_native.lib().moe_ep_return_partials_p2p(
        _p(y_part), y_part.shape[1], _p(recv_counts), num_experts, world, rank, cap,
        y_part.shape[2], ctypes.c_void_p(peer_back), ctypes.c_void_p(peer_flags),
        ctypes.c_void_p(seq), ctypes.c_void_p(done), _stream(dev)), "moe_ep_return_partials_p2p")
