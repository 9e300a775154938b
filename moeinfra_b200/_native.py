"""ctypes binding of ``libmoe_b200.so`` (the C ABI in ``include/moe_b200.h``).

The library is built in-tree by ``moeinfra_b200.build``.  There is no
fallback: if the library is missing or fails to load, every kernel entry
point raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmoe_b200.so"

MOE_MAX_EXPERTS = 16
MOE_ERR_TIMEOUT = 6
MOE_ERR_CODEBOOK = 7
MOE_NOALLOC_SCRATCH_BYTES = 4 << 20


class NF4Matrix(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("absmax", c_void_p), ("code", c_void_p)]


class NF4Expert(ctypes.Structure):
    _fields_ = [("w1", NF4Matrix), ("w3", NF4Matrix), ("w2", NF4Matrix)]


# name -> (restype, argtypes); mirrors include/moe_b200.h one to one.
SIGNATURES: dict[str, tuple] = {
    "moe_status_string": (ctypes.c_char_p, [c_int]),
    "moe_version": (ctypes.c_char_p, []),
    "moe_launch_count": (ctypes.c_uint64, []),
    "moe_take_device_error": (c_int, [ctypes.POINTER(c_int)]),
    "moe_stream_check": (c_int, [c_void_p]),
    "moe_set_wait_limit_ns": (c_int, [ctypes.c_uint64]),
    "moe_wait_limit_ns": (ctypes.c_uint64, []),
    "moe_probe_wait": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "moe_nf4_dequant": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "moe_nf4_tile16": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "moe_nf4_dequant_tile16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                       c_void_p]),
    "moe_nf4_nested_absmax": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_int64, c_int,
                                      c_void_p, c_void_p]),
    "moe_router_topk": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p,
                                c_void_p, c_void_p, c_void_p]),
    "moe_router_topk_from_logits": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p,
                                            c_void_p]),
    "moe_expert_workspace_size": (c_size_t, [c_int64, c_int, c_int]),
    "moe_expert_forward": (c_int, [ctypes.POINTER(NF4Expert), c_void_p, c_int64, c_int, c_int,
                                   c_void_p, c_void_p, c_size_t, c_void_p]),
    "moe_layer_forward_noalloc": (c_int, [c_void_p, c_void_p, ctypes.POINTER(NF4Expert), c_int,
                                          c_int, c_int64, c_int, c_int, c_void_p, c_void_p,
                                          c_void_p, c_void_p]),
    "moe_experts_workspace_size": (c_size_t, [c_int64, c_int, c_int]),
    "moe_experts_forward": (c_int, [ctypes.POINTER(NF4Expert), c_int, c_void_p, c_void_p, c_int64,
                                    c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "moe_layer_workspace_size": (c_size_t, [c_int64, c_int, c_int, c_int, c_int]),
    "moe_layer_forward": (c_int, [c_void_p, c_void_p, ctypes.POINTER(NF4Expert), c_int, c_int,
                                  c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_size_t, c_void_p]),
    "moe_permute": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p,
                            c_void_p, c_void_p, c_void_p]),
    "moe_gather_rows": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "moe_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                            c_void_p, c_void_p]),
    "moe_ep_dispatch": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "moe_ep_receive": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                               c_void_p]),
    "moe_ep_return": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "moe_ep_dispatch_p2p": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                    c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_void_p]),
    "moe_ep_return_p2p": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    "moe_ep_wait_p2p": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "moe_ep_receive_p2p": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_void_p]),
    "moe_combine_p2p": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "moe_ep_front_p2p": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int,
                                 c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "moe_ep_return_partials_p2p": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                           c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                           c_void_p]),
    "moe_expert_splits": (c_int, [c_int]),
    "moe_experts_counter_words": (c_int, [c_int]),
    "moe_experts_forward_partials": (c_int, [ctypes.POINTER(NF4Expert), c_int, c_void_p, c_void_p,
                                             c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                             c_size_t, c_void_p]),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("MOE_B200_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"moeinfra_b200 CUDA library not found at {path}; build it with "
            "`python -m moeinfra_b200.build` (nvcc, sm_100a). There is no CPU fallback.")
    try:
        handle = ctypes.CDLL(str(path))
    except OSError as exc:
        raise RuntimeError(f"failed to load moeinfra_b200 CUDA library {path}: {exc}") from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    _lib = handle
    return handle


def status_string(status: int) -> str:
    return lib().moe_status_string(int(status)).decode()


def launch_count() -> int:
    """Kernels launched (or captured) by the library so far in this process."""
    return int(lib().moe_launch_count())


def take_device_error() -> int:
    """Read and clear the device error words (bit 1: a bounded kernel wait timed
    out; bit 2: experts of one launch carried different codebooks)."""
    v = c_int(0)
    check(lib().moe_take_device_error(ctypes.byref(v)), "moe_take_device_error")
    return v.value


def stream_check(stream: int | None) -> int:
    """Synchronise ``stream`` and return the status of the launches since the last check."""
    return int(lib().moe_stream_check(c_void_p(stream)))


def set_wait_limit_ns(ns: int) -> None:
    """Limit of every bounded device wait (nanoseconds of the GPU's global timer)."""
    check(lib().moe_set_wait_limit_ns(int(ns)), "moe_set_wait_limit_ns")


def wait_limit_ns() -> int:
    return int(lib().moe_wait_limit_ns())


def check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"{what} failed: {status_string(status)} (status {status})")
