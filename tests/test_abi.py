"""CPU: the C-ABI library loads and exports every entry point of include/*.h.

No kernel is launched here; calls below only exercise host-side argument
validation, which returns before any CUDA work is enqueued.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from moeinfra_b200 import _native

ROOT = Path(__file__).resolve().parent.parent


def _declared_functions() -> set[str]:
    names = set()
    for hdr in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", hdr.read_text(), flags=re.S)
        for m in re.finditer(r"\b(moe_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_loads():
    lib = _native.lib()
    assert lib.moe_version().decode().startswith("moe_b200")


def test_every_declared_symbol_is_exported_and_bound():
    lib = _native.lib()
    declared = _declared_functions()
    assert {"moe_nf4_dequant", "moe_router_topk", "moe_layer_forward", "moe_expert_forward"} <= declared
    for name in declared:
        assert hasattr(lib, name), f"{name} missing from libmoe_b200.so"
    assert declared <= set(_native.SIGNATURES), "ctypes signatures out of date with the header"


def test_status_strings():
    for code in range(8):
        assert _native.status_string(code) != "unknown status"
    assert _native.status_string(99) == "unknown status"


def test_workspace_sizes_grow_with_tokens():
    lib = _native.lib()
    a = lib.moe_layer_workspace_size(1, 4096, 14336, 8, 2)
    b = lib.moe_layer_workspace_size(64, 4096, 14336, 8, 2)
    c = lib.moe_layer_workspace_size(4096, 4096, 14336, 8, 2)
    assert 0 < a < b < c
    assert lib.moe_expert_workspace_size(16, 4096, 14336) > lib.moe_expert_workspace_size(1, 4096, 14336)


def test_host_validation_rejects_bad_arguments_without_launching():
    lib = _native.lib()
    # odd numel / bad blocksize / null pointers -> invalid argument
    assert lib.moe_nf4_dequant(None, None, None, 3, 64, None, None) == 1
    assert lib.moe_nf4_dequant(None, None, None, 64, 48, None, None) == 1
    assert lib.moe_router_topk(None, None, 4, 4096, 33, 2, None, None, None, None) == 1
    assert lib.moe_router_topk(None, None, 4, 4096, 8, 9, None, None, None, None) == 1
    # unsupported shapes
    desc = _native.NF4Expert()
    assert lib.moe_expert_forward(ctypes.byref(desc), None, 1, 100, 14336, None, None, 0, None) == 2
    # zero-size work is a no-op success
    assert lib.moe_nf4_dequant(None, None, None, 0, 64, None, None) == 0
    assert lib.moe_router_topk(None, None, 0, 4096, 8, 2, None, None, None, None) == 0


def test_unaligned_workspace_is_rejected_before_any_launch():
    """Workspace entry points return MOE_ERR_ALIGNMENT for a workspace that is
    not 16-byte aligned (the split-K partials are read as 16-byte vectors);
    the pointers below are never dereferenced: the check precedes every launch."""
    lib = _native.lib()
    fake = 0x100000
    m = _native.NF4Matrix(fake, fake, fake)
    desc = _native.NF4Expert(m, m, m)
    need = lib.moe_expert_workspace_size(16, 4096, 14336)
    st = lib.moe_expert_forward(ctypes.byref(desc), ctypes.c_void_p(fake), 16, 4096, 14336,
                                ctypes.c_void_p(fake), ctypes.c_void_p(fake + 8), need, None)
    assert st == 5  # MOE_ERR_ALIGNMENT
    # too small a workspace is reported first
    st = lib.moe_expert_forward(ctypes.byref(desc), ctypes.c_void_p(fake), 16, 4096, 14336,
                                ctypes.c_void_p(fake), ctypes.c_void_p(fake), need - 1, None)
    assert st == 4  # MOE_ERR_WORKSPACE


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setenv("MOE_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _native.lib()
    monkeypatch.delenv("MOE_B200_LIB")
    monkeypatch.setattr(_native, "_lib", None)
    _native.lib()


def test_wrappers_make_their_tensors_device_current(monkeypatch):
    """A call on another GPU's data runs with that GPU current (the library launches on the
    current device); a call on the current GPU's data switches nothing.  Checked on the host
    with the current device and the switch faked (no GPU needed)."""
    import contextlib

    import torch

    from moeinfra_b200 import kernels

    switched = []

    @contextlib.contextmanager
    def fake_device(d):
        switched.append(d)
        yield

    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "device", fake_device)

    @kernels._on_device
    def launch(n: int, device=None):
        return n

    assert launch(3, device=torch.device("cuda", 1)) == 3
    assert switched == [1]
    assert launch(4, device=torch.device("cuda", 0)) == 4
    assert launch(5) == 5  # nothing on a GPU: no switch
    assert switched == [1]


def test_fused_exchange_entries_check_arguments_before_any_launch():
    """The fused expert-parallel entry points refuse bad calls on the host (no pointer below is
    dereferenced: every check precedes the launch)."""
    lib = _native.lib()
    f = ctypes.c_void_p(0x100000)  # 16-byte aligned, never read

    def front(T, E, k, G, rank, cap, hidden=4096, n_zero=0):
        return lib.moe_ep_front_p2p(f, f, T, E, k, G, rank, cap, hidden, f, f, f, f, f, f, f, f,
                                    f, n_zero, None)

    assert front(1, 8, 9, 8, 0, 1) == 1        # k > 8
    assert front(1, 8, 2, 8, 8, 1) == 1        # rank outside [0, G)
    assert front(2, 8, 2, 8, 0, 1) == 1        # T * min(k, E/G) rows exceed cap
    assert front(1, 8, 2, 3, 0, 2) == 1        # E not a multiple of G
    assert front(1, 8, 2, 8, 0, 1, n_zero=-1) == 1
    assert front(149, 8, 2, 8, 0, 149) == 2    # more tokens than SMs: CTAs not all resident
    assert lib.moe_ep_front_p2p(None, None, 1, 8, 2, 8, 0, 1, 4096, f, f, f, f, None, f, f, f,
                                None, 0, None) == 1  # no barrier words
    # partials: decode-sized calls only; the return needs S >= 1
    desc = (_native.NF4Expert * 1)()
    assert lib.moe_experts_forward_partials(desc, 1, f, f, 9, 4096, 14336, f, None, f, 1 << 30,
                                            None) == 2
    assert lib.moe_ep_return_partials_p2p(f, 0, f, 8, 8, 0, 1, 4096, f, f, f, f, None) == 1
    assert lib.moe_expert_splits(14336) == 7 and lib.moe_expert_splits(100) == -1
    assert lib.moe_experts_counter_words(14336) == 2 * 16 * 7
