"""moe_layer_forward_noalloc (static device scratch) against moe_layer_forward.

Kept in its own file, named to be collected last, so it runs both alone and
after every other test in the process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from moeinfra_b200 import _native


def _random_layer(H: int, I: int, E: int, seed: int, device: str = "cuda:0"):
    """Random packed NF4 experts (tile16) and an fp16 gate on ``device``; tensors kept alive."""
    from moeinfra_b200 import kernels
    from moeinfra_b200._native import NF4Expert
    from moeinfra_b200.model.nf4_format import nf4_code_tensor

    g = torch.Generator(device=device).manual_seed(seed)
    code = nf4_code_tensor(device)
    keep, descs = [code], []
    for _ in range(E):
        mats = []
        for rows, cols in ((I, H), (I, H), (H, I)):
            q = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device=device,
                              generator=g)
            a = torch.rand(rows * cols // 64, device=device, generator=g) * 0.05 + 0.01
            qt, at = kernels.nf4_tile16(q, a, rows, cols)
            keep += [qt, at]
            mats.append(kernels.matrix_desc(qt, at, code))
        descs.append(NF4Expert(mats[0], mats[1], mats[2]))
    gate = (torch.randn(E, H, device=device, generator=g) * 0.05).half()
    return kernels.expert_array(descs), gate, keep


@pytest.mark.gpu
@pytest.mark.parametrize("H,I,T", [(256, 512, 1), (256, 512, 4), (4096, 14336, 1), (4096, 14336, 8)])
def test_noalloc_equals_layer_forward_two_calls(H, I, T):
    from moeinfra_b200 import kernels

    E, k = 8, 2
    table, gate, _keep = _random_layer(H, I, E, seed=H + T)
    g = torch.Generator(device="cuda").manual_seed(T)
    hs = [torch.randn(T, H, device="cuda", generator=g).half() for _ in range(2)]
    got = [kernels.layer_forward_noalloc(h, gate, table, k, H, I) for h in hs]  # two in a row
    want = [kernels.layer_forward(h, gate, table, k, H, I) for h in hs]
    torch.cuda.synchronize()
    for (o, i, w), (o2, i2, w2) in zip(got, want):
        assert torch.equal(i, i2)
        assert torch.equal(w, w2)
        assert torch.equal(o.view(torch.int16), o2.view(torch.int16))
    assert not torch.equal(got[0][0], got[1][0])
    # No bounded wait ran out and no codebook mismatch was flagged on either path.
    assert _native.take_device_error() == 0


@pytest.mark.gpu
def test_noalloc_on_a_second_gpu():
    """Kernel attributes, SM count and the scratch address are kept per device."""
    from moeinfra_b200 import kernels

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    H, I, E, k, T = 4096, 14336, 8, 2, 1
    table, gate, _keep = _random_layer(H, I, E, seed=7, device="cuda:1")
    h = torch.randn(T, H, device="cuda:1").half()
    o1, i1, w1 = kernels.layer_forward_noalloc(h, gate, table, k, H, I)
    with torch.cuda.device(1):
        o2, i2, w2 = kernels.layer_forward(h, gate, table, k, H, I)
        torch.cuda.synchronize()
        assert _native.take_device_error() == 0
    assert torch.equal(i1, i2)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))


def test_noalloc_rejects_oversize_without_touching_the_gpu():
    lib = _native.lib()
    H, I, E, k, T = 4096, 14336, 16, 8, 8
    need = lib.moe_layer_workspace_size(T, H, I, E, k)
    assert need > _native.MOE_NOALLOC_SCRATCH_BYTES
    experts = (_native.NF4Expert * E)()
    st = lib.moe_layer_forward_noalloc(None, None, experts, E, k, T, H, I, None, None, None, None)
    assert st == 4  # MOE_ERR_WORKSPACE, before any CUDA call
    # Mixtral decode at bs8 / top-2 fits.
    assert lib.moe_layer_workspace_size(8, H, I, 8, 2) <= _native.MOE_NOALLOC_SCRATCH_BYTES


def test_noalloc_checks_arguments_before_the_size():
    """Bad E / k / shapes report INVALID_ARG / UNSUPPORTED, not a size error; T == 0 is a no-op."""
    lib = _native.lib()
    experts = (_native.NF4Expert * 16)()
    assert lib.moe_layer_forward_noalloc(None, None, experts, 17, 2, 8, 4096, 14336, None, None,
                                         None, None) == 1
    assert lib.moe_layer_forward_noalloc(None, None, experts, 8, 9, 8, 4096, 14336, None, None,
                                         None, None) == 1
    assert lib.moe_layer_forward_noalloc(None, None, experts, 4, 5, 8, 4096, 14336, None, None,
                                         None, None) == 1
    assert lib.moe_layer_forward_noalloc(None, None, experts, 8, 2, 8, 4100, 14336, None, None,
                                         None, None) == 2
    assert lib.moe_layer_forward_noalloc(None, None, experts, 8, 2, 0, 4096, 14336, None, None,
                                         None, None) == 0
