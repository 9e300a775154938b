"""moe_layer_forward_noalloc (static device scratch) against moe_layer_forward.

Kept in its own file, named to be collected last, so it runs both alone and
after every other test in the process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from moeinfra_b200 import _native


def _random_layer(H: int, I: int, E: int, seed: int):
    """Random packed NF4 experts (tile16) and an fp16 gate on cuda:0; tensors kept alive."""
    from moeinfra_b200 import kernels
    from moeinfra_b200._native import NF4Expert
    from moeinfra_b200.model.nf4_format import nf4_code_tensor

    g = torch.Generator(device="cuda").manual_seed(seed)
    code = nf4_code_tensor("cuda")
    keep, descs = [code], []
    for _ in range(E):
        mats = []
        for rows, cols in ((I, H), (I, H), (H, I)):
            q = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda",
                              generator=g)
            a = torch.rand(rows * cols // 64, device="cuda", generator=g) * 0.05 + 0.01
            qt, at = kernels.nf4_tile16(q, a, rows, cols)
            keep += [qt, at]
            mats.append(kernels.matrix_desc(qt, at, code))
        descs.append(NF4Expert(mats[0], mats[1], mats[2]))
    gate = (torch.randn(E, H, device="cuda", generator=g) * 0.05).half()
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
