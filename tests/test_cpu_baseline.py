"""The timed CPU baseline (oracle.cpu_path, torch on host cores) agrees with the numpy oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cpu_path
from oracle import moe as omoe
from oracle import nf4 as onf4
from tests.helpers import assert_close_fp16


def _torch_expert(ex: dict) -> dict:
    return {n: {"q": torch.from_numpy(np.asarray(ex[n]["weight"], np.uint8)),
                "absmax": torch.from_numpy(np.asarray(ex[n]["absmax"], np.float32))}
            for n in ("w1", "w3", "w2")}


@pytest.mark.parametrize("T", [1, 3, 6])
def test_cpu_path_matches_oracle_layer(T):
    H, I, E, k = 128, 256, 4, 2
    rng = np.random.default_rng(11 + T)
    experts = [onf4.make_expert(rng, H, I) for _ in range(E)]
    h = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    wg = (rng.standard_normal((E, H), dtype=np.float32) * 0.05).astype(np.float16)
    ref, ridx, _, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
    code = torch.from_numpy(onf4.nf4_codebook())
    out, idx, _ = cpu_path.layer_forward(torch.from_numpy(h), torch.from_numpy(wg),
                                         [_torch_expert(ex) for ex in experts], code, H, I, k)
    assert np.array_equal(np.sort(idx.numpy(), -1), np.sort(ridx, -1))
    assert_close_fp16(out.numpy(), ref, what=f"cpu_path T={T}")


def test_cpu_dequant_gemv_and_multirow_weights():
    rng = np.random.default_rng(5)
    ex = onf4.make_expert(rng, 64, 128)["w1"]
    q = torch.from_numpy(np.asarray(ex["weight"], np.uint8))
    a = torch.from_numpy(np.asarray(ex["absmax"], np.float32))
    code = torch.from_numpy(onf4.nf4_codebook())
    w_gemv = cpu_path.dequant_store(q, a, code, 128, 64, gemv=True).numpy()
    assert np.array_equal(w_gemv.view(np.uint16),
                          onf4.gemv_weight_f16(ex, (128, 64)).reshape(128, 64).view(np.uint16))
    w_multi = cpu_path.dequant_store(q, a, code, 128, 64, gemv=False).numpy()
    assert np.array_equal(w_multi.view(np.uint16),
                          onf4.dequant_weight_f16(ex, (128, 64)).reshape(128, 64).view(np.uint16))
