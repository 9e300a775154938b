"""Layer parity at the Mixtral shape for the workloads the bench reports.

* config 1 at 64 tokens (hidden 4096, ffn 14336, 8 experts, top-2; gate
  N(0, 0.02), tokens N(0, 1), seed 1): every output row against the oracle;
* config 2 prefill (4096 tokens, gate N(0, 0.05), seed 2, uneven expert loads):
  a sample of output rows that covers, for every expert, its first and last
  token and the tokens on both sides of each 64- and 256-token tile edge of
  its token list, plus random tokens.  Each sampled row is recomputed by the
  oracle exactly (a row of the reference's multi-row fp16 GEMM depends only on
  its own input row), so sampling keeps the numpy oracle cheap.

Routing indices are bit-exact against the oracle; outputs meet the layer
tolerance (rel-L2 <= 2e-3, max-abs <= 1e-2 x max(1, |ref|)).  Experts are
quantized on the device by the package's quantizer, which the CPU suite
checks bit-for-bit against the oracle's quantizer.
"""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import nf4 as onf4
from oracle import router as orouter
from tests.helpers import assert_close_fp16

pytestmark = pytest.mark.gpu
H, I, E, K = 4096, 14336, 8, 2


def _experts(seed: int):
    """Device-quantized N(0, 0.02) experts: (ctypes table, oracle states, objects kept alive)."""
    from moeinfra_b200 import kernels
    from moeinfra_b200.model.nf4_format import quantize_nf4_packed
    from moeinfra_b200.transfer.nf4_reconstruct import ReconstructedNF4Expert

    shape = types.SimpleNamespace(hidden_size=H, intermediate_size=I)
    g = torch.Generator(device="cuda").manual_seed(seed)
    gpu, oracle_states = [], []
    for _ in range(E):
        st, ost = {}, {}
        for name, (rows, cols) in (("w1", (I, H)), ("w3", (I, H)), ("w2", (H, I))):
            w = (torch.randn(rows, cols, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            q, a, code = quantize_nf4_packed(w)
            st[name] = {"weight": q, "absmax": a, "code": code, "offset": None}
            ost[name] = {"weight": q.cpu().numpy(), "absmax": a.cpu().numpy(),
                         "code": code.cpu().numpy(), "offset": None}
        gpu.append(ReconstructedNF4Expert(shape, st))
        oracle_states.append(ost)
    table = kernels.expert_array([x.nf4_descriptor for x in gpu])
    return table, oracle_states, gpu


def _expert_rows_multirow(x16: np.ndarray, ex: dict) -> np.ndarray:
    """The expert on rows of a multi-token call (bitsandbytes' dequant + fp16 GEMM path)."""
    g = onf4.linear_multirow(x16, onf4.dequant_weight_f16(ex["w1"], (I, H)))
    u = onf4.linear_multirow(x16, onf4.dequant_weight_f16(ex["w3"], (I, H)))
    hmid = onf4.swiglu_f16(g, u)
    return onf4.linear_multirow(hmid, onf4.dequant_weight_f16(ex["w2"], (H, I)))


def test_config1_bs64_every_row():
    from moeinfra_b200 import kernels

    table, ox, _keep = _experts(seed=1)
    g = torch.Generator(device="cuda").manual_seed(1)
    gate = (torch.randn(E, H, generator=g, device="cuda") * 0.02).half()
    h = torch.randn(64, H, generator=g, device="cuda").half()
    out, idx, w = kernels.layer_forward(h, gate, table, K, H, I)
    kernels.check_device()
    hn, wn = h.cpu().numpy(), gate.cpu().numpy()
    ref, ridx, rw, _ = omoe.moe_layer_forward(
        hn, wn, ox, H, I, K, expert_fn=lambda x, e: (_expert_rows_multirow(x, ox[e]) if x.shape[0] > 1
                                                      else onf4.expert_forward(x, ox[e], H, I)))
    assert np.array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=0)
    r, m = assert_close_fp16(out.cpu().numpy(), ref, what="config 1 bs64")
    print(f"config 1 bs64: rel_l2={r:.2e} max_abs={m:.2e}; tokens per expert "
          f"{np.bincount(ridx.reshape(-1), minlength=E).tolist()}")


def _sample_tokens(idx: np.ndarray, rng: np.random.Generator) -> np.ndarray:
    picks = set(rng.choice(idx.shape[0], size=16, replace=False).tolist())
    for e in range(E):
        toks = np.nonzero((idx == e).any(-1))[0]
        n = len(toks)
        for p in (0, n - 1, 63, 64, 127, 128, 255, 256, 511, 512, n - 2):
            if 0 <= p < n:
                picks.add(int(toks[p]))
    return np.array(sorted(picks))


def test_config2_prefill_sampled_rows():
    from moeinfra_b200 import kernels

    table, ox, _keep = _experts(seed=2)
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(4096, H, generator=g, device="cuda").half()
    gate = (torch.randn(E, H, generator=g, device="cuda") * 0.05).half()
    out, idx, w = kernels.layer_forward(x, gate, table, K, H, I)
    kernels.check_device()
    xn, wn = x.cpu().numpy(), gate.cpu().numpy()
    _, rw, ridx = orouter.route_with_logits(xn, wn, K)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    loads = np.bincount(ridx.reshape(-1), minlength=E)
    assert loads.min() > 256  # every expert spans several token tiles
    sample = _sample_tokens(ridx, np.random.default_rng(2))
    si, sw, sx = ridx[sample], rw[sample], xn[sample]
    expert_out = {}
    for e in range(E):
        rows = np.nonzero((si == e).any(-1))[0]
        if len(rows):
            expert_out[e] = _expert_rows_multirow(sx[rows], ox[e])
    ref = omoe.combine_expert_outputs(len(sample), H, si, sw, expert_out)
    got = out.cpu().numpy()[sample]
    r, m = assert_close_fp16(got, ref, what="config 2 prefill (sampled rows)")
    print(f"config 2 prefill: {len(sample)} sampled rows, rel_l2={r:.2e} max_abs={m:.2e}; "
          f"loads {loads.tolist()}")
