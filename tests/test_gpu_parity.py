"""GPU parity of the CUDA kernels against the oracle and the reference's golden
vectors.  Bit-exact for dequant, routing indices (on identical logits) and the
combine; expert and layer outputs within the stated fp16 tolerance
(rel-L2 <= 2e-3, max-abs <= 1e-2 x max(1, |ref|))."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import nf4 as onf4
from oracle import router as orouter
from tests.golden.inputs import (
    DISPATCH_CASES, ROUTER_CASES, dispatch_inputs, fake_expert_scale, router_inputs,
)
from tests.helpers import assert_close_fp16, gpu_expert, make_experts

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


# ---------------------------------------------------------------------------
# NF4 dequant (bit-exact)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("numel,offset", [(64, 0), (4096 * 256, 0), (96, 0), (100, 0), (4096, 1)])
def test_nf4_dequant_bit_exact(numel, offset):
    from moeinfra_b200 import kernels

    rng = np.random.default_rng(numel + offset)
    q = rng.integers(0, 256, size=numel // 2 + offset + 16, dtype=np.uint8)
    nb = (numel + 63) // 64
    absmax = (rng.standard_normal(nb).astype(np.float32) * np.float32(0.05))
    absmax[: min(4, nb)] = np.array([0.0, 1e-30, 3.0e4, 7.5e-3], np.float32)[: min(4, nb)]
    code = onf4.nf4_codebook()
    qt = _t(q)[offset:offset + numel // 2]  # offset 1 -> unaligned -> scalar path
    out = kernels.nf4_dequant(qt, _t(absmax), _t(code), numel)
    want = onf4.dequant_nf4_bf16(q[offset:offset + numel // 2], absmax, code, numel)
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("rows,cols", [(16, 64), (48, 256), (14336 // 64, 4096)])
def test_tile16_layout_and_tiled_dequant_bit_exact(rows, cols):
    from moeinfra_b200 import kernels

    rng = np.random.default_rng(rows * 7 + cols)
    q = rng.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
    absmax = rng.standard_normal(rows * cols // 64).astype(np.float32)
    qt, at = kernels.nf4_tile16(_t(q), _t(absmax), rows, cols)
    wq, wa = onf4.tile16(q, absmax, rows, cols)
    assert np.array_equal(qt.cpu().numpy(), wq)
    assert np.array_equal(at.cpu().numpy().view(np.uint32), wa.view(np.uint32))
    code = onf4.nf4_codebook()
    deq = kernels.nf4_dequant_tile16(qt, at, _t(code), rows, cols)
    want = onf4.dequant_nf4_bf16(q, absmax, code, rows * cols).reshape(rows, cols)
    assert np.array_equal(deq.view(torch.int16).cpu().numpy().view(np.uint16), want)


def test_nested_absmax_bit_exact():
    from moeinfra_b200 import kernels

    rng = np.random.default_rng(3)
    absmax = np.abs(rng.standard_normal(5000).astype(np.float32)) * np.float32(0.05)
    qa, a2, c2, off = onf4.quantize_absmax_nested(absmax)
    got = kernels.nested_absmax(_t(qa), _t(a2), _t(c2), float(off)).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), onf4.nested_absmax(qa, a2, c2, off).view(np.uint32))


# ---------------------------------------------------------------------------
# Router
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", sorted(ROUTER_CASES))
def test_router_matches_oracle_and_reference(golden, name):
    from moeinfra_b200 import kernels

    case = ROUTER_CASES[name]
    h, wg = router_inputs(case)
    k = case["k"]
    lg, w, idx = kernels.router_topk(_t(h), _t(wg), k)
    lg_np = lg.cpu().numpy()
    # logits: exact products accumulated in fp64, one rounding -> the
    # correctly rounded dot product, bit-exact with the oracle.
    want_lg = orouter.logits_f16(h, wg)
    assert np.array_equal(lg_np.view(np.uint16), want_lg.view(np.uint16))
    # full routing bit-exact with the oracle (same tie convention)
    ow, oi = orouter.route_from_logits(want_lg, k)
    assert np.array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=1e-6, atol=0)
    # Reference semantics on our logits, computed by torch on the GPU (the
    # reference router's own ops): bit-exact indices, and bit-exact weights
    # for k <= 2.
    p = torch.softmax(lg.float(), dim=-1)
    tw, ti = torch.topk(p, k, dim=-1)
    tw = tw / tw.sum(dim=-1, keepdim=True)
    assert torch.equal(ti, idx)
    same = torch.ones(idx.shape[0], dtype=torch.bool, device=idx.device)
    if k <= 2:
        assert torch.equal(w[same], tw[same])
    else:  # torch's k-element sum order is not reproduced for k > 2
        torch.testing.assert_close(w[same], tw[same], rtol=1e-6, atol=0)
    # Golden: on the reference's own logits, indices bit-exact except ties.
    gw, gi = kernels.router_topk_from_logits(_t(golden[f"router/{name}/logits"]), k)
    ref_i = golden[f"router/{name}/indices"]
    ref_p = orouter.softmax_f32(golden[f"router/{name}/logits"])
    gi_np = gi.cpu().numpy()
    for t in np.where((gi_np != ref_i).any(-1))[0]:
        assert np.array_equal(np.sort(ref_p[t][gi_np[t]]), np.sort(ref_p[t][ref_i[t]]))
    ok = (gi_np == ref_i).all(-1)
    np.testing.assert_allclose(gw.cpu().numpy()[ok], golden[f"router/{name}/weights"][ok], rtol=1e-6)


def test_router_tie_order_matches_torch_cuda_topk():
    from moeinfra_b200 import kernels

    lg = np.array([[0.5, 1.0, 1.0, 0.0, 0.0, 0.0, 0.0, 0.0],
                   [1.0, 1.0, 1.0, 0.0, 0.0, 0.0, 0.0, 0.0],
                   [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 2.0, 2.0],
                   [3.0, 1.0, 3.0, 1.0, 0.0, 0.0, 1.0, 0.0]], np.float16)
    for k in (1, 2, 3):
        w, idx = kernels.router_topk_from_logits(_t(lg), k)
        torch_i = torch.topk(torch.softmax(_t(lg).float(), -1), k, dim=-1).indices
        assert torch.equal(idx, torch_i), (k, idx.tolist(), torch_i.tolist())
        assert np.array_equal(idx.cpu().numpy(), orouter.route_from_logits(lg, k)[1])


# ---------------------------------------------------------------------------
# Permute + combine (bit-exact vs the reference's _forward_tokens)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", sorted(DISPATCH_CASES))
def test_permute_and_combine_bit_exact(golden, name):
    from moeinfra_b200 import kernels

    case = DISPATCH_CASES[name]
    h, _ = dispatch_inputs(case)
    idx = _t(golden[f"dispatch/{name}/indices"])
    w = _t(golden[f"dispatch/{name}/weights"])
    E = case["E"]
    off, ptok, pw, pslot = kernels.permute(idx, w, E)
    idx_np = golden[f"dispatch/{name}/indices"]
    counts = np.bincount(idx_np.reshape(-1), minlength=E)
    assert off.cpu().tolist() == [0] + np.cumsum(counts).tolist()
    ptok_np = ptok.cpu().numpy()
    o = off.cpu().numpy()
    for e in range(E):
        assert ptok_np[o[e]:o[e + 1]].tolist() == np.where((idx_np == e).any(-1))[0].tolist()
    ht = _t(h)
    x_sorted = kernels.gather_rows(ht, ptok)
    scale = torch.tensor([fake_expert_scale(e) for e in range(E)], device=DEV)
    expert_of_slot = torch.repeat_interleave(torch.arange(E, device=DEV),
                                             torch.from_numpy(counts).to(DEV))
    y_sorted = (x_sorted.float() * scale[expert_of_slot][:, None]).half()
    out = kernels.combine(y_sorted, pslot, idx, w)
    ref = golden[f"dispatch/{name}/output"]
    assert np.array_equal(out.cpu().numpy().view(np.uint16), ref.view(np.uint16))


# ---------------------------------------------------------------------------
# Experts
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("n", [1, 2, 3, 4])
def test_expert_forward_small(n):
    H, I = 256, 512
    ex = make_experts(21, 1, H, I, std=0.05)[0]
    x = (np.random.default_rng(n).standard_normal((n, H), dtype=np.float32)).astype(np.float16)
    y = gpu_expert(ex, H, I)(_t(x)).cpu().numpy()
    assert_close_fp16(y, onf4.expert_forward(x, ex, H, I), what=f"expert n={n}")


def test_expert_forward_nested_absmax():
    H, I = 128, 256
    ex = make_experts(22, 1, H, I, std=0.05, nested=True)[0]
    x = (np.random.default_rng(0).standard_normal((3, H), dtype=np.float32)).astype(np.float16)
    y = gpu_expert(ex, H, I)(_t(x)).cpu().numpy()
    assert_close_fp16(y, onf4.expert_forward(x, ex, H, I), what="nested")


@pytest.mark.parametrize("n", [1, 4])
def test_expert_forward_mixtral_shape(n):
    H, I = 4096, 14336
    ex = make_experts(0, 1, H, I)[0]
    x = np.random.default_rng(100 + n).standard_normal((n, H), dtype=np.float32).astype(np.float16)
    y = gpu_expert(ex, H, I)(_t(x)).cpu().numpy()
    r, m = assert_close_fp16(y, onf4.expert_forward(x, ex, H, I), what=f"mixtral n={n}")
    print(f"mixtral expert n={n}: rel_l2={r:.2e} max_abs={m:.2e}")


@pytest.mark.parametrize("H,I", [(2048, 2048), (2048, 4096), (4096, 2048)])
def test_expert_forward_chunk_aligned_shapes(H, I):
    """1-token experts at other sizes whose K extents are whole 2048-element chunks."""
    from moeinfra_b200 import _native

    ex = make_experts(40 + H // 1024 + I // 512, 1, H, I, std=0.03)[0]
    x = np.random.default_rng(H + I).standard_normal((1, H), dtype=np.float32).astype(np.float16)
    for _ in range(2):
        y = gpu_expert(ex, H, I)(_t(x)).cpu().numpy()
        assert_close_fp16(y, onf4.expert_forward(x, ex, H, I), what=f"expert H={H} I={I}")
    assert _native.take_device_error() == 0


# Experts with more than 8 tokens run the tcgen05 grouped GEMM.
@pytest.mark.parametrize("n", [9, 16, 100, 300])
def test_expert_forward_gemm_small(n):
    from moeinfra_b200 import _native

    H, I = 256, 512
    ex = make_experts(50 + n, 1, H, I, std=0.05)[0]
    x = (np.random.default_rng(n).standard_normal((n, H), dtype=np.float32)).astype(np.float16)
    g = gpu_expert(ex, H, I)
    for _ in range(2):
        y = g(_t(x)).cpu().numpy()
        assert_close_fp16(y, onf4.expert_forward(x, ex, H, I), what=f"gemm expert n={n}")
    assert _native.take_device_error() == 0


@pytest.mark.parametrize("n", [16, 300])
def test_expert_forward_gemm_mixtral_shape(n):
    from moeinfra_b200 import _native

    H, I = 4096, 14336
    ex = make_experts(3, 1, H, I)[0]
    x = np.random.default_rng(200 + n).standard_normal((n, H), dtype=np.float32).astype(np.float16)
    y = gpu_expert(ex, H, I)(_t(x)).cpu().numpy()
    r, m = assert_close_fp16(y, onf4.expert_forward(x, ex, H, I), what=f"gemm mixtral n={n}")
    print(f"gemm mixtral expert n={n}: rel_l2={r:.2e} max_abs={m:.2e}")
    assert _native.take_device_error() == 0


# A single expert with few row tiles splits K into chunks (fp32 partials summed
# in order by a second kernel): equal chunks (H 1024 / I 2048: gate 2 chunks,
# down 4) and a ragged last chunk (H 1664: 26 K blocks in chunks of 9, 9, 8).
@pytest.mark.parametrize("H,I,n", [(1024, 2048, 16), (1664, 256, 16), (1024, 2048, 32)])
def test_expert_forward_gemm_split_k(H, I, n):
    from moeinfra_b200 import _native

    ex = make_experts(70 + n, 1, H, I, std=0.05)[0]
    x = np.random.default_rng(H + n).standard_normal((n, H), dtype=np.float32).astype(np.float16)
    g = gpu_expert(ex, H, I)
    for _ in range(2):
        y = g(_t(x)).cpu().numpy()
        assert_close_fp16(y, onf4.expert_forward(x, ex, H, I), what=f"split-K expert H={H} I={I}")
    assert _native.take_device_error() == 0


# ---------------------------------------------------------------------------
# Fused layer
# ---------------------------------------------------------------------------

def _layer_case(T, H, I, E=8, k=2, seed=7, gate_std=0.05):
    rng = np.random.default_rng(seed)
    wg = (rng.standard_normal((E, H), dtype=np.float32) * np.float32(gate_std)).astype(np.float16)
    h = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    experts = make_experts(seed + 1, E, H, I, std=0.05)
    return h, wg, experts


@pytest.mark.parametrize("T", [1, 2, 3, 4])
def test_layer_forward_small(T):
    from moeinfra_b200 import kernels

    H, I, E, k = 256, 512, 8, 2
    h, wg, experts = _layer_case(T, H, I, E, k, seed=30 + T)
    gx = [gpu_expert(ex, H, I) for ex in experts]
    table = kernels.expert_array([g.nf4_descriptor for g in gx])
    out, idx, w = kernels.layer_forward(_t(h), _t(wg), table, k, H, I)
    ref, ridx, rw, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert_close_fp16(out.cpu().numpy(), ref, what=f"layer T={T}")


@pytest.mark.parametrize("T", [1, 2, 5])
def test_layer_forward_chunk_aligned_mixed(T):
    """Chunk-aligned shapes: 1-token experts on the GEMV kernels, 2..8-token
    experts on the multi-token kernels, in one layer."""
    from moeinfra_b200 import _native, kernels

    H, I, E, k = 2048, 4096, 4, 2
    h, wg, experts = _layer_case(T, H, I, E, k, seed=60 + T, gate_std=0.05)
    gx = [gpu_expert(ex, H, I) for ex in experts]
    table = kernels.expert_array([g.nf4_descriptor for g in gx])
    out, idx, w = kernels.layer_forward(_t(h), _t(wg), table, k, H, I)
    ref, ridx, rw, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert_close_fp16(out.cpu().numpy(), ref, what=f"layer 2048x4096 T={T}")
    assert _native.take_device_error() == 0


@pytest.mark.parametrize("T", [9, 64, 700])
def test_layer_forward_gemm(T):
    """Layers past 8 tokens: gather, tcgen05 grouped GEMM, ordered combine."""
    from moeinfra_b200 import _native, kernels

    H, I, E, k = 256, 512, 8, 2
    h, wg, experts = _layer_case(T, H, I, E, k, seed=80 + T)
    gx = [gpu_expert(ex, H, I) for ex in experts]
    table = kernels.expert_array([g.nf4_descriptor for g in gx])
    out, idx, w = kernels.layer_forward(_t(h), _t(wg), table, k, H, I)
    ref, ridx, rw, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert_close_fp16(out.cpu().numpy(), ref, what=f"gemm layer T={T}")
    assert _native.take_device_error() == 0


def test_layer_forward_mixtral_bs1():
    from moeinfra_b200 import kernels

    H, I, E, k = 4096, 14336, 8, 2
    rng = np.random.default_rng(1)
    wg = (rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    h = rng.standard_normal((1, H), dtype=np.float32).astype(np.float16)
    # Only routed experts are read by the kernels; build just those at full size.
    _, _, ridx0 = orouter.route_with_logits(h, wg, k)
    routed = sorted(set(ridx0.reshape(-1).tolist()))
    experts = {e: make_experts(100 + e, 1, H, I)[0] for e in routed}
    gx = {e: gpu_expert(experts[e], H, I) for e in routed}
    table = kernels.expert_array([gx.get(e, gx[routed[0]]).nf4_descriptor for e in range(E)])
    out, idx, w = kernels.layer_forward(_t(h), _t(wg), table, k, H, I)
    ref, ridx, rw, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    r, m = assert_close_fp16(out.cpu().numpy(), ref, what="mixtral layer bs1")
    print(f"mixtral layer bs1: rel_l2={r:.2e} max_abs={m:.2e}")


# ---------------------------------------------------------------------------
# One-token layer in one launch (routing, experts and combine in one kernel)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("E,k,H,I", [
    (16, 2, 256, 512),    # the largest expert count
    (5, 1, 256, 512),     # k = 1
    (8, 8, 256, 512),     # every expert routed
    (4, 2, 2048, 5632),   # last down split partial (5632 = 2 x 2048 + 1536)
    (8, 2, 1024, 2048),   # one 64-element block per warp in gate_up
    (2, 2, 8192, 1024),   # eight blocks per warp; two row vectors per routing thread
])
def test_layer_forward_one_token_fused(E, k, H, I):
    """The fused 1-token layer against the oracle, and its routing against the
    standalone router kernel (same fp16 logits, softmax and top-k)."""
    from moeinfra_b200 import _native, kernels

    h, wg, experts = _layer_case(1, H, I, E, k, seed=11 * E + k + H // 256)
    gx = [gpu_expert(ex, H, I) for ex in experts]
    table = kernels.expert_array([g.nf4_descriptor for g in gx])
    out, idx, w = kernels.layer_forward(_t(h), _t(wg), table, k, H, I)
    ref, ridx, rw, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    _, rw_k, ridx_k = kernels.router_topk(_t(h), _t(wg), k, with_logits=False)
    assert torch.equal(idx, ridx_k)
    np.testing.assert_allclose(w.cpu().numpy(), rw_k.cpu().numpy(), rtol=1e-6, atol=0)
    assert_close_fp16(out.cpu().numpy(), ref, what=f"fused 1-token layer E={E} k={k} {H}x{I}")
    assert _native.take_device_error() == 0


def test_layer_forward_one_token_repeated_calls():
    """Back-to-back calls reuse the wrapper's workspace (its counters are
    zeroed by the layer itself each call); every result matches the oracle."""
    from moeinfra_b200 import _native, kernels

    H, I, E, k = 256, 512, 8, 2
    _, wg, experts = _layer_case(1, H, I, E, k, seed=91)
    gx = [gpu_expert(ex, H, I) for ex in experts]
    table = kernels.expert_array([g.nf4_descriptor for g in gx])
    rng = np.random.default_rng(92)
    for call in range(3):
        h = rng.standard_normal((1, H), dtype=np.float32).astype(np.float16)
        out, _, _ = kernels.layer_forward(_t(h), _t(wg), table, k, H, I, routing=False)
        ref, _, _, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
        assert_close_fp16(out.cpu().numpy(), ref, what=f"repeated 1-token call {call}")
    assert _native.take_device_error() == 0


def test_layer_forward_gemm_narrow_multitile():
    """Narrow grouped-GEMM tiles (<= 64 tokens per expert on average) with one
    expert past 64 tokens, so it spans two token tiles."""
    from moeinfra_b200 import _native, kernels

    T, H, I, E, k = 120, 256, 512, 2, 1
    h, wg, experts = _layer_case(T, H, I, E, k, seed=127, gate_std=0.3)
    _, _, ridx0 = orouter.route_with_logits(h, wg, k)
    assert np.bincount(ridx0.reshape(-1), minlength=E).max() > 64
    gx = [gpu_expert(ex, H, I) for ex in experts]
    table = kernels.expert_array([g.nf4_descriptor for g in gx])
    out, idx, w = kernels.layer_forward(_t(h), _t(wg), table, k, H, I)
    ref, ridx, rw, _ = omoe.moe_layer_forward(h, wg, experts, H, I, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert_close_fp16(out.cpu().numpy(), ref, what="narrow multi-tile layer")
    assert _native.take_device_error() == 0
