"""CPU: pin the oracle against published tables, known answers and the
reference's own golden vectors (tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import moe as omoe
from oracle import nf4 as onf4
from oracle import router as orouter
from tests.golden.inputs import (
    DISPATCH_CASES, ORACLE_LAYER_CASE, ROUTER_CASES, dispatch_inputs, fake_expert_scale,
    oracle_layer_inputs, router_inputs, sha256_arrays,
)


def test_codebook_construction_matches_published_nf4_table():
    code = onf4.nf4_codebook()
    assert code.dtype == np.float32 and code.shape == (16,)
    assert np.array_equal(code, np.asarray(onf4.PUBLISHED_NF4, np.float32))


def test_dynamic_map_shape_and_range():
    m = onf4.dynamic_map_signed()
    assert m.shape == (256,) and m.dtype == np.float32
    assert np.all(np.diff(m) > 0) and m.max() == 1.0 and m.min() > -1.0 and 0.0 in m


def test_product_store_codebooks_match_oracle_construction():
    import torch
    from moeinfra_b200.model.nf4_format import NF4_CODE, _dynamic_map_signed
    assert np.array_equal(np.asarray(NF4_CODE, np.float32), onf4.nf4_codebook())
    assert np.array_equal(_dynamic_map_signed().numpy(), onf4.dynamic_map_signed())


def test_nibble_order_high_nibble_is_even_element():
    q = np.array([0x0F, 0xF0, 0x7A], np.uint8)
    assert onf4.unpack_nf4(q).tolist() == [0, 15, 15, 0, 7, 10]
    assert np.array_equal(onf4.pack_nf4(onf4.unpack_nf4(q)), q)


def test_dequant_known_answers():
    code = np.asarray(onf4.PUBLISHED_NF4, np.float32)
    # byte 0x0F, absmax 2.0 -> [code[0]*2, code[15]*2] = [-2, 2] exactly.
    q = np.full(32, 0x77, np.uint8)  # code[7] == 0.0
    q[0] = 0x0F
    q[1] = 0x8E
    out = onf4.bf16_bits_to_f32(onf4.dequant_nf4_bf16(q, np.array([2.0], np.float32), code, 64))
    assert out[0] == -2.0 and out[1] == 2.0
    # code[8] * 2 = 0.15916059911251068 -> bf16 0.1591796875 (RNE of 0x3E22F8F4 -> 0x3E23)
    assert out[2] == np.float32(0.1591796875)
    # code[14] * 2 = 1.4459136724472046 -> bf16 1.4453125
    assert out[3] == np.float32(1.4453125)
    assert np.all(out[4:] == 0.0)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -8 + 2 ** -20, -0.0, np.inf],
                 np.float32)
    b = onf4.f32_to_bf16_bits(x)
    assert b.tolist() == [0x3F80, 0x3F82, 0x3F81, 0x8000, 0x7F80]
    assert np.isnan(onf4.bf16_bits_to_f32(onf4.f32_to_bf16_bits(np.array([np.nan], np.float32))))[0]


def test_nested_absmax_is_two_rounded_fp32_ops():
    qabs = np.array([0, 255, 128], np.uint8)
    a2 = np.array([0.5], np.float32)
    code2 = onf4.dynamic_map_signed()
    got = onf4.nested_absmax(qabs, a2, code2, np.float32(0.1))
    want = np.array([np.float32(np.float32(code2[q] * np.float32(0.5)) + np.float32(0.1)) for q in qabs],
                    np.float32)
    assert np.array_equal(got, want)


def test_quantizer_round_trip_error_bounded():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((64, 128), dtype=np.float32) * np.float32(0.02)
    q, absmax = onf4.quantize_nf4(w)
    deq = onf4.bf16_bits_to_f32(onf4.dequant_nf4_bf16(q, absmax, onf4.nf4_codebook(), w.size))
    err = np.abs(deq.reshape(w.shape) - w).max()
    assert err <= absmax.max() * 0.16  # half the widest NF4 gap, plus bf16 rounding


@pytest.mark.parametrize("name", sorted(ROUTER_CASES))
def test_router_oracle_matches_reference(golden, name):
    case = ROUTER_CASES[name]
    h, wg = router_inputs(case)
    assert bytes(golden[f"router/{name}/inputs_sha"]) == sha256_arrays(h, wg)
    ref_lg = golden[f"router/{name}/logits"]
    ref_w = golden[f"router/{name}/weights"]
    ref_i = golden[f"router/{name}/indices"]
    lg = orouter.logits_f16(h, wg)
    # fp16 logits: within one ulp plus the error bound of an fp32 accumulation
    # (2^-22 * sum|h*w|) of the reference's CPU fp16 F.linear.
    diff = np.abs(lg.astype(np.float64) - ref_lg.astype(np.float64))
    bound = np.spacing(np.abs(ref_lg)).astype(np.float64) + 2.0 ** -22 * (
        np.abs(h.astype(np.float64)) @ np.abs(wg.astype(np.float64)).T)
    assert np.all(diff <= bound)
    # On identical logits: indices bit-exact except exact probability ties.
    w, idx = orouter.route_from_logits(ref_lg, case["k"])
    p = orouter.softmax_f32(ref_lg)
    mism = np.where((idx != ref_i).any(-1))[0]
    for t in mism:
        assert np.array_equal(np.sort(p[t][idx[t]]), np.sort(p[t][ref_i[t]])), f"non-tie mismatch at {t}"
    assert len(mism) <= max(2, case["T"] // 1000)
    ok = np.setdiff1d(np.arange(case["T"]), mism)
    # fp32 weights: exp implementations differ by an ulp (numpy vs torch CPU).
    np.testing.assert_allclose(w[ok], ref_w[ok], rtol=1e-6, atol=0)


@pytest.mark.parametrize("name", sorted(DISPATCH_CASES))
def test_combine_oracle_bit_exact_vs_reference_forward_tokens(golden, name):
    case = DISPATCH_CASES[name]
    h, wg = dispatch_inputs(case)
    assert bytes(golden[f"dispatch/{name}/inputs_sha"]) == sha256_arrays(h, wg)
    idx = golden[f"dispatch/{name}/indices"]
    w = golden[f"dispatch/{name}/weights"]
    outs = {}
    for e in sorted(set(idx.reshape(-1).tolist())):
        m = (idx == e).any(-1)
        outs[e] = (h[m].astype(np.float32) * np.float32(fake_expert_scale(e))).astype(np.float16)
    out = omoe.combine_expert_outputs(case["T"], case["H"], idx, w, outs)
    assert np.array_equal(out.view(np.uint16), golden[f"dispatch/{name}/output"].view(np.uint16))


def test_oracle_nf4_layer_through_reference_dispatch(golden):
    case = ORACLE_LAYER_CASE
    h, wg, experts = oracle_layer_inputs(case)
    assert bytes(golden["oracle_layer/inputs_sha"]) == sha256_arrays(h, wg)
    idx, w = golden["oracle_layer/indices"], golden["oracle_layer/weights"]
    outs = {e: onf4.expert_forward(h[(idx == e).any(-1)], experts[e], case["hidden"], case["inter"])
            for e in sorted(set(idx.reshape(-1).tolist()))}
    out = omoe.combine_expert_outputs(case["T"], case["hidden"], idx, w, outs)
    assert np.array_equal(out.view(np.uint16), golden["oracle_layer/output"].view(np.uint16))


def test_gemv_and_multirow_semantics_differ_by_bf16_rounding_only():
    rng = np.random.default_rng(4)
    ex = onf4.make_expert(rng, 128, 256)
    st = ex["w1"]
    a = onf4.gemv_weight_f16(st, (256, 128)).astype(np.float32)
    b = onf4.dequant_weight_f16(st, (256, 128)).astype(np.float32)
    rel = np.abs(a - b) / np.maximum(np.abs(b), 1e-30)
    assert rel.max() < 2 ** -7


def test_tile16_is_a_permutation_of_store_blocks():
    rows, cols = 32, 128
    q = np.arange(rows * cols // 2, dtype=np.int64).astype(np.uint8)
    a = np.arange(rows * cols // 64, dtype=np.float32)
    qt, at = onf4.tile16(q, a, rows, cols)
    assert sorted(at.tolist()) == sorted(a.tolist())
    # row 17, block 1 lives in tile 1, block 1, row 1
    seg = ((1 * (cols // 64) + 1) * 16 + 1)
    assert at[seg] == a[17 * (cols // 64) + 1]
    assert np.array_equal(qt[seg * 32:(seg + 1) * 32], q[17 * cols // 2 + 32:17 * cols // 2 + 64])
