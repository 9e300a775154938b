"""CPU contract of the model I/O classes and the NF4 expert-store format.

Follows the reference's ``tests/test_model_loader.py``,
``tests/test_model_loader_fast_path.py`` and
``tests/test_prequantized_expert.py``:

* ``ModelLoader`` reads the dense tensors of an indexed safetensors checkpoint
  (embeddings, final norm, lm_head, per-layer attention / norm / gate
  weights), rejects out-of-range layers, resolves
  ``layer_LL_expert_EE.safetensors`` across several store directories in
  order, and returns a CPU ``PrequantizedNF4Expert`` whose tensors equal the
  stored ones (``torch.equal``); a preloaded expert is served before any file;
* the store round trip: quantize -> write -> load gives bit-identical
  serialized state, and the canonical staging state built from it;
* this package's quantizer (no bitsandbytes) matches the oracle's restatement
  of the NF4 quantizer exactly (codes and absmax).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import tiny_loader, write_tiny_checkpoint

H, I, L, E = 64, 128, 2, 4


def _expert(seed: int, nested: bool = False):
    from moeinfra_b200.model.expert import PrequantizedNF4Expert
    from moeinfra_b200.model.nf4_format import quantize_nf4

    g = torch.Generator().manual_seed(seed)
    st = {}
    for name, shape in (("w1", (I, H)), ("w2", (H, I)), ("w3", (I, H))):
        st[name] = quantize_nf4((torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16),
                                compress_statistics=nested)
    return PrequantizedNF4Expert.from_serialized(st["w1"], st["w2"], st["w3"], hidden_size=H,
                                                 intermediate_size=I)


def _assert_states_equal(got: dict, want: dict):
    assert got.keys() == want.keys()
    for k in want:
        assert torch.equal(got[k], want[k]), k


def test_dense_tensors_come_back_unchanged(tmp_path):
    tensors = write_tiny_checkpoint(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    loader = tiny_loader(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    assert torch.equal(loader.load_embeddings(), tensors["model.embed_tokens.weight"])
    assert torch.equal(loader.load_final_norm(), tensors["model.norm.weight"])
    assert torch.equal(loader.load_lm_head(), tensors["lm_head.weight"])
    lw = loader.load_layer(1)
    p = "model.layers.1"
    assert torch.equal(lw.q_proj, tensors[f"{p}.self_attn.q_proj.weight"])
    assert torch.equal(lw.k_proj, tensors[f"{p}.self_attn.k_proj.weight"])
    assert torch.equal(lw.v_proj, tensors[f"{p}.self_attn.v_proj.weight"])
    assert torch.equal(lw.o_proj, tensors[f"{p}.self_attn.o_proj.weight"])
    assert torch.equal(lw.input_layernorm, tensors[f"{p}.input_layernorm.weight"])
    assert torch.equal(lw.post_attention_layernorm, tensors[f"{p}.post_attention_layernorm.weight"])
    assert torch.equal(lw.moe_gate, tensors[f"{p}.block_sparse_moe.gate.weight"])


def test_loader_argument_and_state_errors(tmp_path):
    from moeinfra_b200.model.loader import ModelLoader

    write_tiny_checkpoint(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    loader = tiny_loader(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    for bad in (-1, L):
        with pytest.raises((IndexError, ValueError)):
            loader.load_layer(bad)
    with pytest.raises((IndexError, ValueError)):
        loader.load_expert(0, E)
    unloaded = ModelLoader(str(tmp_path), num_layers=L, num_experts=E, hidden_size=H,
                           intermediate_size=I)
    with pytest.raises(RuntimeError, match="load"):
        unloaded.load_layer(0)
    with pytest.raises(RuntimeError):
        ModelLoader(str(tmp_path / "nope"), L, E, H, I).load()


def test_store_paths_are_searched_in_order(tmp_path):
    from moeinfra_b200.model.nf4_format import save_expert_store

    write_tiny_checkpoint(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    first, second = tmp_path / "s1", tmp_path / "s2"
    first.mkdir()
    a, b = _expert(1), _expert(2)
    save_expert_store(second, 1, 2, b)  # only in the second store
    save_expert_store(first, 0, 0, a)
    save_expert_store(second, 0, 0, b)  # shadowed by the first store
    loader = tiny_loader(tmp_path, [str(first), str(second)], hidden=H, inter=I, layers=L,
                         experts=E)
    assert loader._resolve_expert_path(1, 2) == second / "layer_01_expert_02.safetensors"
    assert loader._resolve_expert_path(0, 0) == first / "layer_00_expert_00.safetensors"
    got = loader.load_expert(0, 0)
    _assert_states_equal(got.w1, a.w1)
    with pytest.raises(FileNotFoundError, match="Searched stores"):
        loader._resolve_expert_path(1, 3)


@pytest.mark.parametrize("nested", [False, True])
def test_store_round_trip_is_bit_identical_and_stays_on_cpu(tmp_path, nested):
    from moeinfra_b200.model.expert import PrequantizedNF4Expert
    from moeinfra_b200.model.nf4_format import canonical_state, save_expert_store

    write_tiny_checkpoint(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    ex = _expert(3, nested)
    save_expert_store(tmp_path / "store", 1, 3, ex)
    loader = tiny_loader(tmp_path, [str(tmp_path / "store")], hidden=H, inter=I, layers=L,
                         experts=E)
    got = loader.load_expert(1, 3)
    assert isinstance(got, PrequantizedNF4Expert)
    assert got.device.type == "cpu"
    assert (got.hidden_size, got.intermediate_size) == (H, I)
    for proj in ("w1", "w2", "w3"):
        _assert_states_equal(getattr(got, proj), getattr(ex, proj))
        a, b = canonical_state(getattr(got, proj)), canonical_state(getattr(ex, proj))
        for k in b:
            if b[k] is None:
                assert a[k] is None
            else:
                assert torch.equal(a[k], b[k])
    assert got.size_bytes == ex.size_bytes


def test_preloaded_expert_is_served_first(tmp_path):
    write_tiny_checkpoint(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    loader = tiny_loader(tmp_path, [str(tmp_path / "empty")], hidden=H, inter=I, layers=L,
                         experts=E)
    ex = _expert(4)
    loader.set_preloaded_cpu_experts({(1, 1): ex})
    assert loader.load_expert(1, 1) is ex


def test_without_a_store_the_checkpoint_weights_are_quantized(tmp_path):
    from moeinfra_b200.model.expert import QuantizedMixtralExpert
    from moeinfra_b200.model.nf4_format import quantize_nf4

    tensors = write_tiny_checkpoint(tmp_path, hidden=H, inter=I, layers=L, experts=E)
    loader = tiny_loader(tmp_path, None, hidden=H, inter=I, layers=L, experts=E)
    ex = loader.load_expert(0, 2)
    assert isinstance(ex, QuantizedMixtralExpert)
    assert (ex.hidden_size, ex.intermediate_size) == (H, I)
    want = quantize_nf4(tensors["model.layers.0.block_sparse_moe.experts.2.w1.weight"])
    assert torch.equal(ex.w1.state["weight"], want["weight"])
    assert torch.equal(ex.w1.state["weight.absmax"], want["weight.absmax"])


def test_required_serialized_keys_are_enforced():
    from moeinfra_b200.model.expert import PrequantizedNF4Expert

    ex = _expert(5)
    broken = dict(ex.w2)
    del broken["weight.quant_map"]
    with pytest.raises(ValueError, match="w2"):
        PrequantizedNF4Expert.from_serialized(ex.w1, broken, ex.w3, H, I)


def test_unparseable_metadata_blob_falls_back_to_defaults():
    """The reference's own fixtures store an arbitrary 8-byte blob."""
    from moeinfra_b200.model.nf4_format import BLOB_KEY, canonical_state

    st = dict(_expert(6).w1)
    st[BLOB_KEY] = torch.tensor([64, 0, 0, 0, 0, 0, 0, 0], dtype=torch.uint8)
    c = canonical_state(st, "w1")
    assert torch.equal(c["weight"], st["weight"]) and c["offset"] is None


@pytest.mark.parametrize("shape", [(128, 64), (64, 256)])
def test_quantizer_matches_the_oracle_exactly(shape):
    from moeinfra_b200.model.nf4_format import quantize_nf4_packed
    from oracle import nf4 as onf4

    g = torch.Generator().manual_seed(shape[0])
    w = (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)
    q, a, code = quantize_nf4_packed(w)
    qo, ao = onf4.quantize_nf4(w.float().numpy())
    assert np.array_equal(q.numpy(), qo)
    assert np.array_equal(a.numpy().view(np.uint32), ao.view(np.uint32))
    assert np.array_equal(code.numpy(), onf4.nf4_codebook())
