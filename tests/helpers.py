"""Test helpers: seeded NF4 experts (via the oracle) moved into product objects."""
from __future__ import annotations

import types
from pathlib import Path

import numpy as np
import torch

from oracle import nf4 as onf4


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


# Expert / layer output tolerance (fp16 outputs, fp32 accumulation in both the
# kernels and the oracle; differences come from accumulation order only).
REL_L2_TOL = 2e-3
MAX_ABS_TOL = 1e-2


def assert_close_fp16(actual, expected, rel=REL_L2_TOL, mabs=MAX_ABS_TOL, what=""):
    a = np.asarray(actual, np.float32)
    e = np.asarray(expected, np.float32)
    r, m = rel_l2(a, e), max_abs(a, e)
    scale = max(1.0, float(np.abs(e).max()))
    assert r <= rel and m <= mabs * scale, f"{what}: rel_l2={r:.3e} max_abs={m:.3e} (scale {scale:.3g})"
    return r, m


def state_to_torch(st: dict, device) -> dict:
    out = {}
    for k, v in st.items():
        if v is None:
            out[k] = None
        elif k == "offset":
            out[k] = torch.tensor(float(np.asarray(v).reshape(-1)[0]), dtype=torch.float32)
        else:
            out[k] = torch.from_numpy(np.ascontiguousarray(v)).to(device)
    return out


def gpu_expert(ex_np: dict, hidden: int, inter: int, device="cuda"):
    from moeinfra_b200.transfer.nf4_reconstruct import ReconstructedNF4Expert

    original = types.SimpleNamespace(hidden_size=hidden, intermediate_size=inter)
    gpu_state = {n: state_to_torch(ex_np[n], device) for n in ("w1", "w2", "w3")}
    return ReconstructedNF4Expert(original, gpu_state)


def make_experts(seed: int, E: int, hidden: int, inter: int, std: float = 0.02, nested=False):
    rng = np.random.default_rng(seed)
    return [onf4.make_expert(rng, hidden, inter, std=std, nested=nested) for _ in range(E)]


def write_tiny_checkpoint(path, hidden: int = 64, inter: int = 128, layers: int = 2,
                          experts: int = 4, vocab: int = 32, heads: int = 4, kv_heads: int = 2,
                          seed: int = 0) -> dict:
    """A small Mixtral-shaped safetensors checkpoint (dense tensors + index) under ``path``."""
    import json

    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    hd = hidden // heads

    def r(*shape):
        return (torch.randn(*shape, generator=g) * 0.05).to(torch.bfloat16)

    tensors = {"model.embed_tokens.weight": r(vocab, hidden),
               "model.norm.weight": (1 + r(hidden).float() * 0.1).to(torch.bfloat16),
               "lm_head.weight": r(vocab, hidden)}
    for l in range(layers):
        p = f"model.layers.{l}"
        tensors.update({
            f"{p}.input_layernorm.weight": (1 + r(hidden).float() * 0.1).to(torch.bfloat16),
            f"{p}.self_attn.q_proj.weight": r(heads * hd, hidden),
            f"{p}.self_attn.k_proj.weight": r(kv_heads * hd, hidden),
            f"{p}.self_attn.v_proj.weight": r(kv_heads * hd, hidden),
            f"{p}.self_attn.o_proj.weight": r(hidden, heads * hd),
            f"{p}.post_attention_layernorm.weight": (1 + r(hidden).float() * 0.1).to(torch.bfloat16),
            f"{p}.block_sparse_moe.gate.weight": r(experts, hidden),
        })
        for e in range(experts):
            q = f"{p}.block_sparse_moe.experts.{e}"
            tensors[f"{q}.w1.weight"] = r(inter, hidden)
            tensors[f"{q}.w2.weight"] = r(hidden, inter)
            tensors[f"{q}.w3.weight"] = r(inter, hidden)
    shard = "model-00001-of-00001.safetensors"
    save_file(tensors, str(Path(path) / shard))
    (Path(path) / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {k: shard for k in tensors}}))
    return tensors


def tiny_loader(path, store_paths=None, hidden: int = 64, inter: int = 128, layers: int = 2,
                experts: int = 4):
    from moeinfra_b200.model.loader import ModelLoader

    loader = ModelLoader(model_name=str(path), num_layers=layers, num_experts=experts,
                         hidden_size=hidden, intermediate_size=inter,
                         expert_store_paths=store_paths)
    loader.load()
    return loader
