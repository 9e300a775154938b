"""Checkpoint index and NF4 expert-store loader (API of the reference's ``model/loader.py``).

* ``load()`` indexes ``model.safetensors.index.json`` (``:80-150``);
* ``load_layer / load_embeddings / load_final_norm / load_lm_head`` read dense
  tensors, each shard opened once (``:160-301``);
* ``load_expert`` serves the preloaded-RAM tier first (``:343-348``), then the
  per-expert store file ``layer_{LL:02d}_expert_{EE:02d}.safetensors`` searched
  across ``expert_store_paths`` in order (``:303-316``, ``:353-381``), and
  otherwise quantizes the checkpoint's bf16 expert weights with this
  package's NF4 quantizer (the reference uses bitsandbytes, ``:383-421``).
"""
from __future__ import annotations

import json
import logging
from pathlib import Path
from typing import Optional

import torch
from safetensors import safe_open

from moeinfra_b200.model.expert import PrequantizedNF4Expert, QuantizedMixtralExpert
from moeinfra_b200.model.nf4_format import store_file_name
from moeinfra_b200.model.types import LayerWeights


def expert_filename(layer_id: int, expert_id: int) -> str:
    return store_file_name(layer_id, expert_id)


class ModelLoader:
    """Loads Mixtral dense weights and NF4 experts on demand."""

    def __init__(self, model_name: str, num_layers: int, num_experts: int, hidden_size: int,
                 intermediate_size: int, quantization: str = "int4",
                 logger: Optional[logging.Logger] = None,
                 expert_store_paths: Optional[list] = None) -> None:
        self.model_name = model_name
        self.num_layers = num_layers
        self.num_experts = num_experts
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.quantization = quantization
        self._logger = logger or logging.getLogger(__name__)
        self._expert_store_paths = [Path(p) for p in (expert_store_paths or [])]
        self._checkpoint_path: Optional[Path] = None
        self._is_loaded = False
        self._weight_map: dict[str, str] = {}
        self._preloaded_cpu_experts: dict[tuple[int, int], PrequantizedNF4Expert] = {}

    def load(self) -> None:
        """Locate and index the safetensors checkpoint (no weights are read)."""
        path = Path(self.model_name)
        if not path.exists():
            raise RuntimeError(f"Checkpoint path does not exist: {path}")
        if not path.is_dir():
            raise RuntimeError(f"Checkpoint path is not a directory: {path}")
        index_path = path / "model.safetensors.index.json"
        if not index_path.exists():
            raise RuntimeError(f"Safetensors index not found: {index_path}")
        try:
            index = json.loads(index_path.read_text(encoding="utf-8"))
        except (OSError, json.JSONDecodeError) as exc:
            raise RuntimeError(f"Failed to read safetensors index: {index_path}") from exc
        weight_map = index.get("weight_map")
        if not isinstance(weight_map, dict) or not weight_map:
            raise RuntimeError(f"Invalid or empty weight_map in {index_path}")
        missing = {s for s in weight_map.values() if not (path / s).exists()}
        if missing:
            raise RuntimeError(f"Checkpoint index references missing shards: {sorted(missing)}")
        self._checkpoint_path = path
        self._weight_map = weight_map
        self._is_loaded = True

    def _require_loaded(self) -> None:
        if not self._is_loaded or self._checkpoint_path is None:
            raise RuntimeError("Call ModelLoader.load() before requesting model weights.")

    def _load_tensors(self, names: dict[str, str]) -> dict[str, torch.Tensor]:
        self._require_loaded()
        try:
            by_shard: dict[str, list[str]] = {}
            for t in names.values():
                by_shard.setdefault(self._weight_map[t], []).append(t)
        except KeyError as exc:
            raise RuntimeError(f"Tensor not found in checkpoint index: {exc}") from exc
        out: dict[str, torch.Tensor] = {}
        for shard, tensors in by_shard.items():
            with safe_open(self._checkpoint_path / shard, framework="pt", device="cpu") as f:
                for t in tensors:
                    out[t] = f.get_tensor(t)
        return out

    def set_preloaded_cpu_experts(self, experts: dict) -> None:
        """Register permanently resident CPU experts prepared before inference."""
        self._preloaded_cpu_experts = dict(experts)

    def load_embeddings(self) -> torch.Tensor:
        return self._load_tensors({"e": "model.embed_tokens.weight"})["model.embed_tokens.weight"]

    def load_final_norm(self) -> torch.Tensor:
        return self._load_tensors({"n": "model.norm.weight"})["model.norm.weight"]

    def load_lm_head(self) -> torch.Tensor:
        return self._load_tensors({"h": "lm_head.weight"})["lm_head.weight"]

    def load_layer(self, layer_id: int) -> LayerWeights:
        self._require_loaded()
        if not 0 <= layer_id < self.num_layers:
            raise IndexError(f"layer_id {layer_id} out of range [0, {self.num_layers})")
        p = f"model.layers.{layer_id}"
        names = {
            "input_layernorm": f"{p}.input_layernorm.weight",
            "q_proj": f"{p}.self_attn.q_proj.weight",
            "k_proj": f"{p}.self_attn.k_proj.weight",
            "v_proj": f"{p}.self_attn.v_proj.weight",
            "o_proj": f"{p}.self_attn.o_proj.weight",
            "post_attention_layernorm": f"{p}.post_attention_layernorm.weight",
            "moe_gate": f"{p}.block_sparse_moe.gate.weight",
        }
        t = self._load_tensors(names)
        return LayerWeights(**{k: t[v] for k, v in names.items()})

    def _resolve_expert_path(self, layer_id: int, expert_id: int) -> Path:
        name = expert_filename(layer_id, expert_id)
        for store in self._expert_store_paths:
            if (store / name).is_file():
                return store / name
        searched = ", ".join(str(p) for p in self._expert_store_paths)
        raise FileNotFoundError(f"Pre-quantized expert not found: {name}. Searched stores: {searched}")

    def load_expert(self, layer_id: int, expert_id: int):
        if not self._is_loaded:
            raise RuntimeError("Call ModelLoader.load() before requesting individual experts.")
        if not 0 <= layer_id < self.num_layers:
            raise IndexError(f"layer_id {layer_id} out of range [0, {self.num_layers})")
        if not 0 <= expert_id < self.num_experts:
            raise IndexError(f"expert_id {expert_id} out of range [0, {self.num_experts})")
        pre = self._preloaded_cpu_experts.get((layer_id, expert_id))
        if pre is not None:
            return pre
        if self._checkpoint_path is None:
            raise RuntimeError("Checkpoint path is not initialized.")
        if self._expert_store_paths:
            path = self._resolve_expert_path(layer_id, expert_id)
            with safe_open(path, framework="pt", device="cpu") as f:
                state = {k: f.get_tensor(k) for k in f.keys()}

            def extract(prefix: str) -> dict:
                return {k[len(prefix):]: v for k, v in state.items() if k.startswith(prefix)}

            return PrequantizedNF4Expert.from_serialized(
                extract("w1."), extract("w2."), extract("w3."),
                hidden_size=self.hidden_size, intermediate_size=self.intermediate_size)
        prefix = f"model.layers.{layer_id}.block_sparse_moe.experts.{expert_id}."
        names = {n: prefix + n + ".weight" for n in ("w1", "w2", "w3")}
        t = self._load_tensors(names)
        return QuantizedMixtralExpert(w1=t[names["w1"]].to(torch.bfloat16),
                                      w2=t[names["w2"]].to(torch.bfloat16),
                                      w3=t[names["w3"]].to(torch.bfloat16))

    def get_expert_size_bytes(self) -> int:
        """Packed INT4 bytes of one expert (0.5 byte per parameter)."""
        return int(3 * self.hidden_size * self.intermediate_size * 0.5)

    def __repr__(self) -> str:
        return (f"ModelLoader(model={self.model_name!r}, layers={self.num_layers}, "
                f"experts={self.num_experts}, quant={self.quantization}, loaded={self._is_loaded})")
