"""End-to-end Mixtral NF4 inference (API of the reference's ``engine/engine.py``).

``InferenceEngine(config).generate(ForwardRequest) -> ForwardResult`` with the
reference's config keys (``model.*``, ``cache.*``, ``transfer.*``,
``engine/engine.py:69-178``) and result fields (``logits``, ``token_ids``,
``ttft_ms``, ``tps``, ``stage_timings``; ``:453-498``).  What differs, B200-first:

* the transfer scheduler gets a real pinned staging pool and a copy stream
  (the reference wires ``staging_pool=None, transfer_stream=None``,
  ``:148-150``, with which no expert can ever reach the GPU);
* decode is batched: B sequences of equal prompt length advance together
  (the reference decodes batch 1 only, ``:579-580``);
* the dense part is :class:`~moeinfra_b200.engine.dense.DenseStack` (fused
  q/k/v projection, static KV cache) instead of HF modules over a
  ``DynamicCache``; with every expert GPU-resident the whole decode step
  (32 layers, routing and experts included) is captured once as a CUDA graph
  and replayed per token, and greedy tokens stay on the device until the end;
* offloaded experts flow store -> CPU tier -> pinned slab -> one H2D copy ->
  resident expert (``MoELayer._ensure_expert_on_gpu``), and the optional
  ``PrefetchEngine`` (``transfer.prefetch_policy``) requests the next layer's
  experts on the copy stream while the current layer computes.

Extra config keys (all optional): ``model.{num_attention_heads,
num_key_value_heads, vocab_size, rope_theta, rms_norm_eps}`` when the
checkpoint has no ``config.json``; ``cache.gpu_budget_bytes``;
``transfer.{prefetch_policy, staging_slots}``; ``engine.{max_batch,
max_seq_len, cuda_graphs, preload_experts}``; ``parallel.expert_parallel``:
one process per GPU (``torch.distributed`` initialised), rank r keeps experts
``[r*E/G, (r+1)*E/G)`` of every layer resident and runs its own sequences;
each MoE layer is an ``ExpertParallelMoE`` (peer-memory exchange for decode
steps, NCCL all-to-all for prefill); every rank must call ``generate`` with
the same batch shape.
"""
from __future__ import annotations

import json
import logging
import time
from pathlib import Path
from typing import Optional

import torch

from moeinfra_b200 import kernels
from moeinfra_b200.cache.manager import CacheManager
from moeinfra_b200.cache.types import EvictionPolicy
from moeinfra_b200.engine.dense import DenseConfig, DenseStack
from moeinfra_b200.engine.prefetch import PrefetchEngine
from moeinfra_b200.engine.router import ExpertRouter
from moeinfra_b200.engine.types import ForwardRequest, ForwardResult, PrefetchPolicy
from moeinfra_b200.model.loader import ModelLoader
from moeinfra_b200.model.moe_layer import MoELayer
from moeinfra_b200.transfer.pinned_memory import PinnedMemoryBudget
from moeinfra_b200.transfer.reusable_staging import ReusablePinnedStagingPool
from moeinfra_b200.transfer.scheduler import TransferScheduler

_DTYPES = {"float16": torch.float16, "fp16": torch.float16}


def _mixtral_config(model_cfg: dict):
    """HF ``MixtralConfig`` from the checkpoint's config.json, else from the config dict."""
    from transformers import MixtralConfig

    name = model_cfg.get("name")
    if name and (Path(name) / "config.json").is_file():
        return MixtralConfig.from_pretrained(name)
    fields = {
        "hidden_size": model_cfg.get("hidden_size", 4096),
        "intermediate_size": model_cfg.get("intermediate_size", 14336),
        "num_hidden_layers": model_cfg.get("num_layers", 32),
        "num_attention_heads": model_cfg.get("num_attention_heads", 32),
        "num_key_value_heads": model_cfg.get("num_key_value_heads", 8),
        "num_local_experts": model_cfg.get("num_experts", 8),
        "num_experts_per_tok": model_cfg.get("num_experts_per_tok", 2),
        "vocab_size": model_cfg.get("vocab_size", 32000),
        "rms_norm_eps": model_cfg.get("rms_norm_eps", 1e-5),
        "rope_theta": model_cfg.get("rope_theta", 1e6),
    }
    return MixtralConfig(**fields)


def expert_bytes(hidden: int, inter: int) -> int:
    """Store bytes of one NF4 expert (packed codes, fp32 absmax, codebooks, metadata slack)."""
    per = hidden * inter // 2 + hidden * inter // 64 * 4 + 64
    return 3 * per


class InferenceEngine:
    """Mixtral NF4 MoE inference with GPU-resident or CPU-offloaded experts."""

    def __init__(self, config: dict, logger: Optional[logging.Logger] = None,
                 model_loader=None) -> None:
        """``model_loader`` (optional) replaces the ``ModelLoader`` built from ``model.name``:
        any object with the loader's ``load`` / ``load_layer`` / ``load_embeddings`` /
        ``load_final_norm`` / ``load_lm_head`` / ``load_expert`` methods."""
        self.config = config
        self._logger = logger or logging.getLogger(__name__)
        model_cfg = config.get("model", {})
        cache_cfg = config.get("cache", {})
        transfer_cfg = config.get("transfer", {})
        engine_cfg = config.get("engine", {})
        self._num_experts = model_cfg.get("num_experts", 8)
        self._num_experts_per_tok = model_cfg.get("num_experts_per_tok", 2)
        self._num_layers = model_cfg.get("num_layers", 32)
        self._device = torch.device(model_cfg.get("device", "cuda"))
        if self._device.type != "cuda":
            raise RuntimeError("InferenceEngine runs on a CUDA device (there is no CPU path)")
        dtype = str(model_cfg.get("dtype", "float16")).lower()
        if dtype not in _DTYPES:
            raise ValueError(f"Unsupported model dtype {dtype!r}; the NF4 kernels compute in fp16")
        self._dtype = _DTYPES[dtype]
        self._mixtral_config = _mixtral_config(model_cfg)
        self._hidden = model_cfg.get("hidden_size", self._mixtral_config.hidden_size)
        self._inter = model_cfg.get("intermediate_size", self._mixtral_config.intermediate_size)
        self._max_batch = int(engine_cfg.get("max_batch", 1))
        self._max_len = int(engine_cfg.get("max_seq_len", 2048))
        self._use_graphs = bool(engine_cfg.get("cuda_graphs", True))
        self._preload = bool(engine_cfg.get("preload_experts", False))
        self._ep = bool(config.get("parallel", {}).get("expert_parallel", False))
        self._peer = None
        if self._ep and not (torch.distributed.is_available() and torch.distributed.is_initialized()):
            raise RuntimeError("parallel.expert_parallel needs an initialised process group")

        self._cache_manager = CacheManager(
            gpu_slots=cache_cfg.get("gpu_slots", 8), cpu_slots=cache_cfg.get("cpu_slots", 32),
            policy=EvictionPolicy(cache_cfg.get("eviction_policy", "lru")), logger=self._logger,
            gpu_budget_bytes=cache_cfg.get("gpu_budget_bytes"))
        slot = expert_bytes(self._hidden, self._inter) + (1 << 20)
        nslots = int(transfer_cfg.get("staging_slots", 2))
        self._staging_pool = ReusablePinnedStagingPool(PinnedMemoryBudget(nslots * slot), slot)
        with torch.cuda.device(self._device):
            self._transfer_stream = torch.cuda.Stream(self._device)
        self._transfer_scheduler = TransferScheduler(
            cache_manager=self._cache_manager,
            bandwidth_gbps=transfer_cfg.get("bandwidth_gbps", 8.0),
            max_concurrent=transfer_cfg.get("max_concurrent_transfers", 4),
            staging_pool=self._staging_pool, transfer_stream=self._transfer_stream,
            logger=self._logger)
        self._prefetch_engine = PrefetchEngine(
            cache_manager=self._cache_manager, transfer_scheduler=self._transfer_scheduler,
            policy=PrefetchPolicy(transfer_cfg.get("prefetch_policy", "none")),
            depth=transfer_cfg.get("prefetch_depth", 2), logger=self._logger)
        self._model = model_loader if model_loader is not None else ModelLoader(
            model_name=model_cfg.get("name"), num_layers=self._num_layers,
            num_experts=self._num_experts, hidden_size=self._hidden,
            intermediate_size=self._inter, quantization=model_cfg.get("quantization", "int4"),
            logger=self._logger, expert_store_paths=model_cfg.get("expert_store_paths"))
        self._stack: Optional[DenseStack] = None
        self._moe_layers: list[MoELayer] = []
        self._graphs: dict = {}
        self._last_logits: Optional[torch.Tensor] = None
        self._runtime_initialized = False

    # -- runtime ------------------------------------------------------------------------
    @torch.no_grad()
    def _initialize_runtime(self) -> None:
        if self._runtime_initialized:
            return
        self._model.load()
        dev = self._device
        layers = []
        if self._ep:
            from moeinfra_b200.ep import ExpertParallelMoE, capacity, local_experts
            from moeinfra_b200.ep_p2p import PeerExchange
            from moeinfra_b200.transfer.nf4_reconstruct import resident_expert
            rank = torch.distributed.get_rank()
            world = torch.distributed.get_world_size()
            owned = local_experts(rank, self._num_experts, world)
            if world > 1:
                self._peer = PeerExchange(self._num_layers, world, rank,
                                          capacity(self._max_batch, self._num_experts_per_tok,
                                                   self._num_experts, world), self._hidden,
                                          device=dev)
        for layer_id in range(self._num_layers):
            w = self._model.load_layer(layer_id)
            router = ExpertRouter(w.moe_gate.to(device=dev, dtype=self._dtype),
                                  num_experts_per_tok=self._num_experts_per_tok,
                                  logger=self._logger)
            if self._ep:
                with torch.cuda.device(dev):
                    local = [resident_expert(self._model.load_expert(layer_id, e), dev)
                             for e in owned]
                self._moe_layers.append(ExpertParallelMoE(
                    router, local, rank=rank, world_size=world,
                    max_tokens=self._max_batch * self._max_len, peer=self._peer,
                    layer_slot=layer_id))
                layers.append(w)
                continue
            moe = MoELayer(layer_id, router, self._cache_manager, self._model,
                           self._transfer_scheduler, logger=self._logger,
                           prefetch_engine=self._prefetch_engine)
            moe.check_each_call = False  # generate() checks the device once per generation
            self._moe_layers.append(moe)
            layers.append(w)
        self._stack = DenseStack(
            DenseConfig.from_mixtral(self._mixtral_config), layers,
            self._model.load_embeddings(), self._model.load_final_norm(),
            self._model.load_lm_head(), self._moe_layers, dev, self._max_batch, self._max_len,
            self._dtype)
        if self._prefetch_engine.policy != PrefetchPolicy.NONE:
            self._stack.layer_hook = self._after_layer
        if self._preload:
            self.preload_experts()
        self._runtime_initialized = True

    def _after_layer(self, layer_id: int, moe: MoELayer) -> None:
        idx = getattr(moe, "last_expert_indices", None)
        if idx is not None:
            self._prefetch_engine.on_layer_complete(layer_id, idx)

    def preload_experts(self) -> None:
        """Make every expert GPU-resident now (needs gpu_slots >= layers x experts)."""
        if self._ep:
            return  # expert-parallel layers hold their shards resident from the start
        with torch.cuda.device(self._device):
            for moe in self._moe_layers:
                for e in range(self._num_experts):
                    moe._ensure_expert_on_gpu(e)
        torch.cuda.synchronize(self._device)

    def all_experts_resident(self) -> bool:
        if self._ep:
            return True  # every rank holds its shard of every layer resident
        cm = self._cache_manager
        return all(cm.is_gpu_resident(l, e) for l in range(self._num_layers)
                   for e in range(self._num_experts))

    # -- generation -----------------------------------------------------------------------
    def generate(self, request: ForwardRequest) -> ForwardResult:
        """Prefill the prompt, then greedy-decode ``max_new_tokens`` tokens."""
        self._initialize_runtime()
        timings: dict = {}
        B = request.input_ids.shape[0] if request.input_ids.ndim == 2 else 0
        if (self._use_graphs and request.max_new_tokens > 1 and 0 < B <= self._max_batch
                and self.all_experts_resident()):
            with torch.cuda.device(self._device):
                self._graph_for(B)  # built once per batch size, outside the timed stages
        torch.cuda.synchronize(self._device)
        t0 = time.perf_counter()
        logits = self._prefill(request.input_ids, request.attention_mask)
        torch.cuda.synchronize(self._device)
        ttft_ms = (time.perf_counter() - t0) * 1e3
        timings["prefill"] = ttft_ms
        t1 = time.perf_counter()
        tokens = self._decode(logits, request.max_new_tokens)
        torch.cuda.synchronize(self._device)
        decode_ms = (time.perf_counter() - t1) * 1e3
        timings["decode"] = decode_ms
        kernels.check_device(self._device)
        B = logits.shape[0]
        steps = max(request.max_new_tokens - 1, 0)
        tps = B * steps / (decode_ms / 1e3) if steps > 0 and decode_ms > 0 else 0.0
        timings["cuda_graph_decode"] = bool(self._graphs)
        timings["h2d_bytes"] = sum(
            p.get("bytes_transferred", 0) for p in self._transfer_scheduler_profile())
        token_ids = tokens[0] if B == 1 else tokens
        return ForwardResult(logits=self._last_logits if self._last_logits is not None else logits,
                             token_ids=token_ids, ttft_ms=ttft_ms, tps=tps, stage_timings=timings)

    def _transfer_scheduler_profile(self) -> list:
        from moeinfra_b200.transfer.scheduler import EXECUTE_NEXT_PROFILE
        return EXECUTE_NEXT_PROFILE

    @torch.no_grad()
    def _prefill(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None):
        if self._stack is None:
            raise RuntimeError("Inference runtime has not been initialized")
        if input_ids.ndim != 2:
            raise ValueError(f"input_ids must have shape (batch, seq_len), got {tuple(input_ids.shape)}")
        B, S = input_ids.shape
        if S <= 0:
            raise ValueError("input_ids must contain at least one token")
        if B > self._max_batch:
            raise ValueError(f"batch {B} exceeds engine.max_batch={self._max_batch}")
        if attention_mask is not None:
            if attention_mask.shape != input_ids.shape:
                raise ValueError("attention_mask must have the same shape as input_ids")
            if not bool((attention_mask != 0).all()):
                raise ValueError("padded prompts are not supported: sequences of one batch "
                                 "must have equal length")
        ids = input_ids.to(device=self._device, dtype=torch.long, non_blocking=True)
        with torch.cuda.device(self._device):
            logits = self._stack.forward(ids, pos0=0)
        self._prompt_len = S
        self._last_logits = logits[:, None, :]
        return self._last_logits

    def _decode_step_fn(self, ids_buf, pos_buf):
        def step():
            logits = self._stack.forward(ids_buf, decode_pos=pos_buf)
            ids_buf.copy_(logits.argmax(dim=-1, keepdim=True))
            pos_buf.add_(1)
            return logits
        return step

    @torch.no_grad()
    def _decode(self, next_token_logits: torch.Tensor, max_new_tokens: int) -> list:
        if self._stack is None:
            raise RuntimeError("Inference runtime has not been initialized")
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens must be non-negative")
        if max_new_tokens == 0:
            return [[] for _ in range(next_token_logits.shape[0])]
        B = next_token_logits.shape[0]
        S = self._prompt_len
        if S + max_new_tokens > self._max_len:
            raise ValueError(f"{S + max_new_tokens} positions exceed engine.max_seq_len={self._max_len}")
        dev = self._device
        with torch.cuda.device(dev):
            hist = torch.empty(B, max_new_tokens, dtype=torch.long, device=dev)
            first = next_token_logits[:, -1, :].argmax(dim=-1)
            hist[:, 0] = first
            if max_new_tokens > 1:
                use_graph = self._use_graphs and self.all_experts_resident()
                if use_graph:
                    g, ids_buf, pos_buf, out = self._graph_for(B)
                    ids_buf.copy_(first[:, None])
                    pos_buf.fill_(S)
                    for i in range(1, max_new_tokens):
                        g.replay()
                        hist[:, i] = ids_buf[:, 0]
                    self._last_logits = out[:, None, :]
                else:
                    ids_buf = first[:, None].clone()
                    pos_buf = torch.full((1,), S, dtype=torch.long, device=dev)
                    step = self._decode_step_fn(ids_buf, pos_buf)
                    for i in range(1, max_new_tokens):
                        logits = step()
                        hist[:, i] = ids_buf[:, 0]
                    self._last_logits = logits[:, None, :]
        return hist.cpu().tolist()

    def _graph_for(self, B: int):
        """The captured decode step for batch B (built once; replays advance it on the device)."""
        ent = self._graphs.get(B)
        if ent is not None:
            return ent
        dev = self._device
        ids_buf = torch.zeros(B, 1, dtype=torch.long, device=dev)
        pos_buf = torch.zeros(1, dtype=torch.long, device=dev)
        step = self._decode_step_fn(ids_buf, pos_buf)
        # Warm up on a side stream (allocations, one-time kernel setup), then
        # capture.  The warm-up runs at the last cache position, which a
        # generation writes before it ever reads it.
        pos_buf.fill_(self._max_len - 1)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = step()
        ent = (g, ids_buf, pos_buf, out)
        self._graphs[B] = ent
        return ent

    def close(self) -> None:
        for g, *_ in self._graphs.values():
            g.reset()
        self._graphs.clear()
        if self._peer is not None:
            torch.cuda.synchronize(self._device)
            torch.distributed.barrier()
            self._peer.close()
            self._peer = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False

    @property
    def cache_manager(self) -> CacheManager:
        return self._cache_manager

    @property
    def transfer_scheduler(self) -> TransferScheduler:
        return self._transfer_scheduler

    @property
    def prefetch_engine(self) -> PrefetchEngine:
        return self._prefetch_engine

    @property
    def model_loader(self) -> ModelLoader:
        return self._model
