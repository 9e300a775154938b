"""Mixtral sparse-MoE layer with expert offloading (API of ``model/moe_layer.py``).

``_forward_tokens`` keeps the reference's semantics (``:117-211``): one routing
pass, the routed experts made GPU-resident in ascending id, each expert run
once on its tokens, ``output[mask] += y * w`` in ascending expert id with one
fp16 rounding per expert, and experts that were not resident beforehand
demoted afterwards.  How it runs on a B200:

* all experts of the layer GPU-resident (the resident serving mode): one fused
  launch sequence -- router, permute, NF4 SwiGLU experts, combine -- with no
  host synchronisation and no per-expert cache lookups;
* otherwise (offload mode): route on the GPU, read back the routed set (the
  one device->host sync the residency decision needs, like the reference's
  ``unique().tolist()`` at ``:150-153``), make those experts resident through
  ``_ensure_expert_on_gpu`` (same seam, ``:39-115``), then permute / experts /
  combine kernels on that same routing (no second routing pass), and read the
  device error word at that sync point;
* experts that are not NF4 GPU experts (e.g. test doubles installed through
  the ``_ensure_expert_on_gpu`` seam) are called one by one on their tokens and
  combined by the same combine kernel.
"""
from __future__ import annotations

import logging
import time
from typing import Optional

import torch

from moeinfra_b200 import kernels
from moeinfra_b200.transfer.types import TransferDirection, TransferPriority, TransferRequest


class MoELayer:
    """Single Mixtral MoE layer with expert offloading."""

    def __init__(self, layer_id: int, router, cache_manager, model_loader, transfer_scheduler,
                 logger: Optional[logging.Logger] = None, prefetch_engine=None) -> None:
        self.layer_id = layer_id
        self.router = router
        self.cache_manager = cache_manager
        self.model_loader = model_loader
        self.transfer_scheduler = transfer_scheduler
        self.prefetch_engine = prefetch_engine
        self._logger = logger or logging.getLogger(__name__)
        self._desc_cache: Optional[tuple] = None
        # Routing of the last offloaded call (device int64 [T, k]); None after a
        # resident call.  The engine hands it to the prefetcher.
        self.last_expert_indices: Optional[torch.Tensor] = None
        # Read the device error word at the offload path's sync point (one more
        # stream synchronisation per call).  An owner that checks at its own
        # sync points (the engine, once per generation) turns this off.
        self.check_each_call = True

    # -- residency (reference :39-115) -------------------------------------------
    def _ensure_expert_on_gpu(self, expert_id: int):
        """Return an expert that is resident on GPU."""
        expert = self.cache_manager.get(self.layer_id, expert_id)
        if expert is None:
            expert = self.model_loader.load_expert(self.layer_id, expert_id)
            self.cache_manager.put(self.layer_id, expert_id, expert, device="cpu")
        if expert.device.type == "cuda":
            return expert
        # A prefetch of this expert may already be on the copy stream: adopt it.
        adopt = getattr(self.transfer_scheduler, "adopt_async", None)
        if adopt is not None:
            adopted = adopt(self.layer_id, expert_id)
            if adopted is not None:
                if self.prefetch_engine is not None:
                    self.prefetch_engine.forget(self.layer_id, expert_id)
                return adopted
        request = TransferRequest(
            request_id=f"layer-{self.layer_id}-expert-{expert_id}-{id(self)}",
            layer_id=self.layer_id, expert_id=expert_id,
            direction=TransferDirection.CPU_TO_GPU, priority=TransferPriority.HIGH,
            issued_at=time.monotonic())
        if not self.transfer_scheduler.submit(request):
            raise RuntimeError(
                f"Failed to submit transfer for layer={self.layer_id}, expert={expert_id}")
        result = self.transfer_scheduler.execute_next()
        if result is None or not result.success:
            error = result.error if result is not None else "no transfer result"
            raise RuntimeError(
                f"Failed to transfer expert layer={self.layer_id}, expert={expert_id}: {error}")
        expert = self.cache_manager.get(self.layer_id, expert_id)
        if expert is None or expert.device.type != "cuda":
            raise RuntimeError(f"Expert layer={self.layer_id}, expert={expert_id} "
                               "was not resident on GPU after transfer")
        return expert

    # -- fused-kernel helpers ------------------------------------------------------
    def _descriptor_array(self, experts: dict):
        """ctypes expert table for the fused kernels; ``None`` if any expert is not NF4."""
        E = self.router.num_experts
        descs = []
        sig = None
        fill = None
        for e in range(E):
            ex = experts.get(e)
            if ex is None:
                descs.append(None)
                continue
            d = getattr(ex, "nf4_descriptor", None)
            if d is None:
                return None
            s = getattr(ex, "code_signature", None)
            if sig is None:
                sig = s
            elif s != sig:
                return None  # the fused kernels share one codebook per launch
            descs.append(d)
            fill = fill or d
        if fill is None:
            return None
        # Unrouted experts are never read by the kernels (zero tokens); any valid
        # descriptor fills their slot.
        return kernels.expert_array([d if d is not None else fill for d in descs])

    def _resident_table(self):
        cm = self.cache_manager
        if cm is None or not hasattr(cm, "peek_gpu"):
            return None
        experts = {}
        for e in range(self.router.num_experts):
            ex = cm.peek_gpu(self.layer_id, e)
            if ex is None:
                return None
            experts[e] = ex
        key = tuple(id(experts[e]) for e in range(self.router.num_experts))
        if self._desc_cache is not None and self._desc_cache[0] == key:
            return self._desc_cache[1]
        table = self._descriptor_array(experts)
        if table is not None:
            self._desc_cache = (key, table, experts)
        return table

    def _fused(self, hidden_states: torch.Tensor, table, inter: int) -> torch.Tensor:
        router = self.router
        out, _, _ = kernels.layer_forward(hidden_states.contiguous(), router.gate_f16(), table,
                                          router.num_experts_per_tok, router.hidden_size, inter,
                                          routing=False)
        return out

    # -- forward -------------------------------------------------------------------
    @torch.no_grad()
    def _forward_tokens(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if hidden_states.ndim != 2:
            raise ValueError("hidden_states must have shape (tokens, hidden_size)")
        if hidden_states.shape[-1] != self.router.hidden_size:
            raise ValueError(f"hidden size {hidden_states.shape[-1]} != "
                             f"router hidden size {self.router.hidden_size}")
        if hidden_states.shape[0] == 0:
            return torch.zeros_like(hidden_states)

        table = self._resident_table()
        if table is not None:
            self.last_expert_indices = None
            return self._fused(hidden_states, table, self._desc_cache[2][0].intermediate_size)

        expert_indices, expert_weights = self.router.route(hidden_states)
        self.last_expert_indices = expert_indices
        unique_ids = sorted(int(e) for e in expert_indices.reshape(-1).unique().tolist())
        was_resident = {
            e: (self.cache_manager.is_gpu_resident(self.layer_id, e)
                if self.cache_manager is not None else True)
            for e in unique_ids
        }
        gpu_experts: dict = {}
        try:
            for e in unique_ids:
                gpu_experts[e] = self._ensure_expert_on_gpu(e)
            table = self._descriptor_array(gpu_experts)
            if table is not None:
                # The routing computed above is the one used: unrouted expert
                # slots get zero tokens from these same indices and are never read.
                inter = next(iter(gpu_experts.values())).intermediate_size
                out = kernels.routed_layer_forward(hidden_states.contiguous(), expert_indices,
                                                   expert_weights, table,
                                                   self.router.hidden_size, inter)
            else:
                out = self._per_expert(hidden_states, expert_indices, expert_weights, unique_ids,
                                       gpu_experts)
            # The offload path synchronises anyway (routing read-back): surface
            # any error a kernel flagged on the device here.
            if self.check_each_call:
                kernels.check_device(hidden_states.device)
            return out
        finally:
            if self.cache_manager is not None:
                for e in unique_ids:
                    if not was_resident[e]:
                        self.cache_manager.demote_to_cpu(self.layer_id, e)
            gpu_experts.clear()

    def check_device_errors(self) -> None:
        """Synchronise and raise ``RuntimeError`` if a kernel flagged an error.

        The resident path launches without host synchronisation; callers check
        at their own sync points (end of a decode step) with this.
        """
        kernels.check_device()

    def _per_expert(self, h, idx, w, unique_ids, experts) -> torch.Tensor:
        """Generic experts: call each on its tokens, then the ordered fp16 combine kernel."""
        E = self.router.num_experts
        offsets, pair_token, _, pair_slot = kernels.permute(idx.contiguous(), w.contiguous(), E)
        off = offsets.tolist()
        y_sorted = torch.empty(idx.numel(), h.shape[1], dtype=torch.float16, device=h.device)
        for e in unique_ids:
            lo, hi = off[e], off[e + 1]
            if hi == lo:
                continue
            x_e = h[pair_token[lo:hi].long()]
            y_sorted[lo:hi] = experts[e](x_e).to(torch.float16)
        return kernels.combine(y_sorted, pair_slot, idx.contiguous(), w.contiguous())

    def forward(self, hidden_states):
        if hidden_states.ndim == 3:
            b, s, hdim = hidden_states.shape
            out = self._forward_tokens(hidden_states.reshape(b * s, hdim))
            return out.reshape(b, s, hdim)
        if hidden_states.ndim == 2:
            return self._forward_tokens(hidden_states)
        raise ValueError("hidden_states must have shape (tokens, hidden_size) or "
                         "(batch, sequence, hidden_size)")
