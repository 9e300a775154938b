"""Expert prefetch on the asynchronous transfer API (API of the reference's ``engine/prefetch.py``).

``PrefetchEngine(cache_manager, transfer_scheduler, policy, depth)`` keeps the
reference's behaviour (``engine/prefetch.py:54-309``):

* ``schedule_prefetch(current_layer, expert_indices)`` -- nothing for
  ``PrefetchPolicy.NONE``; for ``NEXT_LAYER`` the unique experts routed in the
  current layer are requested for layer ``current_layer + 1``; for
  ``LOOKAHEAD`` for layers ``current_layer + 1 .. current_layer + depth``.
  An expert already GPU-resident or already requested is skipped; a request
  the scheduler does not accept (``REJECTED``) is not remembered, so it can be
  asked for again later.  Requests go out at ``TransferPriority.LOW`` through
  ``TransferScheduler.submit_async`` (a copy on the copy stream that overlaps
  the layers still computing);
* ``cancel_stale(current_layer)`` forgets every request for a layer below
  ``current_layer`` and asks the scheduler to cancel it (a copy already on the
  wire still lands; the scheduler frees its slot when it does);
* ``on_layer_complete(layer_id, expert_indices)`` = ``cancel_stale(layer_id + 1)``
  then ``schedule_prefetch(layer_id, expert_indices)``.

Unlike the reference engine, this package's engine calls
``on_layer_complete`` after each offloaded MoE layer, and ``MoELayer`` adopts a
prefetched copy (waits on its copy event) instead of transferring again.
"""
from __future__ import annotations

import logging
import time
import uuid
from typing import Optional

import torch

from moeinfra_b200.engine.types import PrefetchPolicy
from moeinfra_b200.transfer.types import (
    TransferDirection, TransferPriority, TransferRequest, TransferStatus,
)


class PrefetchEngine:
    """Requests the experts of upcoming layers ahead of their use."""

    def __init__(self, cache_manager, transfer_scheduler, policy: PrefetchPolicy, depth: int,
                 logger: Optional[logging.Logger] = None) -> None:
        self._cache_manager = cache_manager
        self._transfer_scheduler = transfer_scheduler
        self.policy = policy
        self.depth = depth
        self._logger = logger or logging.getLogger(__name__)
        self._in_flight: dict[tuple[int, int], str] = {}
        self.submitted = 0  # requests the scheduler accepted, over the engine's life

    @staticmethod
    def _unique(expert_indices) -> list[int]:
        if isinstance(expert_indices, torch.Tensor):
            return sorted({int(v) for v in expert_indices.reshape(-1).tolist()})
        return sorted({int(v) for v in expert_indices})

    def _targets(self, current_layer: int) -> list[int]:
        if self.policy == PrefetchPolicy.NEXT_LAYER:
            return [current_layer + 1]
        if self.policy == PrefetchPolicy.LOOKAHEAD:
            return [current_layer + d for d in range(1, self.depth + 1)]
        return []

    def _request(self, layer_id: int, expert_id: int) -> Optional[str]:
        key = (layer_id, expert_id)
        if key in self._in_flight or self._cache_manager.is_gpu_resident(layer_id, expert_id):
            return None
        rid = f"prefetch-{layer_id}-{expert_id}-{uuid.uuid4().hex[:12]}"
        handle = self._transfer_scheduler.submit_async(TransferRequest(
            request_id=rid, layer_id=layer_id, expert_id=expert_id,
            direction=TransferDirection.CPU_TO_GPU, priority=TransferPriority.LOW,
            issued_at=time.monotonic()))
        if handle.status != TransferStatus.IN_FLIGHT:
            return None
        self._in_flight[key] = handle.request_id
        self.submitted += 1
        return handle.request_id

    def schedule_prefetch(self, current_layer: int, expert_indices) -> list[str]:
        """Request the predicted experts of the upcoming layer(s); returns the new request ids."""
        targets = self._targets(current_layer)
        if not targets:
            return []
        experts = self._unique(expert_indices)
        out = []
        for layer in targets:
            for e in experts:
                rid = self._request(layer, e)
                if rid is not None:
                    out.append(rid)
        return out

    def cancel_stale(self, current_layer: int) -> int:
        """Drop (and cancel) requests for layers below ``current_layer``; returns cancellations."""
        stale = [k for k in self._in_flight if k[0] < current_layer]
        cancelled = 0
        for key in stale:
            rid = self._in_flight.pop(key)
            if self._transfer_scheduler.cancel(rid):
                cancelled += 1
        return cancelled

    def on_layer_complete(self, layer_id: int, expert_indices) -> None:
        self.cancel_stale(layer_id + 1)
        self.schedule_prefetch(layer_id, expert_indices)

    def forget(self, layer_id: int, expert_id: int) -> None:
        """The layer consumed (or adopted) this prefetch: stop tracking it."""
        self._in_flight.pop((layer_id, expert_id), None)

    @property
    def in_flight(self) -> dict:
        return dict(self._in_flight)
