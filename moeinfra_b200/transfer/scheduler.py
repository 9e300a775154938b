"""Priority scheduler of expert residency transfers.

API of the reference's ``transfer/scheduler.py`` (``TransferScheduler``,
``:35-628``): ``submit`` (dedupe + priority heap), ``execute_next`` (one
synchronous-API transfer with a per-stage profile appended to
``EXECUTE_NEXT_PROFILE``), ``drain``, ``cancel``, ``pending_count``,
``bandwidth_monitor``, ``submit_async`` / ``poll_async`` (event-gated
handles; a cancelled DMA keeps its slot until the copy finishes, ``:584-595``).

B200 change on the CPU->GPU path: the reference blocks the host on
``transfer_stream.synchronize()`` (``:279``) before building the expert.  Here
the copy stream records an event and the compute stream waits on it on the
device, so the host returns immediately and the copy overlaps whatever the
GPU is still executing; pass ``synchronous=True`` to restore the blocking
behaviour (and CUDA-event timing of the copy in the profile).
"""
from __future__ import annotations

import heapq
import logging
import time
from typing import Optional

import torch

from moeinfra_b200.transfer.bandwidth import BandwidthMonitor
from moeinfra_b200.transfer.nf4_reconstruct import ReconstructedNF4Expert
from moeinfra_b200.transfer.nf4_transfer import (
    transfer_pinned_expert_to_gpu, transfer_staged_expert_to_gpu,
)
from moeinfra_b200.transfer.types import (
    TransferDirection, TransferHandle, TransferRequest, TransferResult, TransferStatus,
)

EXECUTE_NEXT_PROFILE: list[dict] = []


class TransferScheduler:
    """Priority-queue scheduler for expert residency transfers."""

    def __init__(self, cache_manager, bandwidth_gbps: float, max_concurrent: int,
                 staging_pool=None, transfer_stream=None,
                 logger: Optional[logging.Logger] = None, synchronous: bool = False) -> None:
        if max_concurrent <= 0:
            raise ValueError("max_concurrent must be positive")
        self._cache_manager = cache_manager
        self.bandwidth_gbps = bandwidth_gbps
        self.max_concurrent = max_concurrent
        self._logger = logger or logging.getLogger(__name__)
        self._bw_monitor = BandwidthMonitor(window_s=5.0)
        self._heap: list[tuple[tuple[int, float, int], TransferRequest]] = []
        self._queue: list[TransferRequest] = []
        self._in_flight: list[TransferRequest] = []
        self._staging_pool = staging_pool
        self._transfer_stream = transfer_stream
        self._async_in_flight: dict[tuple[int, int], TransferHandle] = {}
        self._seq = 0
        self.synchronous = synchronous

    # -- queueing ------------------------------------------------------------
    def _is_duplicate(self, request: TransferRequest) -> bool:
        triple = (request.layer_id, request.expert_id, request.direction)
        for other in (*self._queue, *self._in_flight):
            if other.request_id == request.request_id:
                return True
            if (other.layer_id, other.expert_id, other.direction) == triple:
                return True
        return (request.layer_id, request.expert_id) in self._async_in_flight

    def _key(self, request: TransferRequest) -> tuple[int, float, int]:
        self._seq += 1
        return (request.priority.value, request.issued_at, self._seq)

    def submit(self, request: TransferRequest) -> bool:
        """Queue ``request`` unless an equivalent one is queued or executing."""
        if self._is_duplicate(request):
            return False
        heapq.heappush(self._heap, (self._key(request), request))
        self._queue.append(request)
        return True

    def pending_count(self) -> int:
        return len(self._queue)

    @property
    def bandwidth_monitor(self) -> BandwidthMonitor:
        return self._bw_monitor

    # -- synchronous-API execution ------------------------------------------
    def _copy_pinned(self, cpu_expert, profile: dict):
        """The CPU copy already lives in a pinned slab: one H2D copy, no staging."""
        start = torch.cuda.Event(enable_timing=True) if self.synchronous else None
        if start is not None:
            start.record(self._transfer_stream)
        profile["staging_ms"] = 0.0
        gpu_state = transfer_pinned_expert_to_gpu(cpu_expert, self._transfer_stream)
        done = torch.cuda.Event(enable_timing=self.synchronous)
        done.record(self._transfer_stream)
        if self.synchronous:
            self._transfer_stream.synchronize()
            profile["h2d_cuda_ms"] = start.elapsed_time(done)
        else:
            torch.cuda.current_stream().wait_event(done)
        return gpu_state

    def _stage_and_copy(self, cpu_expert, request: TransferRequest, profile: dict):
        """Stage into a pinned slab, one H2D copy; returns the device state."""
        if getattr(cpu_expert, "pinned_slab", None) is not None:
            return self._copy_pinned(cpu_expert, profile)
        slot = self._staging_pool.acquire(wait=True)
        if slot is None:
            raise RuntimeError("No staging slot available for synchronous transfer")
        try:
            t = time.perf_counter()
            self._staging_pool.stage_expert(slot, cpu_expert, request.layer_id, request.expert_id)
            profile["staging_ms"] = (time.perf_counter() - t) * 1e3
            start = torch.cuda.Event(enable_timing=True) if self.synchronous else None
            if start is not None:
                start.record(self._transfer_stream)
            gpu_state = transfer_staged_expert_to_gpu(slot, self._transfer_stream)
            done = torch.cuda.Event(enable_timing=self.synchronous)
            done.record(self._transfer_stream)
            if self.synchronous:
                t = time.perf_counter()
                self._transfer_stream.synchronize()
                profile["h2d_wall_ms"] = (time.perf_counter() - t) * 1e3
                profile["h2d_cuda_ms"] = start.elapsed_time(done)
            else:
                torch.cuda.current_stream().wait_event(done)
            self._staging_pool.mark_transfer_complete(slot, self._transfer_stream)
            return gpu_state
        finally:
            self._staging_pool.release(slot)

    def execute_next(self) -> Optional[TransferResult]:
        """Execute the highest-priority pending transfer (per-stage profile recorded)."""
        if not self._heap:
            return None
        _, request = heapq.heappop(self._heap)
        self._queue.remove(request)
        self._in_flight.append(request)
        started = time.perf_counter()
        nbytes = 0
        error: Optional[str] = None
        success = False
        profile = {"layer_id": request.layer_id, "expert_id": request.expert_id,
                   "direction": request.direction.value}
        try:
            t = time.perf_counter()
            nbytes = self._cache_manager.get_size_bytes(request.layer_id, request.expert_id)
            profile["metadata_lookup_ms"] = (time.perf_counter() - t) * 1e3
            if request.direction == TransferDirection.CPU_TO_GPU:
                if self._staging_pool is None or self._transfer_stream is None:
                    raise RuntimeError(
                        "Synchronous CPU_TO_GPU transfer requires staging_pool and transfer_stream")
                cpu_expert = self._cache_manager.peek_cpu(request.layer_id, request.expert_id)
                if cpu_expert is None:
                    raise RuntimeError(f"CPU expert not found in cache: layer={request.layer_id}, "
                                       f"expert={request.expert_id}")
                gpu_state = self._stage_and_copy(cpu_expert, request, profile)
                t = time.perf_counter()
                gpu_expert = ReconstructedNF4Expert(cpu_expert, gpu_state)
                profile["reconstruction_call_ms"] = (time.perf_counter() - t) * 1e3
                t = time.perf_counter()
                self._cache_manager.put(request.layer_id, request.expert_id, gpu_expert,
                                        device=f"cuda:{torch.cuda.current_device()}")
                profile["cache_put_call_ms"] = (time.perf_counter() - t) * 1e3
                success = True
            elif request.direction == TransferDirection.GPU_TO_CPU:
                t = time.perf_counter()
                success = self._cache_manager.demote_to_cpu(request.layer_id, request.expert_id)
                profile["demotion_ms"] = (time.perf_counter() - t) * 1e3
            else:
                raise ValueError(f"Unsupported transfer direction: {request.direction!r}")
            if not success:
                error = (f"Transfer failed for layer={request.layer_id}, expert={request.expert_id}, "
                         f"direction={request.direction.value}")
        except Exception as exc:  # errors cross the scheduler as values (reference :363-370)
            error = str(exc)
            self._logger.error("execute_next: FAILED id=%s error=%s", request.request_id, error)
        elapsed_ms = (time.perf_counter() - started) * 1e3
        profile.update(total_execute_next_ms=elapsed_ms, success=success,
                       bytes_transferred=nbytes if success else 0)
        EXECUTE_NEXT_PROFILE.append(profile)
        self._in_flight.remove(request)
        if success:
            self._bw_monitor.record(nbytes)
        return TransferResult(request_id=request.request_id, success=success, elapsed_ms=elapsed_ms,
                              bytes_transferred=nbytes if success else 0, error=error)

    def drain(self) -> list[TransferResult]:
        results = []
        while self._heap:
            r = self.execute_next()
            if r is not None:
                results.append(r)
        return results

    def cancel(self, request_id: str) -> bool:
        """Cancel queued work, or mark an in-flight async copy cancelled (DMA runs to completion)."""
        target = next((r for r in self._queue if r.request_id == request_id), None)
        if target is not None:
            self._queue.remove(target)
            self._heap = [(k, r) for k, r in self._heap if r is not target]
            heapq.heapify(self._heap)
            return True
        handle = next((h for h in self._async_in_flight.values() if h.request_id == request_id), None)
        if handle is None or handle.status != TransferStatus.IN_FLIGHT:
            return False
        handle.status = TransferStatus.CANCELLED
        return True

    def __repr__(self) -> str:
        return (f"TransferScheduler(pending={len(self._queue)}, in_flight={len(self._in_flight)}, "
                f"bandwidth={self.bandwidth_gbps:.1f} GB/s)")

    # -- asynchronous API ------------------------------------------------------
    def _handle(self, request: TransferRequest, status: TransferStatus, slot=None, event=None):
        return TransferHandle(request_id=request.request_id, layer_id=request.layer_id,
                              expert_id=request.expert_id, slot=slot, event=event, status=status)

    def _release_slot(self, slot) -> None:
        """Hand a staging slot back once its copy (queued on the copy stream) is done."""
        if slot is not None:
            self._staging_pool.mark_transfer_complete(slot, self._transfer_stream)
            self._staging_pool.release(slot)

    def _reap_cancelled(self) -> None:
        """Free the slots of cancelled copies that have landed."""
        for key, h in list(self._async_in_flight.items()):
            if h.status == TransferStatus.CANCELLED and h.event.query():
                self._release_slot(h.slot)
                del self._async_in_flight[key]

    def submit_async(self, request: TransferRequest) -> TransferHandle:
        """Start a CPU->GPU copy; the handle becomes READY through :meth:`poll_async`.

        A copy of the same expert that was cancelled but is still registered
        is revived (its bytes land regardless) instead of copied again.
        """
        if request.direction != TransferDirection.CPU_TO_GPU:
            raise ValueError("submit_async() only supports CPU_TO_GPU transfers")
        key = (request.layer_id, request.expert_id)
        if self._cache_manager.is_gpu_resident(*key):
            return self._handle(request, TransferStatus.READY)
        existing = self._async_in_flight.get(key)
        if existing is not None:
            if existing.status == TransferStatus.CANCELLED:
                existing.status = TransferStatus.IN_FLIGHT
            return existing
        if self._staging_pool is not None and self._transfer_stream is not None:
            self._reap_cancelled()
        if len(self._async_in_flight) >= self.max_concurrent:
            return self._handle(request, TransferStatus.REJECTED)
        if self._staging_pool is None or self._transfer_stream is None:
            raise RuntimeError("Async transfer requires staging_pool and transfer_stream")
        expert = self._cache_manager.peek_cpu(*key)
        if expert is None:
            return self._handle(request, TransferStatus.REJECTED)
        slot = None
        if getattr(expert, "pinned_slab", None) is not None:
            gpu_state = transfer_pinned_expert_to_gpu(expert, self._transfer_stream)
            event = torch.cuda.Event()
            event.record(self._transfer_stream)
        else:
            slot = self._staging_pool.acquire()
            if slot is None:
                return self._handle(request, TransferStatus.REJECTED)
            try:
                self._staging_pool.stage_expert(slot, expert, *key)
                gpu_state = transfer_staged_expert_to_gpu(slot, self._transfer_stream)
                event = torch.cuda.Event()
                event.record(self._transfer_stream)
            except Exception:
                self._staging_pool.release(slot)
                raise
        handle = self._handle(request, TransferStatus.IN_FLIGHT, slot=slot, event=event)
        handle.gpu_state = gpu_state
        handle.cpu_expert = expert
        self._async_in_flight[key] = handle
        return handle

    def adopt_async(self, layer_id: int, expert_id: int):
        """Take over an asynchronous copy now; returns the GPU expert or ``None``.

        The caller needs the expert before the copy has been polled complete:
        the current stream waits on the copy's event (no host wait), the expert
        is reconstructed and cached as :meth:`poll_async` would.  A copy that
        was cancelled but not yet reaped is taken too.  ``None`` when no copy
        of this expert is registered.
        """
        key = (layer_id, expert_id)
        handle = self._async_in_flight.get(key)
        # A cancelled copy still lands: its bytes are as good as a new copy's.
        if handle is None or handle.status not in (TransferStatus.IN_FLIGHT,
                                                   TransferStatus.CANCELLED):
            return None
        torch.cuda.current_stream().wait_event(handle.event)
        try:
            expert = ReconstructedNF4Expert(handle.cpu_expert, handle.gpu_state)
            self._cache_manager.put(layer_id, expert_id, expert,
                                    device=f"cuda:{torch.cuda.current_device()}")
            handle.status = TransferStatus.READY
            self._bw_monitor.record(self._cache_manager.get_size_bytes(layer_id, expert_id))
            return expert
        finally:
            self._release_slot(handle.slot)
            del self._async_in_flight[key]

    def poll_async(self, layer_id: int, expert_id: int) -> TransferStatus:
        key = (layer_id, expert_id)
        handle = self._async_in_flight.get(key)
        if handle is None:
            return TransferStatus.REJECTED
        done = handle.event.query()
        if handle.status == TransferStatus.CANCELLED:
            if not done:
                return TransferStatus.CANCELLED
            self._release_slot(handle.slot)
            del self._async_in_flight[key]
            return TransferStatus.CANCELLED
        if not done:
            return TransferStatus.IN_FLIGHT
        try:
            expert = ReconstructedNF4Expert(handle.cpu_expert, handle.gpu_state)
            self._cache_manager.put(layer_id, expert_id, expert, device="cuda")
            handle.status = TransferStatus.READY
            self._release_slot(handle.slot)
            del self._async_in_flight[key]
            return TransferStatus.READY
        except Exception:
            handle.status = TransferStatus.REJECTED
            if handle.slot is not None:
                self._staging_pool.release(handle.slot)
            del self._async_in_flight[key]
            raise
