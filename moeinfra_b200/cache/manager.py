"""Two-tier (GPU + CPU) expert residency cache.

API of the reference's ``cache/manager.py`` (``CacheManager``, ``:122-508``):
``get / put / evict / promote_to_gpu / demote_to_cpu / get_size_bytes / stats /
is_gpu_resident / peek_cpu / peek_gpu``, keyed by ``(layer_id, expert_id)``.
The CPU tier is authoritative (serialized NF4); GPU entries are disposable
device copies, so GPU eviction and demotion only drop the device copy
(``:369-373``, ``:420-451``).  Single-threaded by design, like the reference.

Eviction: LRU (oldest ``last_access``, first-inserted on ties), LFU (lowest
``access_count``, then LRU), ARC (recency list T1, frequency list T2, ghost
lists B1/B2 and the adaptive target ``p``).  Additions over the reference:
an optional byte budget for the GPU tier (``gpu_budget_bytes``), and ARC
registers newly inserted keys in T1 so the ARC-managed GPU tier stays bounded.
"""
from __future__ import annotations

import logging
import time
from typing import Any, Optional

from moeinfra_b200.cache.types import CacheEntry, CacheStats, EvictionPolicy

Key = tuple[int, int]


class _ArcLists:
    """ARC bookkeeping for one tier (T1 recency, T2 frequency, B1/B2 ghosts)."""

    def __init__(self, capacity: int) -> None:
        self.capacity = capacity
        self.p = 0
        self.t1: list[Key] = []
        self.t2: list[Key] = []
        self.b1: list[Key] = []
        self.b2: list[Key] = []

    def hit(self, key: Key) -> None:
        if key in self.t1:
            self.t1.remove(key)
            self.t2.append(key)
        elif key in self.t2:
            self.t2.remove(key)
            self.t2.append(key)

    def admit(self, key: Key) -> None:
        """A key (re)enters the cache: adapt ``p`` on ghost hits, then join T1."""
        if key in self.b1:
            self.p = min(self.capacity, self.p + max(1, len(self.b2) // max(1, len(self.b1))))
            self.b1.remove(key)
        elif key in self.b2:
            self.p = max(0, self.p - max(1, len(self.b1) // max(1, len(self.b2))))
            self.b2.remove(key)
        if key not in self.t1 and key not in self.t2:
            self.t1.append(key)
        del self.b1[:max(0, len(self.b1) - self.capacity)]
        del self.b2[:max(0, len(self.b2) - self.capacity)]

    def victim(self) -> Optional[Key]:
        if not self.t1 and not self.t2:
            return None
        if self.t1 and (len(self.t1) > self.p or not self.t2):
            key = self.t1.pop(0)
            self.b1.append(key)
        else:
            key = self.t2.pop(0)
            self.b2.append(key)
        return key

    def drop(self, key: Key) -> None:
        for lst in (self.t1, self.t2):
            if key in lst:
                lst.remove(key)


def _is_gpu(device: str) -> bool:
    return device.startswith(("cuda", "gpu"))


class CacheManager:
    """Two-level LRU/LFU/ARC expert cache (GPU slots + CPU slots)."""

    def __init__(self, gpu_slots: int, cpu_slots: int, policy: EvictionPolicy,
                 logger: Optional[logging.Logger] = None,
                 gpu_budget_bytes: Optional[int] = None) -> None:
        self.gpu_slots = gpu_slots
        self.cpu_slots = cpu_slots
        self.policy = policy
        self.gpu_budget_bytes = gpu_budget_bytes
        self._gpu_cache: dict[Key, CacheEntry] = {}
        self._cpu_cache: dict[Key, CacheEntry] = {}
        self._stats = CacheStats()
        self._logger = logger or logging.getLogger(__name__)
        self._arc = {True: _ArcLists(gpu_slots), False: _ArcLists(cpu_slots)}

    # -- helpers -----------------------------------------------------------
    def _tier(self, device: str) -> dict[Key, CacheEntry]:
        return self._gpu_cache if _is_gpu(device) else self._cpu_cache

    def _sync_counts(self) -> None:
        self._stats.gpu_slots_used = len(self._gpu_cache)
        self._stats.cpu_slots_used = len(self._cpu_cache)

    def _touch(self, key: Key, entry: CacheEntry) -> None:
        entry.last_access = time.monotonic()
        entry.access_count += 1
        if self.policy == EvictionPolicy.ARC:
            self._arc[_is_gpu(entry.device)].hit(key)

    def gpu_bytes(self) -> int:
        return sum(e.size_bytes for e in self._gpu_cache.values())

    # -- public API --------------------------------------------------------
    def get(self, layer_id: int, expert_id: int) -> Optional[Any]:
        """GPU tier first, then CPU; a hit refreshes recency/frequency."""
        key = (layer_id, expert_id)
        for tier in (self._gpu_cache, self._cpu_cache):
            entry = tier.get(key)
            if entry is not None:
                self._touch(key, entry)
                self._stats.hits += 1
                return entry.expert
        # ARC adapts its target on the (re)insertion that follows a miss (put).
        self._stats.misses += 1
        return None

    def put(self, layer_id: int, expert_id: int, expert: Any, device: str) -> None:
        """Insert or refresh; evicts from a full tier first."""
        key = (layer_id, expert_id)
        tier = self._tier(device)
        gpu = _is_gpu(device)
        entry = tier.get(key)
        if entry is not None:
            entry.expert = expert
            entry.device = device
            self._touch(key, entry)
            return
        limit = self.gpu_slots if gpu else self.cpu_slots
        if len(tier) >= limit and self.evict(device) is None:
            self._logger.warning("put: tier full but nothing evictable (layer=%d expert=%d %s)",
                                 layer_id, expert_id, device)
        size = int(getattr(expert, "size_bytes", 0))
        if gpu and self.gpu_budget_bytes is not None:
            while self._gpu_cache and self.gpu_bytes() + size > self.gpu_budget_bytes:
                if self.evict(device) is None:
                    break
        tier[key] = CacheEntry(expert_id=expert_id, layer_id=layer_id, device=device,
                               expert=expert, last_access=time.monotonic(), access_count=1,
                               size_bytes=size)
        if self.policy == EvictionPolicy.ARC:
            self._arc[gpu].admit(key)
        self._sync_counts()

    def evict(self, device: str) -> Optional[CacheEntry]:
        """Remove one entry of the tier chosen by the policy; ``None`` if empty."""
        tier = self._tier(device)
        if not tier:
            return None
        gpu = _is_gpu(device)
        if self.policy == EvictionPolicy.LFU:
            key = min(tier, key=lambda k: (tier[k].access_count, tier[k].last_access))
        elif self.policy == EvictionPolicy.ARC:
            key = self._arc[gpu].victim()
            if key is None or key not in tier:
                key = min(tier, key=lambda k: tier[k].last_access)
        else:
            key = min(tier, key=lambda k: tier[k].last_access)
        entry = tier.pop(key)
        if gpu:
            entry.device = "cuda"
        if self.policy == EvictionPolicy.ARC:
            self._arc[gpu].drop(key)
        self._stats.evictions += 1
        self._sync_counts()
        return entry

    def promote_to_gpu(self, layer_id: int, expert_id: int) -> bool:
        """GPU residency is created by the transfer scheduler; True if already resident."""
        return self.is_gpu_resident(layer_id, expert_id)

    def demote_to_cpu(self, layer_id: int, expert_id: int) -> bool:
        """Drop the disposable GPU copy; the CPU backing copy is untouched."""
        key = (layer_id, expert_id)
        entry = self._gpu_cache.pop(key, None)
        if entry is None:
            return False
        if self.policy == EvictionPolicy.ARC:
            self._arc[True].drop(key)
        self._sync_counts()
        return True

    def get_size_bytes(self, layer_id: int, expert_id: int) -> int:
        key = (layer_id, expert_id)
        entry = self._gpu_cache.get(key) or self._cpu_cache.get(key)
        if entry is None:
            raise KeyError(f"Expert not present in cache: layer={layer_id}, expert={expert_id}")
        return entry.size_bytes

    def stats(self) -> CacheStats:
        return self._stats

    def is_gpu_resident(self, layer_id: int, expert_id: int) -> bool:
        return (layer_id, expert_id) in self._gpu_cache

    def peek_cpu(self, layer_id: int, expert_id: int) -> Optional[Any]:
        entry = self._cpu_cache.get((layer_id, expert_id))
        return None if entry is None else entry.expert

    def peek_gpu(self, layer_id: int, expert_id: int) -> Optional[Any]:
        entry = self._gpu_cache.get((layer_id, expert_id))
        return None if entry is None else entry.expert

    def __repr__(self) -> str:
        return (f"CacheManager(gpu={len(self._gpu_cache)}/{self.gpu_slots}, "
                f"cpu={len(self._cpu_cache)}/{self.cpu_slots}, policy={self.policy.value})")
