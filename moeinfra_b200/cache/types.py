"""Cache types (API of the reference's ``cache/types.py``)."""
from __future__ import annotations

import dataclasses
import enum
import time
from typing import Any, Optional


class EvictionPolicy(enum.Enum):
    """Cache eviction strategy: least-recently used, least-frequently used, ARC."""

    LRU = "lru"
    LFU = "lfu"
    ARC = "arc"


@dataclasses.dataclass
class CacheEntry:
    """One cached expert in either tier."""

    expert_id: int
    layer_id: int
    device: str
    expert: Optional[Any]
    last_access: float
    access_count: int
    size_bytes: int

    @property
    def is_on_gpu(self) -> bool:
        return self.device.startswith("cuda")

    @property
    def age(self) -> float:
        return time.monotonic() - self.last_access


@dataclasses.dataclass
class CacheStats:
    """Counters of a :class:`~moeinfra_b200.cache.manager.CacheManager`."""

    hits: int = 0
    misses: int = 0
    evictions: int = 0
    gpu_slots_used: int = 0
    cpu_slots_used: int = 0

    @property
    def hit_rate(self) -> float:
        total = self.hits + self.misses
        return self.hits / total if total > 0 else 0.0
