"""CPU contract of ``CacheManager`` (the reference's ``cache/manager.py`` API).

The checks follow what the reference's ``tests/test_cache.py`` pins for the
two-tier residency cache: slot accounting, hit/miss/eviction statistics,
LRU / LFU victim choice (LFU ties broken by recency), the ``"gpu"`` alias of
the device tier, ``get_size_bytes`` without side effects, and the
CPU-authoritative model in which ``promote_to_gpu`` only reports residency
(the transfer scheduler creates GPU copies) and ``demote_to_cpu`` drops the
GPU copy while the CPU copy stays (``cache/manager.py:390-451``).  ARC and the
optional GPU byte budget are additions of this package and are checked for
boundedness.
"""
from __future__ import annotations

import time

import pytest

from moeinfra_b200.cache.manager import CacheManager
from moeinfra_b200.cache.types import CacheEntry, CacheStats, EvictionPolicy


class Stub:
    """Stand-in expert: the cache only reads ``size_bytes``."""

    def __init__(self, size_bytes: int = 1000, tag: str = "") -> None:
        self.size_bytes = size_bytes
        self.tag = tag


def lru(gpu: int = 2, cpu: int = 4) -> CacheManager:
    return CacheManager(gpu_slots=gpu, cpu_slots=cpu, policy=EvictionPolicy.LRU)


def lfu(gpu: int = 2, cpu: int = 4) -> CacheManager:
    return CacheManager(gpu_slots=gpu, cpu_slots=cpu, policy=EvictionPolicy.LFU)


# -- construction, entries, stats --------------------------------------------------

def test_construction_records_slots_policy_and_zero_stats():
    cm = CacheManager(gpu_slots=4, cpu_slots=8, policy=EvictionPolicy.LRU)
    assert (cm.gpu_slots, cm.cpu_slots, cm.policy) == (4, 8, EvictionPolicy.LRU)
    text = repr(cm)
    assert "CacheManager" in text and "gpu=" in text and "cpu=" in text
    s = cm.stats()
    assert (s.hits, s.misses, s.evictions, s.gpu_slots_used, s.cpu_slots_used) == (0, 0, 0, 0, 0)
    assert s.hit_rate == 0.0
    assert cm.stats() is s  # the same object, updated in place


def test_cache_entry_device_and_age():
    now = time.monotonic()
    e_cpu = CacheEntry(expert_id=1, layer_id=2, device="cpu", expert=Stub(), last_access=now,
                       access_count=1, size_bytes=10)
    e_gpu = CacheEntry(expert_id=1, layer_id=2, device="cuda:0", expert=Stub(), last_access=now,
                       access_count=1, size_bytes=10)
    assert not e_cpu.is_on_gpu and e_gpu.is_on_gpu
    a0 = e_cpu.age
    time.sleep(0.01)
    assert e_cpu.age > a0


def test_hit_rate_arithmetic():
    assert CacheStats(hits=3, misses=1).hit_rate == pytest.approx(0.75)
    assert CacheStats(hits=5, misses=0).hit_rate == 1.0
    assert CacheStats().hit_rate == 0.0


# -- put / get -----------------------------------------------------------------------

def test_put_get_hit_and_miss_counting():
    cm = lru()
    ex = Stub()
    cm.put(0, 0, ex, "cpu")
    assert cm.stats().cpu_slots_used == 1
    assert cm.get(0, 0) is ex
    assert cm.get(0, 1) is None
    assert cm.get(7, 7) is None
    s = cm.stats()
    assert (s.hits, s.misses) == (1, 2)
    assert s.hit_rate == pytest.approx(1 / 3)


def test_put_of_an_existing_key_refreshes_in_place():
    cm = lru()
    cm.put(0, 0, Stub(tag="a"), "cpu")
    newer = Stub(tag="b")
    cm.put(0, 0, newer, "cpu")
    assert cm.stats().cpu_slots_used == 1
    assert cm.get(0, 0) is newer


def test_gpu_tier_wins_over_cpu_tier():
    cm = lru()
    cpu_copy, gpu_copy = Stub(tag="cpu"), Stub(tag="gpu")
    cm.put(3, 1, cpu_copy, "cpu")
    cm.put(3, 1, gpu_copy, "cuda:0")
    assert cm.get(3, 1) is gpu_copy
    assert cm.peek_cpu(3, 1) is cpu_copy
    assert cm.peek_gpu(3, 1) is gpu_copy
    assert cm.is_gpu_resident(3, 1)
    assert cm.stats().gpu_slots_used == 1 and cm.stats().cpu_slots_used == 1


def test_peek_does_not_touch_statistics():
    cm = lru()
    cm.put(0, 0, Stub(), "cpu")
    cm.peek_cpu(0, 0)
    cm.peek_gpu(0, 0)
    assert (cm.stats().hits, cm.stats().misses) == (0, 0)


# -- eviction -------------------------------------------------------------------------

def test_evict_on_an_empty_tier_returns_none():
    assert lru().evict("cpu") is None
    assert lru().evict("cuda") is None


def test_evict_removes_one_entry_and_counts_it():
    cm = lru()
    cm.put(0, 0, Stub(), "cpu")
    cm.put(0, 1, Stub(), "cpu")
    victim = cm.evict("cpu")
    assert victim is not None and victim.device == "cpu"
    assert cm.stats().cpu_slots_used == 1
    assert cm.stats().evictions == 1


def test_gpu_alias_evicts_the_device_tier_only():
    cm = CacheManager(gpu_slots=1, cpu_slots=1, policy=EvictionPolicy.LRU)
    cpu_copy, gpu_copy = Stub(), Stub()
    cm.put(0, 0, cpu_copy, "cpu")
    cm.put(0, 0, gpu_copy, "cuda")
    victim = cm.evict("gpu")
    assert victim is not None and victim.expert is gpu_copy
    assert cm.peek_gpu(0, 0) is None
    assert cm.peek_cpu(0, 0) is cpu_copy


def test_lru_victim_is_the_least_recently_used():
    cm = lru(cpu=3)
    for e in range(3):
        cm.put(0, e, Stub(), "cpu")
        time.sleep(0.002)
    cm.get(0, 0)  # (0, 0) becomes the most recent; (0, 1) is now the oldest
    assert cm.evict("cpu").expert_id == 1


def test_full_tier_evicts_once_per_insert_and_stays_at_capacity():
    cm = lru(cpu=2)
    cm.put(0, 0, Stub(), "cpu")
    time.sleep(0.002)
    cm.put(0, 1, Stub(), "cpu")
    cm.get(0, 0)
    cm.put(0, 2, Stub(), "cpu")  # (0, 1) is the LRU entry
    assert cm.stats().evictions == 1
    assert cm.peek_cpu(0, 1) is None
    assert cm.peek_cpu(0, 0) is not None and cm.peek_cpu(0, 2) is not None
    for i in range(3):
        cm.put(1, i, Stub(), "cpu")
    assert cm.stats().evictions == 4
    assert cm.stats().cpu_slots_used == 2


def test_no_eviction_below_capacity():
    cm = lru(cpu=4)
    for i in range(4):
        cm.put(0, i, Stub(), "cpu")
    assert cm.stats().evictions == 0
    assert cm.stats().cpu_slots_used == 4


def test_lfu_victim_is_the_least_frequent_then_least_recent():
    cm = lfu(cpu=3)
    for e in range(3):
        cm.put(0, e, Stub(), "cpu")
        time.sleep(0.002)
    for _ in range(3):
        cm.get(0, 0)
        cm.get(0, 2)
    assert cm.evict("cpu").expert_id == 1
    cm2 = lfu(cpu=3)
    cm2.put(0, 5, Stub(), "cpu")
    time.sleep(0.002)
    cm2.put(0, 6, Stub(), "cpu")
    assert cm2.evict("cpu").expert_id == 5  # equal counts: the older entry goes


def test_manual_evictions_drain_the_tier():
    cm = lru(cpu=3)
    for i in range(3):
        cm.put(0, i, Stub(), "cpu")
    for _ in range(3):
        assert cm.evict("cpu") is not None
    assert cm.stats().cpu_slots_used == 0
    assert cm.stats().evictions == 3
    assert cm.evict("cpu") is None


# -- sizes, promotion, demotion ------------------------------------------------------

def test_get_size_bytes_reads_either_tier_without_side_effects():
    cm = lru()
    cm.put(0, 0, Stub(4096), "cpu")
    cm.put(5, 3, Stub(8192), "cuda:0")
    hits = cm.stats().hits
    assert cm.get_size_bytes(0, 0) == 4096
    assert cm.get_size_bytes(5, 3) == 8192
    assert cm.stats().hits == hits
    with pytest.raises(KeyError, match="Expert not present"):
        cm.get_size_bytes(99, 99)


def test_promote_only_reports_residency():
    cm = lru()
    assert cm.promote_to_gpu(0, 9) is False  # not cached anywhere
    cm.put(0, 0, Stub(), "cpu")
    assert cm.promote_to_gpu(0, 0) is False  # the scheduler makes GPU copies
    assert cm.peek_cpu(0, 0) is not None
    cm.put(0, 0, Stub(), "cuda:0")
    assert cm.promote_to_gpu(0, 0) is True


def test_demote_drops_the_gpu_copy_and_keeps_the_cpu_copy():
    cm = lru()
    assert cm.demote_to_cpu(0, 0) is False
    cpu_copy = Stub()
    cm.put(0, 0, cpu_copy, "cpu")
    cm.put(0, 0, Stub(), "cuda:0")
    assert cm.demote_to_cpu(0, 0) is True
    assert not cm.is_gpu_resident(0, 0)
    assert cm.peek_cpu(0, 0) is cpu_copy
    assert cm.stats().gpu_slots_used == 0 and cm.stats().cpu_slots_used == 1


# -- ARC and the GPU byte budget (this package's additions) -----------------------

def test_arc_keeps_each_tier_within_its_slots_and_protects_frequent_keys():
    cm = CacheManager(gpu_slots=4, cpu_slots=4, policy=EvictionPolicy.ARC)
    for e in range(2):
        cm.put(0, e, Stub(), "cuda:0")
        cm.get(0, e)  # seen twice: the frequency list
    for e in range(2, 40):  # a one-pass scan over many keys
        cm.put(0, e, Stub(), "cuda:0")
        assert cm.stats().gpu_slots_used <= 4
    assert cm.is_gpu_resident(0, 0) and cm.is_gpu_resident(0, 1)


def test_gpu_byte_budget_evicts_until_the_new_entry_fits():
    cm = CacheManager(gpu_slots=100, cpu_slots=10, policy=EvictionPolicy.LRU,
                      gpu_budget_bytes=3000)
    for e in range(3):
        cm.put(0, e, Stub(1000), "cuda:0")
        time.sleep(0.002)
    assert cm.gpu_bytes() == 3000
    cm.put(0, 3, Stub(1500), "cuda:0")
    assert cm.gpu_bytes() <= 3000
    assert not cm.is_gpu_resident(0, 0) and not cm.is_gpu_resident(0, 1)
    assert cm.is_gpu_resident(0, 2) and cm.is_gpu_resident(0, 3)
