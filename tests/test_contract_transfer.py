"""CPU contract of the transfer subsystem (the reference's ``transfer/`` API).

Follows what the reference's ``tests/test_transfer.py``,
``tests/test_reusable_staging.py`` and ``tests/test_pinned_memory.py`` pin:

* ``TransferScheduler``: duplicate suppression (same request id, or same
  (layer, expert, direction) already queued), priority order HIGH < NORMAL <
  LOW with FIFO inside a priority, ``cancel`` of queued work keeping the heap
  ordered, ``execute_next`` / ``drain`` returning ``TransferResult`` values
  (failures as values whose error names the expert; zero bytes on failure),
  the bandwidth monitor fed on success;
* ``BandwidthMonitor``: zero until two samples, peak >= current, reset;
* ``ReusablePinnedStagingPool``: budget-bounded slot creation, release and
  reuse, double release refused, a slot whose copy event has not completed is
  not handed out again, staging copies every canonical tensor (nested state
  included) bit-for-bit into the slot, leaves the source pageable and reuses
  the slot's buffer;
* ``PinnedMemoryBudget``: reservation arithmetic and its error cases.

CPU_TO_GPU execution needs a GPU and is covered by the GPU offload tests.
"""
from __future__ import annotations

import time
import uuid

import pytest
import torch

from moeinfra_b200.transfer.bandwidth import BandwidthMonitor
from moeinfra_b200.transfer.pinned_memory import PinnedMemoryBudget
from moeinfra_b200.transfer.reusable_staging import ReusablePinnedStagingPool, SLAB_ALIGN
from moeinfra_b200.transfer.scheduler import EXECUTE_NEXT_PROFILE, TransferScheduler
from moeinfra_b200.transfer.types import (
    TransferDirection, TransferPriority, TransferRequest, TransferResult, TransferStatus,
)

D2H, H2D = TransferDirection.GPU_TO_CPU, TransferDirection.CPU_TO_GPU


class RecordingCache:
    """Cache double: sizes per key, GPU copies that demotion removes, a call log."""

    def __init__(self) -> None:
        self.sizes: dict = {}
        self.gpu: set = set()
        self.demoted: list = []

    def add(self, layer: int, expert: int, size: int, on_gpu: bool = True) -> None:
        self.sizes[(layer, expert)] = size
        if on_gpu:
            self.gpu.add((layer, expert))

    def get_size_bytes(self, layer: int, expert: int) -> int:
        if (layer, expert) not in self.sizes:
            raise KeyError(f"Expert not present in cache: layer={layer}, expert={expert}")
        return self.sizes[(layer, expert)]

    def demote_to_cpu(self, layer: int, expert: int) -> bool:
        self.demoted.append((layer, expert))
        if (layer, expert) not in self.gpu:
            return False
        self.gpu.discard((layer, expert))
        return True

    def is_gpu_resident(self, layer: int, expert: int) -> bool:
        return (layer, expert) in self.gpu

    def peek_cpu(self, layer: int, expert: int):
        return None


def req(layer=0, expert=0, direction=D2H, priority=TransferPriority.NORMAL, rid=None):
    return TransferRequest(request_id=rid or uuid.uuid4().hex, layer_id=layer, expert_id=expert,
                           direction=direction, priority=priority, issued_at=time.monotonic())


def sched(cache=None, **kw) -> TransferScheduler:
    return TransferScheduler(cache if cache is not None else RecordingCache(),
                             bandwidth_gbps=8.0, max_concurrent=kw.pop("max_concurrent", 4), **kw)


# -- types and the bandwidth monitor ----------------------------------------------------

def test_request_and_result_types():
    r = req(3, 7, direction=H2D)
    assert (r.layer_id, r.expert_id, r.direction, r.priority) == (3, 7, H2D,
                                                                  TransferPriority.NORMAL)
    assert r.issued_at > 0 and isinstance(r.request_id, str)
    assert req().request_id != req().request_id
    assert not hasattr(r, "tensor")  # requests name experts; the cache owns them
    with pytest.raises((AttributeError, TypeError)):
        r.layer_id = 1  # frozen
    ok = TransferResult(request_id="a", success=True, elapsed_ms=1.0, bytes_transferred=10)
    bad = TransferResult(request_id="b", success=False, elapsed_ms=0.5, bytes_transferred=0,
                         error="boom")
    assert ok.error is None and bad.error == "boom" and bad.bytes_transferred == 0


def test_bandwidth_monitor():
    mon = BandwidthMonitor(window_s=5.0)
    assert mon.current_gbps() == 0.0 and mon.peak_gbps() == 0.0
    mon.record(1 << 30)
    assert mon.current_gbps() == 0.0  # one sample is not a rate
    time.sleep(0.01)
    mon.record(1 << 30)
    assert mon.current_gbps() > 0.0
    assert mon.peak_gbps() >= mon.current_gbps() > 0.0
    mon.reset()
    assert mon.current_gbps() == 0.0 and mon.peak_gbps() == 0.0


# -- submit / priority / cancel ------------------------------------------------------------

def test_submit_suppresses_duplicates():
    s = sched()
    assert s.submit(req(0, 0)) is True
    assert s.pending_count() == 1
    assert s.submit(req(0, 0)) is False  # same (layer, expert, direction)
    fixed = uuid.uuid4().hex
    assert s.submit(req(0, 1, rid=fixed)) is True
    assert s.submit(req(0, 2, rid=fixed)) is False  # same request id
    assert s.submit(req(0, 0, direction=H2D)) is True  # other direction: distinct
    assert s.submit(req(0, 3)) is True
    assert s.pending_count() == 4


def _drain_order(s: TransferScheduler) -> list:
    return [r.request_id for r in s.drain()]


def test_priority_order_and_fifo_within_a_priority():
    cache = RecordingCache()
    for e in range(6):
        cache.add(0, e, 100)
    s = sched(cache)
    s.submit(req(0, 0, priority=TransferPriority.LOW, rid="low"))
    s.submit(req(0, 1, priority=TransferPriority.NORMAL, rid="n1"))
    s.submit(req(0, 2, priority=TransferPriority.HIGH, rid="high"))
    s.submit(req(0, 3, priority=TransferPriority.NORMAL, rid="n2"))
    s.submit(req(0, 4, priority=TransferPriority.NORMAL, rid="n3"))
    assert _drain_order(s) == ["high", "n1", "n2", "n3", "low"]
    assert s.pending_count() == 0


def test_cancel_removes_only_the_named_request_and_keeps_order():
    cache = RecordingCache()
    for e in range(5):
        cache.add(0, e, 100)
    s = sched(cache)
    for e, p in enumerate([TransferPriority.LOW, TransferPriority.HIGH, TransferPriority.NORMAL,
                           TransferPriority.HIGH, TransferPriority.NORMAL]):
        s.submit(req(0, e, priority=p, rid=f"r{e}"))
    assert s.cancel("r1") is True
    assert s.pending_count() == 4
    assert s.cancel("r1") is False
    assert s.cancel("unknown") is False
    assert _drain_order(s) == ["r3", "r2", "r4", "r0"]


# -- execute_next / drain -------------------------------------------------------------------

def test_execute_next_on_an_empty_queue():
    assert sched().execute_next() is None
    assert sched().drain() == []


def test_gpu_to_cpu_demotes_and_reports_the_bytes():
    cache = RecordingCache()
    cache.add(1, 3, 4096)
    s = sched(cache)
    r = req(1, 3)
    s.submit(r)
    before = len(EXECUTE_NEXT_PROFILE)
    result = s.execute_next()
    assert cache.demoted == [(1, 3)]
    assert result.success and result.bytes_transferred == 4096
    assert result.request_id == r.request_id
    assert result.elapsed_ms >= 0.0
    assert s.pending_count() == 0
    assert len(EXECUTE_NEXT_PROFILE) == before + 1
    assert EXECUTE_NEXT_PROFILE[-1]["success"] is True


def test_failures_are_values_with_zero_bytes():
    cache = RecordingCache()
    cache.add(0, 0, 1024, on_gpu=False)  # known size, but nothing to demote
    s = sched(cache)
    s.submit(req(0, 0))
    r1 = s.execute_next()
    assert not r1.success and r1.bytes_transferred == 0 and r1.error
    s.submit(req(9, 8))  # not cached at all
    r2 = s.execute_next()
    assert not r2.success and r2.bytes_transferred == 0
    assert "9" in r2.error and "8" in r2.error


def test_cpu_to_gpu_without_a_pinned_pool_fails_as_a_value():
    cache = RecordingCache()
    cache.add(0, 0, 1024, on_gpu=False)
    s = sched(cache)
    s.submit(req(0, 0, direction=H2D))
    r = s.execute_next()
    assert not r.success and "staging_pool" in r.error


def test_drain_runs_everything_and_feeds_the_bandwidth_monitor():
    cache = RecordingCache()
    for e in range(3):
        cache.add(2, e, 1 << 20)
    s = sched(cache)
    for e in range(3):
        s.submit(req(2, e))
        time.sleep(0.002)
    results = s.drain()
    assert len(results) == 3 and all(r.success for r in results)
    assert s.pending_count() == 0
    assert s.bandwidth_monitor.peak_gbps() > 0.0


def test_async_api_rejections_without_a_gpu():
    cache = RecordingCache()
    cache.add(0, 0, 100, on_gpu=True)
    s = sched(cache)
    with pytest.raises(ValueError):
        s.submit_async(req(0, 0, direction=D2H))
    assert s.submit_async(req(0, 0, direction=H2D)).status == TransferStatus.READY
    assert s.poll_async(5, 5) == TransferStatus.REJECTED
    assert "TransferScheduler" in repr(s)


# -- pinned budget ----------------------------------------------------------------------------

def test_pinned_budget_arithmetic():
    b = PinnedMemoryBudget(1000)
    assert (b.budget_bytes, b.used_bytes, b.available_bytes) == (1000, 0, 1000)
    assert b.reserve(300) is True and b.reserve(400) is True
    assert (b.used_bytes, b.available_bytes) == (700, 300)
    assert b.can_reserve(300) and not b.can_reserve(301)
    assert b.used_bytes == 700  # can_reserve changes nothing
    assert b.reserve(301) is False and b.used_bytes == 700
    assert b.reserve(300) is True and b.available_bytes == 0
    assert b.reserve(0) is True
    b.release(1000)
    assert b.used_bytes == 0 and b.peak_bytes == 1000
    b.release(0)
    assert b.reserve(1000) is True
    assert repr(b) == "PinnedMemoryBudget(budget_bytes=1000, used_bytes=1000, available_bytes=0)"


@pytest.mark.parametrize("bad", [-1, -1000])
def test_pinned_budget_rejects_negative_sizes(bad):
    b = PinnedMemoryBudget(100)
    with pytest.raises(ValueError):
        b.reserve(bad)
    with pytest.raises(ValueError):
        b.can_reserve(bad)
    with pytest.raises(ValueError):
        b.release(bad)
    with pytest.raises(ValueError):
        PinnedMemoryBudget(bad)


def test_pinned_budget_underflow_is_an_error():
    b = PinnedMemoryBudget(100)
    with pytest.raises(ValueError):
        b.release(1)
    b.reserve(50)
    with pytest.raises(ValueError):
        b.release(51)
    assert b.used_bytes == 50


# -- reusable staging pool ------------------------------------------------------------------

class FakeEvent:
    """Copy-completion event double: ``query()`` answers what the test sets."""

    def __init__(self, done: bool) -> None:
        self.done = done

    def query(self) -> bool:
        return self.done

    def synchronize(self) -> None:
        self.done = True

    def record(self, stream=None) -> None:
        pass


def test_pool_slots_are_budget_bounded_and_reused():
    budget = PinnedMemoryBudget(3 * 1024)
    pool = ReusablePinnedStagingPool(budget, 1024)
    assert (pool.slot_count, pool.active_slots) == (0, 0)
    a = pool.acquire()
    assert a is not None and a.in_use and pool.slot_count == 1 and budget.used_bytes == 1024
    b, c = pool.acquire(), pool.acquire()
    assert len({a.slot_id, b.slot_id, c.slot_id}) == 3
    assert pool.acquire() is None  # budget exhausted, all slots busy
    pool.release(b)
    assert pool.active_slots == 2
    assert pool.acquire() is b  # the same slot comes back
    pool.release(a)
    with pytest.raises(RuntimeError):
        pool.release(a)  # double release


def test_a_slot_is_not_reused_before_its_copy_completes(monkeypatch):
    pool = ReusablePinnedStagingPool(PinnedMemoryBudget(1024), 1024)
    slot = pool.acquire()
    pool.release(slot)
    with pytest.raises(RuntimeError):
        pool.mark_transfer_complete(slot, None)  # only an acquired slot can carry a copy
    slot = pool.acquire()
    assert slot is not None
    monkeypatch.setattr(torch.cuda, "Event", lambda *a, **k: FakeEvent(False))
    pool.mark_transfer_complete(slot, stream=None)
    pool.release(slot)
    assert pool.acquire() is None  # its copy is still in flight, and no budget is left
    slot.ready_event.done = True
    again = pool.acquire()
    assert again is slot and again.ready_event is None


def _expert_states(nested: bool):
    from moeinfra_b200.model.expert import PrequantizedNF4Expert
    from moeinfra_b200.model.nf4_format import quantize_nf4

    g = torch.Generator().manual_seed(1)
    st = {}
    for name, shape in (("w1", (128, 64)), ("w2", (64, 128)), ("w3", (128, 64))):
        st[name] = quantize_nf4((torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16),
                                compress_statistics=nested)
    return PrequantizedNF4Expert.from_serialized(st["w1"], st["w2"], st["w3"], hidden_size=64,
                                                 intermediate_size=128)


@pytest.mark.parametrize("nested", [False, True])
def test_stage_expert_copies_every_canonical_tensor_exactly(nested):
    from moeinfra_b200.model.nf4_format import canonical_state

    ex = _expert_states(nested)
    pool = ReusablePinnedStagingPool(PinnedMemoryBudget(1 << 20), 1 << 16)
    slot = pool.acquire()
    pool.stage_expert(slot, ex, 4, 2)
    assert slot.expert_key == (4, 2)
    total = 0
    for proj in ("w1", "w2", "w3"):
        want = canonical_state(getattr(ex, proj), proj)
        got = slot.tensors[proj]
        for key, t in want.items():
            if t is None:
                assert got[key] is None
                continue
            assert torch.equal(got[key], t), (proj, key)
            total += t.numel() * t.element_size()
        if nested:
            assert got["state2_absmax"] is not None and got["state2_code"] is not None
    for proj, key, off, shape, dtype in slot.layout:
        assert off is None or off % SLAB_ALIGN == 0
    assert total <= slot.used_bytes <= slot.size_bytes
    assert not ex.w1["weight"].is_pinned()  # the source stays pageable
    slab = slot.slab.data_ptr()
    pool.release(slot)
    again = pool.acquire()
    pool.stage_expert(again, _expert_states(nested), 4, 3)
    assert again.slab.data_ptr() == slab  # the slot's buffer is reused


def test_stage_expert_refuses_an_expert_larger_than_the_slot():
    pool = ReusablePinnedStagingPool(PinnedMemoryBudget(1 << 20), 4096)
    slot = pool.acquire()
    with pytest.raises(ValueError, match="staging bytes"):
        pool.stage_expert(slot, _expert_states(False), 0, 0)


@pytest.mark.parametrize("nested", [False, True])
def test_pin_expert_packs_one_slab_and_rebinds_the_tensors(nested):
    from moeinfra_b200.model.nf4_format import canonical_state
    from moeinfra_b200.transfer.reusable_staging import pin_expert, slab_views

    ex = _expert_states(nested)
    want = {p: {k: (None if v is None else v.clone()) for k, v in
                canonical_state(getattr(ex, p), p).items()} for p in ("w1", "w2", "w3")}
    nbytes = pin_expert(ex)
    assert nbytes == ex.pinned_bytes and pin_expert(ex) == nbytes  # idempotent
    views = slab_views(ex.pinned_slab, ex.pinned_layout)
    for p in ("w1", "w2", "w3"):
        for k, t in want[p].items():
            if t is not None:
                assert torch.equal(views[p][k], t), (p, k)
        # the expert's own tensors now alias the slab: no second host copy
        w = getattr(ex, p)["weight"]
        base = ex.pinned_slab.data_ptr()
        assert base <= w.data_ptr() < base + ex.pinned_slab.numel()
