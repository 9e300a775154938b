"""CPU contract of ``PrefetchEngine`` (the reference's ``engine/prefetch.py``).

Follows the reference's ``tests/test_prefetch.py`` and the prefetch half of
``tests/test_engine.py``: NONE submits nothing; NEXT_LAYER requests each
unique routed expert for the next layer; LOOKAHEAD for every layer up to the
depth; GPU-resident experts and already-requested experts are skipped;
rejected submissions are not remembered; ``cancel_stale`` cancels requests of
past layers (and forgets them even when the scheduler can no longer cancel);
``on_layer_complete`` cancels stale requests before scheduling new ones.
"""
from __future__ import annotations

import torch

from moeinfra_b200.engine.prefetch import PrefetchEngine
from moeinfra_b200.engine.types import PrefetchPolicy
from moeinfra_b200.transfer.types import TransferHandle, TransferPriority, TransferStatus


class Residency:
    def __init__(self, resident=()):
        self.resident = set(resident)

    def is_gpu_resident(self, layer, expert):
        return (layer, expert) in self.resident


class FakeAsyncScheduler:
    """Records async submissions and cancellations; can reject or refuse to cancel."""

    def __init__(self, reject=(), cancel_ok=True):
        self.submitted = []
        self.cancelled = []
        self.reject = set(reject)
        self.cancel_ok = cancel_ok

    def submit_async(self, request):
        self.submitted.append(request)
        status = (TransferStatus.REJECTED if (request.layer_id, request.expert_id) in self.reject
                  else TransferStatus.IN_FLIGHT)
        return TransferHandle(request_id=request.request_id, layer_id=request.layer_id,
                              expert_id=request.expert_id, slot=None, event=None, status=status)

    def cancel(self, request_id):
        self.cancelled.append(request_id)
        return self.cancel_ok


def engine(policy, depth=2, resident=(), **kw):
    sched = FakeAsyncScheduler(**kw)
    return PrefetchEngine(Residency(resident), sched, policy, depth), sched


def keys(sched):
    return [(r.layer_id, r.expert_id) for r in sched.submitted]


def test_none_policy_submits_nothing():
    pe, sched = engine(PrefetchPolicy.NONE)
    assert pe.schedule_prefetch(3, torch.tensor([[1, 2]])) == []
    assert sched.submitted == []


def test_next_layer_requests_unique_experts_for_the_next_layer_at_low_priority():
    pe, sched = engine(PrefetchPolicy.NEXT_LAYER)
    ids = pe.schedule_prefetch(4, torch.tensor([[3, 1], [1, 6], [6, 3]]))
    assert keys(sched) == [(5, 1), (5, 3), (5, 6)]
    assert len(ids) == 3 and len(set(ids)) == 3
    assert all(r.priority == TransferPriority.LOW for r in sched.submitted)


def test_lookahead_covers_each_layer_up_to_the_depth():
    pe, sched = engine(PrefetchPolicy.LOOKAHEAD, depth=3)
    pe.schedule_prefetch(0, torch.tensor([[2, 5]]))
    assert keys(sched) == [(1, 2), (1, 5), (2, 2), (2, 5), (3, 2), (3, 5)]


def test_resident_and_duplicate_experts_are_skipped():
    pe, sched = engine(PrefetchPolicy.NEXT_LAYER, resident={(1, 2)})
    pe.schedule_prefetch(0, torch.tensor([[2, 4]]))
    pe.schedule_prefetch(0, torch.tensor([[4, 7]]))
    assert keys(sched) == [(1, 4), (1, 7)]


def test_rejected_requests_are_not_tracked_and_can_be_retried():
    pe, sched = engine(PrefetchPolicy.NEXT_LAYER, reject={(2, 0)})
    assert pe.schedule_prefetch(1, torch.tensor([[0, 1]])) != []
    assert (2, 0) not in pe.in_flight and (2, 1) in pe.in_flight
    sched.reject.clear()
    pe.schedule_prefetch(1, torch.tensor([[0]]))
    assert (2, 0) in pe.in_flight


def test_cancel_stale_drops_past_layers_only():
    pe, sched = engine(PrefetchPolicy.LOOKAHEAD, depth=2)
    pe.schedule_prefetch(0, torch.tensor([[1]]))  # layers 1, 2
    pe.schedule_prefetch(2, torch.tensor([[3]]))  # layers 3, 4
    assert pe.cancel_stale(3) == 2
    assert sorted(pe.in_flight) == [(3, 3), (4, 3)]
    assert len(sched.cancelled) == 2


def test_cancel_stale_forgets_even_when_the_scheduler_cannot_cancel():
    pe, sched = engine(PrefetchPolicy.NEXT_LAYER, cancel_ok=False)
    pe.schedule_prefetch(0, torch.tensor([[1, 2]]))
    assert pe.cancel_stale(5) == 0
    assert pe.in_flight == {}
    pe.schedule_prefetch(0, torch.tensor([[1]]))  # can be requested again
    assert keys(sched)[-1] == (1, 1)


def test_on_layer_complete_cancels_then_schedules():
    pe, sched = engine(PrefetchPolicy.NEXT_LAYER)
    pe.schedule_prefetch(0, torch.tensor([[1]]))  # (1, 1)
    pe.on_layer_complete(1, torch.tensor([[5]]))
    assert len(sched.cancelled) == 1  # layer 1's request is now stale
    assert list(pe.in_flight) == [(2, 5)]
    pe.forget(2, 5)
    assert pe.in_flight == {}
