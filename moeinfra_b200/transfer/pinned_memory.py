"""Byte budget for page-locked host memory.

Same public surface as the reference's ``transfer/pinned_memory.py``
(``PinnedMemoryBudget(budget_bytes)`` with ``budget_bytes``, ``used_bytes``,
``available_bytes``, ``can_reserve``, ``reserve``, ``release`` and its
``repr``), designed for this package's staging pool: the staging slabs are
reserved and released from the host thread that runs the layer and, with the
asynchronous prefetcher, from the thread that polls finished copies, so the
ledger is updated under a lock and also records the high-water mark (how much
pinned memory the run actually needed).
"""
from __future__ import annotations

import threading


def _nonnegative(size_bytes: int) -> int:
    size = int(size_bytes)
    if size < 0:
        raise ValueError(f"size_bytes must be >= 0, got {size}")
    return size


class PinnedMemoryBudget:
    """Upper bound on the pinned bytes the staging pool may hold at once."""

    __slots__ = ("_limit", "_used", "_peak", "_lock")

    def __init__(self, budget_bytes: int):
        limit = int(budget_bytes)
        if limit < 0:
            raise ValueError(f"budget_bytes must be >= 0, got {limit}")
        self._limit = limit
        self._used = 0
        self._peak = 0
        self._lock = threading.Lock()

    @property
    def budget_bytes(self) -> int:
        return self._limit

    @property
    def used_bytes(self) -> int:
        return self._used

    @used_bytes.setter
    def used_bytes(self, value: int) -> None:
        # Only a pool tearing down all of its slabs resets the ledger.
        value = _nonnegative(value)
        with self._lock:
            self._used = value

    @property
    def available_bytes(self) -> int:
        return self._limit - self._used

    @property
    def peak_bytes(self) -> int:
        """Largest ``used_bytes`` seen so far."""
        return self._peak

    def can_reserve(self, size_bytes: int) -> bool:
        return _nonnegative(size_bytes) <= self._limit - self._used

    def reserve(self, size_bytes: int) -> bool:
        """Take ``size_bytes`` from the budget; False (and no change) if they do not fit."""
        size = _nonnegative(size_bytes)
        with self._lock:
            if size > self._limit - self._used:
                return False
            self._used += size
            self._peak = max(self._peak, self._used)
            return True

    def release(self, size_bytes: int) -> None:
        """Give ``size_bytes`` back; releasing more than is held is an accounting error."""
        size = _nonnegative(size_bytes)
        with self._lock:
            if size > self._used:
                raise ValueError(
                    f"release of {size} bytes exceeds the {self._used} bytes held (underflow)")
            self._used -= size

    def __repr__(self) -> str:
        return (f"PinnedMemoryBudget(budget_bytes={self._limit}, used_bytes={self._used}, "
                f"available_bytes={self.available_bytes})")
