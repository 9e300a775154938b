"""Rolling host-link bandwidth monitor (API of the reference's ``transfer/bandwidth.py``).

Throughput is bytes in the window divided by the time since the window's
first sample, reported in GiB/s like the reference (``:58-83``).
"""
from __future__ import annotations

import collections
import time


class BandwidthMonitor:
    def __init__(self, window_s: float = 5.0) -> None:
        self.window_s = window_s
        self._samples: collections.deque[tuple[float, int]] = collections.deque()
        self._peak_gbps = 0.0

    def record(self, bytes_transferred: int) -> None:
        now = time.monotonic()
        self._samples.append((now, int(bytes_transferred)))
        while self._samples and self._samples[0][0] < now - self.window_s:
            self._samples.popleft()
        self._peak_gbps = max(self._peak_gbps, self.current_gbps())

    def current_gbps(self) -> float:
        if len(self._samples) < 2:
            return 0.0
        now = time.monotonic()
        live = [s for s in self._samples if s[0] >= now - self.window_s]
        if not live:
            return 0.0
        span = now - live[0][0]
        if span <= 0:
            return 0.0
        return sum(b for _, b in live) / span / float(1 << 30)

    def peak_gbps(self) -> float:
        return self._peak_gbps

    def reset(self) -> None:
        self._samples.clear()
        self._peak_gbps = 0.0
