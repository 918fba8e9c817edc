"""Per-peer token bucket scaled by reputation (reference ``schedule/ratelimit.py``).

A peer with reputation r gets ``capacity * (0.5 + r)`` burst and the same factor on
the refill rate; a request costing more than the available tokens is refused.
"""

from __future__ import annotations

import threading
import time


class RateLimiter:
    def __init__(self, *, capacity: float = 8.0, refill_per_sec: float = 2.0):
        self.capacity, self.refill = float(capacity), float(refill_per_sec)
        self._buckets: dict[str, tuple[float, float]] = {}
        self._lock = threading.Lock()

    @staticmethod
    def _scale(reputation: float) -> float:
        return 0.5 + reputation

    def allow(self, peer_id: str | None, *, reputation: float = 0.5, cost: float = 1.0) -> bool:
        if peer_id is None:
            return True
        k = self._scale(reputation)
        cap, now = self.capacity * k, time.monotonic()
        with self._lock:
            tokens, ts = self._buckets.get(peer_id, (cap, now))
            tokens = min(cap, tokens + (now - ts) * self.refill * k)
            ok = tokens >= cost
            self._buckets[peer_id] = (tokens - cost if ok else tokens, now)
            return ok
