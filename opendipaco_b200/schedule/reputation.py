"""Per-peer reputation (reference ``src/opendipaco/schedule/reputation.py``).

A score in ``[lo, hi]`` starting at ``floor``; ``credit`` adds a small step for an
accepted contribution, ``debit`` removes a larger one for a rejected / divergent
one, and the distance from ``floor`` decays with half-life ``decay_halflife`` (s).
Scores gate owner eligibility, lease priority and rate-limit generosity.
"""

from __future__ import annotations

import threading
import time


class Reputation:
    def __init__(self, *, floor: float = 0.5, credit: float = 0.02, debit: float = 0.2,
                 decay_halflife: float = 3600.0, lo: float = 0.0, hi: float = 1.0):
        if not lo <= floor <= hi:
            raise ValueError("floor must be within [lo, hi]")
        self.floor, self.credit_step, self.debit_step = floor, credit, debit
        self.decay_halflife, self.lo, self.hi = decay_halflife, lo, hi
        self._scores: dict[str, tuple[float, float]] = {}
        self._lock = threading.Lock()

    def _current(self, pid: str, now: float) -> float:
        if pid not in self._scores:
            return self.floor
        score, ts = self._scores[pid]
        if self.decay_halflife > 0 and now > ts:
            score = self.floor + (score - self.floor) * 0.5 ** ((now - ts) / self.decay_halflife)
        return score

    def _store(self, pid: str, score: float, now: float) -> None:
        self._scores[pid] = (min(self.hi, max(self.lo, score)), now)

    def get(self, peer_id: str | None) -> float:
        if peer_id is None:
            return self.floor
        with self._lock:
            return self._current(peer_id, time.monotonic())

    def _adjust(self, peer_id: str | None, delta: float) -> float:
        if peer_id is None:
            return self.floor
        now = time.monotonic()
        with self._lock:
            self._store(peer_id, self._current(peer_id, now) + delta, now)
            return self._scores[peer_id][0]

    def credit(self, peer_id: str | None) -> float:
        return self._adjust(peer_id, self.credit_step)

    def debit(self, peer_id: str | None) -> float:
        return self._adjust(peer_id, -self.debit_step)

    def eligible(self, peer_id: str | None, threshold: float) -> bool:
        return peer_id is None or self.get(peer_id) >= threshold

    def snapshot(self) -> dict:
        now = time.monotonic()
        with self._lock:
            return {p: self._current(p, now) for p in self._scores}

    def restore(self, scores: dict) -> None:
        now = time.monotonic()
        with self._lock:
            for p, s in (scores or {}).items():
                self._store(str(p), float(s), now)
