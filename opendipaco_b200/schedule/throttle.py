"""Uplink bandwidth shaping for volunteer workers (reference ``schedule/throttle.py``).

``tailor_encoding`` picks a per-worker wire encoding from its advertised uplink
(>= 20 Mbps: the run default; >= 5: int8; below: int4 with at most 50% density),
never weaker than the run's own compression. ``TokenBucket`` / ``ThrottledSocket``
meter a socket's bytes against a shared bucket.
"""

from __future__ import annotations

import math
import threading
import time

_RANK = {"none": 0, "bf16": 1, "int8": 2, "int4": 3}


def tailor_encoding(max_mbps: float | None, *, base_compress: str = "none", base_density: float = 1.0,
                    hi: float = 20.0, lo: float = 5.0):
    if max_mbps is None or not math.isfinite(max_mbps) or max_mbps >= hi:
        comp, dens = base_compress, base_density
    elif max_mbps >= lo:
        comp, dens = "int8", base_density
    else:
        comp, dens = "int4", min(base_density, 0.5)
    if _RANK.get(base_compress, 0) > _RANK.get(comp, 0):
        comp = base_compress
    return comp, dens


def rate_from_mbps(max_mbps: float | None) -> float | None:
    if max_mbps is None or not math.isfinite(max_mbps) or max_mbps <= 0:
        return None
    return max_mbps * 1e6 / 8.0


class TokenBucket:
    def __init__(self, rate_bytes_per_sec: float, *, capacity: float | None = None):
        self.rate = float(rate_bytes_per_sec)
        self.capacity = float(capacity if capacity is not None else rate_bytes_per_sec)
        self._tokens, self._ts = self.capacity, time.monotonic()
        self._lock = threading.Lock()
        self.sent_bytes = self.recv_bytes = 0

    def take(self, n: int) -> None:
        if n <= 0 or self.rate <= 0:
            return
        with self._lock:
            now = time.monotonic()
            self._tokens = min(self.capacity, self._tokens + (now - self._ts) * self.rate) - n
            self._ts = now
            deficit = max(0.0, -self._tokens)
        if deficit:
            time.sleep(deficit / self.rate)


class ThrottledSocket:
    def __init__(self, sock, bucket: TokenBucket):
        self._sock, self._bucket = sock, bucket

    def __getattr__(self, name):
        return getattr(self._sock, name)

    def sendall(self, data, *args):
        self._bucket.take(len(data))
        self._bucket.sent_bytes += len(data)
        return self._sock.sendall(data, *args)

    def send(self, data, *args) -> int:
        self._bucket.take(len(data))
        n = self._sock.send(data, *args)
        self._bucket.sent_bytes += n
        return n

    def recv(self, bufsize, *args):
        data = self._sock.recv(bufsize, *args)
        if data:
            self._bucket.recv_bytes += len(data)
            self._bucket.take(len(data))
        return data

    def close(self):
        return self._sock.close()


def throttled(sock, bucket: TokenBucket | None):
    return ThrottledSocket(sock, bucket) if bucket is not None else sock
