"""Leaderless work assignment and version-vector staleness (reference ``schedule/assignment.py``).

Workers are ranked for a ``(path, generation)`` slot by rendezvous hashing
``sha256(salt \\0 path \\0 generation \\0 peer_id)`` (the same inputs as the
reference, so mixed peers agree); the slot passes to the next-ranked worker every
``lease_ttl`` seconds it stays open (takeover without a scheduler).
"""

from __future__ import annotations

import hashlib


def _path_str(path) -> str:
    return "-".join(str(int(i)) for i in path)


def _wscore(salt: str, path, generation: int, peer_id: str) -> bytes:
    return hashlib.sha256(f"{salt}\x00{_path_str(path)}\x00{int(generation)}\x00{peer_id}".encode()).digest()


def rank_workers(path, generation: int, workers, *, salt: str = "") -> list[str]:
    ids = [w["peer_id"] if isinstance(w, dict) else w for w in workers]
    return sorted(ids, key=lambda p: (_wscore(salt, path, generation, p), p), reverse=True)


def responsible_rank(elapsed: float, lease_ttl: float, n_workers: int) -> int:
    if n_workers <= 0 or lease_ttl <= 0:
        return 0
    return min(int(max(0.0, elapsed) // lease_ttl), n_workers - 1)


def assignee(path, generation: int, workers, *, salt: str = "", elapsed: float = 0.0,
             lease_ttl: float = 0.0) -> str | None:
    ranked = rank_workers(path, generation, workers, salt=salt)
    return ranked[responsible_rank(elapsed, lease_ttl, len(ranked))] if ranked else None


def is_assignee(peer_id: str, path, generation: int, workers, *, salt: str = "", elapsed: float = 0.0,
                lease_ttl: float = 0.0) -> bool:
    return peer_id is not None and assignee(path, generation, workers, salt=salt, elapsed=elapsed,
                                            lease_ttl=lease_ttl) == peer_id


def _pair(v) -> tuple[int, int]:
    return (int(v[0]), int(v[1])) if v is not None else (0, 0)


def version_lag(fetched: dict, current: dict) -> int | None:
    """Max counter lag over the fetched base versions; None when incomparable
    (unknown key, different epoch, or a fetched version from the future)."""
    if not fetched:
        return 0
    lag = 0
    for key, fv in fetched.items():
        if key not in current:
            return None
        (fe, fc), (ce, cc) = _pair(fv), _pair(current[key])
        if fe != ce or cc < fc:
            return None
        lag = max(lag, cc - fc)
    return lag


def coordinator_key(path_keys) -> str:
    """The path's first private key if any (it is unique to the path), else its
    lexicographically first key."""
    from ..topology import is_private_key

    keys = sorted(path_keys)
    priv = [k for k in keys if is_private_key(k)]
    return priv[0] if priv else keys[0]


def path_primary(path_keys, epoch_record) -> dict | None:
    from .ownership import owners_for

    owners = owners_for(coordinator_key(path_keys), epoch_record)
    return owners[0] if owners else None
