"""Quorum reads and cross-owner digest agreement (reference ``schedule/quorum.py``).

Replica owners report ``{key: [version, digest]}``; a value is confirmed when at
least ``quorum`` reports agree on both, preferring the highest version. A peer that
reports the confirmed version with a different digest is divergent (Byzantine).
"""

from __future__ import annotations


def _pair(v) -> tuple:
    return tuple(v) if isinstance(v, (tuple, list)) else (0, int(v))


def valid_report(vd):
    """``((epoch, counter), digest)`` from an untrusted ``[version, digest]``, or None."""
    try:
        ver, dig = vd[0], vd[1]
    except (TypeError, IndexError, KeyError):
        return None
    if not isinstance(dig, str) or not isinstance(ver, (list, tuple)) or len(ver) != 2:
        return None
    if not all(isinstance(x, int) and not isinstance(x, bool) for x in ver):
        return None
    return (int(ver[0]), int(ver[1])), dig


def confirm_version(reports, quorum: int):
    counts: dict = {}
    for v, d in reports:
        counts[(_pair(v), d)] = counts.get((_pair(v), d), 0) + 1
    ok = [vd for vd, n in counts.items() if n >= max(1, quorum)]
    return max(ok, key=lambda vd: vd[0]) if ok else None


def divergent_peers(reports_by_peer: dict, confirmed) -> set:
    if confirmed is None:
        return set()
    cv, cd = _pair(confirmed[0]), confirmed[1]
    return {p for p, r in reports_by_peer.items()
            if r is not None and _pair(r[0]) == cv and r[1] != cd}


def read_quorum_versions(addrs, keys, quorum: int, rpc) -> dict:
    per: dict = {k: [] for k in keys}
    for addr in addrs:
        try:
            reply = rpc(addr, {"type": "digest", "keys": list(keys)})
        except (OSError, ConnectionError):
            continue
        for k, vd in ((reply or {}).get("digests") or {}).items():
            r = valid_report(vd)
            if k in per and r is not None:
                per[k].append(r)
    out = {}
    for k, reps in per.items():
        c = confirm_version(reps, quorum)
        if c is not None:
            out[k] = c
    return out
