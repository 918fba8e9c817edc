"""Owner sets and epochs (reference ``src/opendipaco/schedule/ownership.py``).

An *epoch record* names the owners (parameter servers) of the moment; every module
key maps to its ``k`` replicas by rendezvous (highest-random-weight) hashing,
``sha256(salt \\0 key \\0 peer_id)``, so a membership change moves only the keys of
the peers that came or went. The first-ranked replica is the key's *primary* (the
only writer in scheduler mode); the others pull its state.

Records come in two kinds: scheduler-signed (``make_epoch_record``) and
``deterministic`` (``derive_epoch``), which every node recomputes from the same
directory, whose epoch number bumps only when the membership hash changes.
``EpochManager`` adds hysteresis (an owner leaves only after ``owner_grace``
seconds unseen, or at once on a fresh signed tombstone) and rate limiting
(``min_epoch_interval``) to directory-driven epoch changes.

The record layout and the HRW score are wire/placement contracts shared with the
reference, so mixed clusters place keys identically.
"""

from __future__ import annotations

import hashlib
import json
import time

from .identity import PeerIdentity, sign_record, verify_record

OWNER_ROLE = "owner"
DEFAULT_REPLICATION = 3


# ----------------------------------------------------------------------- addresses
def owner_addr(record: dict):
    """Where to dial an owner: its public ``addr`` or its first relay circuit address."""
    if record.get("addr"):
        return record["addr"]
    circ = record.get("circuit_addrs") or []
    return circ[0] if circ else None


def owner_addrs(record: dict) -> list:
    return [record["addr"]] if record.get("addr") else list(record.get("circuit_addrs") or [])


def owner_addr_sig(record: dict) -> tuple:
    """Hashable form of an owner's addresses (a re-register at a new address is a change)."""
    return tuple(tuple(a) if isinstance(a, list) else a for a in owner_addrs(record))


def owner_eligible(record: dict) -> bool:
    """A directory record that may own keys: role ``owner`` and dialable."""
    if not isinstance(record, dict) or record.get("kind") != "peer":
        return False
    if OWNER_ROLE not in (record.get("roles") or []) or not isinstance(record.get("peer_id"), str):
        return False
    reach = record.get("reachability")
    if reach == "public":
        return bool(record.get("addr"))
    return reach == "nat" and bool(record.get("circuit_addrs"))


def _issued_at(record: dict) -> float:
    ts = record.get("issued_at") if isinstance(record, dict) else None
    return float(ts) if isinstance(ts, (int, float)) and not isinstance(ts, bool) else 0.0


# ------------------------------------------------------------------------ placement
def _score(salt: str, key: str, peer_id: str) -> bytes:
    return hashlib.sha256(f"{salt}\x00{key}\x00{peer_id}".encode()).digest()


def rank_owners(key: str, owners, *, salt: str = "") -> list[dict]:
    """All owners, best HRW score first (ties broken by peer id)."""
    return sorted(owners, key=lambda o: (_score(salt, key, o["peer_id"]), o["peer_id"]), reverse=True)


def owners_for(key: str, epoch_record: dict, k: int | None = None) -> list[dict]:
    """The ``k`` replicas of ``key`` under an epoch; element 0 is the primary."""
    k = int(epoch_record.get("k", DEFAULT_REPLICATION)) if k is None else k
    return rank_owners(key, epoch_record["owners"], salt=epoch_record.get("salt", ""))[:max(1, k)]


def _owner_entry(r: dict) -> dict:
    return {"peer_id": r["peer_id"], "addr": owner_addr(r), "addrs": owner_addrs(r)}


# -------------------------------------------------------------------------- records
def make_epoch_record(identity: PeerIdentity, *, epoch: int, owner_records, k: int = DEFAULT_REPLICATION,
                      salt: str = "", bootstrap: bool = False) -> dict:
    """A scheduler-signed epoch over ``owner_records`` (each must be owner-eligible)."""
    owners = []
    for r in owner_records:
        if not owner_eligible(r):
            raise ValueError(f"record not owner-eligible: {r.get('peer_id')!r}")
        owners.append(_owner_entry(r))
    owners.sort(key=lambda o: o["peer_id"])
    return sign_record(identity, {"kind": "epoch", "epoch": int(epoch), "k": int(k), "salt": salt,
                                  "bootstrap": bool(bootstrap), "owners": owners, "issued_at": time.time()})


def _members_sig(owners) -> str:
    payload = [[o["peer_id"], o["addr"]] for o in owners]
    return hashlib.sha256(json.dumps(payload, sort_keys=True).encode()).hexdigest()


def derive_epoch(owner_records, *, k: int = DEFAULT_REPLICATION, salt: str = "", prev: dict | None = None,
                 is_eligible=None) -> dict:
    """Unsigned epoch every node derives identically from the same directory.

    Unchanged membership (same hash, same ``k``) returns ``prev`` itself; a change
    bumps the epoch number. Never marked ``bootstrap``: a node joining a running
    cluster must sync gained keys rather than serve its freshly seeded bank.
    """
    owners = sorted((_owner_entry(r) for r in owner_records
                     if owner_eligible(r) and (is_eligible is None or is_eligible(r["peer_id"]))),
                    key=lambda o: o["peer_id"])
    sig = _members_sig(owners)
    if prev is not None and prev.get("members_sig") == sig and int(prev.get("k", k)) == int(k):
        return prev
    return {"kind": "epoch", "epoch": 0 if prev is None else int(prev["epoch"]) + 1, "k": int(k), "salt": salt,
            "bootstrap": False, "owners": owners, "members_sig": sig, "deterministic": True,
            "issued_at": time.time()}


def _well_formed(record) -> bool:
    if record.get("kind") != "epoch":
        return False
    for field, lo in (("epoch", 0), ("k", 1)):
        v = record.get(field)
        if not isinstance(v, int) or isinstance(v, bool) or v < lo:
            return False
    if not isinstance(record.get("issued_at"), (int, float)):
        return False
    owners = record.get("owners")
    if not isinstance(owners, list):
        return False
    ids = set()
    for o in owners:
        if not (isinstance(o, dict) and isinstance(o.get("peer_id"), str) and o.get("addr")):
            return False
        if o["peer_id"] in ids:  # a duplicate would double that owner's placement odds
            return False
        ids.add(o["peer_id"])
    return True


def verify_epoch_record(record, *, signer_pub: str | None = None, allow_deterministic: bool = False) -> bool:
    """Valid signature (by ``signer_pub`` when pinned) and well-formed; with
    ``allow_deterministic`` an unsigned derived record is checked on structure only."""
    if not isinstance(record, dict):
        return False
    if allow_deterministic and record.get("deterministic") and "sig" not in record:
        return _well_formed(record)
    if not verify_record(record):
        return False
    if signer_pub is not None and str(record.get("pub", "")).lower() != signer_pub.lower():
        return False
    return _well_formed(record)


def epoch_newer(a: dict, b: dict | None) -> bool:
    """Ordered by ``(epoch, issued_at)`` so a re-issued record of one epoch supersedes."""
    return b is None or (a["epoch"], a["issued_at"]) > (b["epoch"], b["issued_at"])


class EpochManager:
    """Decides when the owner set changed enough to publish a new epoch."""

    def __init__(self, *, owner_grace: float = 240.0, min_epoch_interval: float = 60.0, is_eligible=None):
        self.owner_grace, self.min_epoch_interval = owner_grace, min_epoch_interval
        self.is_eligible = is_eligible
        self._seen: dict = {}          # peer_id -> (last seen, record)
        self._current = None           # {(peer_id, addr signature)}
        self._last_bump = None

    def observe(self, records, *, tombstoned=None, now: float | None = None):
        """One directory snapshot in; owner records of a due new epoch out (else None).

        ``tombstoned`` maps peer id -> ``issued_at`` of its signed deregister; it evicts
        at once only when it is newer than the registration held (a replayed old
        tombstone must not evict a peer that rejoined)."""
        now = time.monotonic() if now is None else now
        for r in records:
            if owner_eligible(r) and (self.is_eligible is None or self.is_eligible(r["peer_id"])):
                self._seen[r["peer_id"]] = (now, r)
        for p, ts in dict(tombstoned or {}).items():
            held = self._seen.get(p)
            if held is not None and isinstance(ts, (int, float)) and not isinstance(ts, bool) \
                    and ts > _issued_at(held[1]):
                del self._seen[p]
        for p in [p for p, (t, _) in self._seen.items() if now - t >= self.owner_grace]:
            del self._seen[p]
        if not self._seen:
            return None
        live = {p: rec for p, (_, rec) in self._seen.items()}
        sig = {(p, owner_addr_sig(rec)) for p, rec in live.items()}
        if sig == self._current:
            return None
        if self._last_bump is not None and now - self._last_bump < self.min_epoch_interval:
            return None
        self._current, self._last_bump = sig, now
        return [live[p] for p in sorted(live)]
