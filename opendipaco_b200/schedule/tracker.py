"""Peer directory / rendezvous tracker (reference ``src/opendipaco/schedule/tracker.py``).

Peers publish self-certifying Ed25519-signed records ``{kind: "peer", reachability,
addr, roles, capabilities, issued_at[, circuit_addrs]}``; the tracker admits a
record only with a valid signature, an enrolled key (unless enrollment is open),
a legal reachability and a fresher ``issued_at`` than the one it holds, keeps it
for ``ttl`` seconds, and serves the directory filtered by role / reachability.
A signed ``deregister`` leaves a tombstone (also served, so an epoch watcher can
fail a graceful leave over at once). The tracker also caches the scheduler's
signed epoch record (first valid signer is pinned; only newer epochs replace it)
and the run manifest.

Every record is re-verified by the client (``fetch_directory``), so a tracker or
relay is never trusted for content; ``fetch_directory_multi`` takes the union over
several seeds (freshest record per peer, verified tombstones suppress older
registrations, optional M-of-N seed quorum against injected Sybils).

Message types and record fields are the reference's wire contract.
"""

from __future__ import annotations

import threading
import time
from concurrent.futures import ThreadPoolExecutor

from .identity import PeerIdentity, sign_record, verify_record
from .ownership import epoch_newer, verify_epoch_record
from .reactor import ReactorServer
from .rpc import one_shot, record_issued_at
from .wire import DEFAULT_MAX_MSG_BYTES

REACHABILITY = ("public", "nat")
# directory frames are small JSON-like records, never tensors
TRACKER_MAX_MSG_BYTES = 16 * 1024 * 1024


def make_peer_record(identity: PeerIdentity, *, reachability: str = "nat", addr=None, roles=(), capabilities=None,
                     circuit_addrs=None) -> dict:
    """This peer's signed directory record. ``public`` peers must give ``addr=(host, port)``;
    ``nat`` peers dial out only and may advertise relay ``circuit_addrs``."""
    if reachability not in REACHABILITY:
        raise ValueError(f"reachability must be one of {REACHABILITY}, got {reachability!r}")
    if reachability == "public" and not addr:
        raise ValueError("a 'public' peer must advertise addr=(host, port)")
    if reachability == "nat" and addr:
        raise ValueError("a 'nat' peer is dial-out-only; it cannot advertise an addr")
    rec = {"kind": "peer", "reachability": reachability, "addr": list(addr) if addr else None,
           "roles": sorted(roles), "capabilities": dict(capabilities or {}), "issued_at": time.time()}
    if circuit_addrs:
        rec["circuit_addrs"] = list(circuit_addrs)
    return sign_record(identity, rec)


class Tracker(ReactorServer):
    def __init__(self, *, host: str = "0.0.0.0", port: int = 0, ttl: float = 120.0, open_enrollment: bool = False,
                 enroll_peers=None, auth_key=None, max_peers: int = 65536,
                 max_msg_bytes: int = TRACKER_MAX_MSG_BYTES, epoch_signer=None, **kw):
        super().__init__(host=host, port=port, auth_key=auth_key, max_msg_bytes=max_msg_bytes, **kw)
        self.ttl, self.max_peers, self.open_enrollment = ttl, max_peers, open_enrollment
        self._dir_lock = threading.Lock()
        self._enrolled = {self._pub(p) for p in enroll_peers or []}
        self._peers: dict = {}      # peer_id -> {record | None, deregister, issued_at, expires}
        self._epoch = None
        self._epoch_signer = self._pub(epoch_signer) if epoch_signer else None
        self._manifest = None

    def serve_manifest(self, manifest: dict | None) -> None:
        self._manifest = manifest

    @staticmethod
    def _pub(p) -> str:
        return getattr(p, "public_key_hex", p).lower()

    def enroll(self, pub) -> None:
        with self._dir_lock:
            self._enrolled.add(self._pub(pub))

    def expel(self, pub) -> None:
        """Revoke enrollment and tombstone the peer's record at once."""
        pub = self._pub(pub)
        with self._dir_lock:
            self._enrolled.discard(pub)
            for pid, e in list(self._peers.items()):
                if e["record"] is not None and e["record"].get("pub", "").lower() == pub:
                    self._tombstone(pid, time.time())

    def _handle(self, msg: dict, nbytes: int, peer_id: str | None = None):
        kind = msg.get("type")
        if kind == "register":
            return self._register(msg.get("record"))
        if kind == "deregister":
            return self._deregister(msg.get("record"))
        if kind == "directory":
            return self._directory(msg)
        if kind == "import":
            recs = msg.get("records") or []
            n = sum(1 for r in recs if self._register(r).get("type") == "registered")
            return {"type": "imported", "accepted": n}
        if kind == "epoch_put":
            return self._epoch_put(msg.get("record"))
        if kind == "epoch_get":
            with self._dir_lock:
                return {"type": "epoch", "record": self._epoch}
        if kind == "manifest":
            return {"type": "manifest", "manifest": self._manifest}
        return None

    # -- admission --------------------------------------------------------------
    def _admit(self, rec) -> str:
        if not verify_record(rec):
            return "bad signature"
        if rec.get("kind") != "peer":
            return "not a peer record"
        if not (self.open_enrollment or rec["pub"].lower() in self._enrolled):
            return "not enrolled"
        if rec.get("reachability") not in REACHABILITY:
            return "bad reachability"
        if rec["reachability"] == "public" and not rec.get("addr"):
            return "public peer without addr"
        if not isinstance(rec.get("issued_at"), (int, float)):
            return "missing issued_at"
        return ""

    def _register(self, rec) -> dict:
        why = self._admit(rec)
        if why:
            return {"type": "refused", "reason": why}
        with self._dir_lock:
            self._purge()
            held = self._peers.get(rec["peer_id"])
            if held is not None and rec["issued_at"] <= held["issued_at"]:
                return {"type": "refused", "reason": "stale record"}
            if held is None and len(self._peers) >= self.max_peers:
                return {"type": "refused", "reason": "directory full"}
            self._peers[rec["peer_id"]] = {"record": rec, "issued_at": rec["issued_at"],
                                           "expires": time.monotonic() + self.ttl}
        return {"type": "registered", "ttl": self.ttl}

    def _deregister(self, rec) -> dict:
        if not verify_record(rec) or rec.get("kind") != "deregister":
            return {"type": "refused", "reason": "bad signature"}
        with self._dir_lock:
            held = self._peers.get(rec["peer_id"])
            if held is not None and rec.get("issued_at", 0) <= held["issued_at"]:
                return {"type": "refused", "reason": "stale record"}
            self._tombstone(rec["peer_id"], rec.get("issued_at", time.time()), rec)
        return {"type": "deregistered"}

    def _epoch_put(self, rec) -> dict:
        if not verify_epoch_record(rec):
            return {"type": "refused", "reason": "bad epoch record"}
        pub = rec["pub"].lower()
        with self._dir_lock:
            if self._epoch_signer is not None and pub != self._epoch_signer:
                return {"type": "refused", "reason": "wrong signer"}
            if not epoch_newer(rec, self._epoch):
                return {"type": "refused", "reason": "stale epoch"}
            self._epoch_signer, self._epoch = pub, rec
        return {"type": "epoch_cached"}

    def _directory(self, msg: dict) -> dict:
        roles, reach = set(msg.get("roles") or []), msg.get("reachability")
        with self._dir_lock:
            self._purge()
            recs = [e["record"] for e in self._peers.values() if e["record"] is not None]
            tombs = [e["deregister"] for e in self._peers.values() if e["record"] is None and e.get("deregister")]
        if roles:
            recs = [r for r in recs if roles & set(r.get("roles") or [])]
        if reach:
            recs = [r for r in recs if r.get("reachability") == reach]
        out = {"type": "directory", "records": recs}
        if msg.get("include_tombstones"):
            out["tombstones"] = tombs
        return out

    def _tombstone(self, peer_id: str, issued_at: float, deregister=None) -> None:
        self._peers[peer_id] = {"record": None, "deregister": deregister, "issued_at": issued_at,
                                "expires": time.monotonic() + self.ttl}

    def _purge(self) -> None:
        now = time.monotonic()
        for pid in [p for p, e in self._peers.items() if now >= e["expires"]]:
            del self._peers[pid]

    def records(self) -> list[dict]:
        with self._dir_lock:
            self._purge()
            return [e["record"] for e in self._peers.values() if e["record"] is not None]

    def tombstones(self) -> list[str]:
        with self._dir_lock:
            self._purge()
            return [p for p, e in self._peers.items() if e["record"] is None]


# ================================================================= client helpers
def tracker_rpc(addr, msg, *, auth_key=None, tls=None, timeout: float = 10.0,
                max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES):
    return one_shot(tuple(addr), msg, auth_key=auth_key, tls=tls, timeout=timeout, max_msg_bytes=max_msg_bytes)


def register_peer(addr, identity: PeerIdentity, *, reachability: str = "nat", peer_addr=None, roles=(),
                  capabilities=None, auth_key=None, tls=None, timeout: float = 10.0, circuit_addrs=None) -> dict:
    """Register (or refresh, before ``ttl`` runs out) this peer's record; a ``nat`` peer
    may advertise the relay ``circuit_addrs`` it is reachable through."""
    rec = make_peer_record(identity, reachability=reachability, addr=peer_addr, roles=roles,
                           capabilities=capabilities, circuit_addrs=circuit_addrs)
    return tracker_rpc(addr, {"type": "register", "record": rec}, auth_key=auth_key, tls=tls, timeout=timeout)


def deregister_peer(addr, identity: PeerIdentity, *, auth_key=None, tls=None, timeout: float = 10.0) -> dict:
    rec = sign_record(identity, {"kind": "deregister", "issued_at": time.time()})
    return tracker_rpc(addr, {"type": "deregister", "record": rec}, auth_key=auth_key, tls=tls, timeout=timeout)


def fetch_directory(addr, *, roles=None, reachability=None, auth_key=None, tls=None, timeout: float = 10.0,
                    verify: bool = True) -> list[dict]:
    reply = tracker_rpc(addr, {"type": "directory", "roles": list(roles or []), "reachability": reachability},
                        auth_key=auth_key, tls=tls, timeout=timeout) or {}
    recs = reply.get("records") or []
    return [r for r in recs if verify_record(r)] if verify else recs


def fetch_directory_and_tombstones(addr, *, roles=None, reachability=None, auth_key=None, tls=None,
                                   timeout: float = 10.0, verify: bool = True):
    """``(records, {peer_id: deregister issued_at})`` in one round trip."""
    reply = tracker_rpc(addr, {"type": "directory", "roles": list(roles or []), "reachability": reachability,
                               "include_tombstones": True}, auth_key=auth_key, tls=tls, timeout=timeout) or {}
    recs, tombs = reply.get("records") or [], reply.get("tombstones") or []
    if verify:
        recs = [r for r in recs if verify_record(r)]
        tombs = [t for t in tombs if verify_record(t) and t.get("kind") == "deregister"]
    out = {}
    for t in tombs:
        ts = record_issued_at(t)
        if ts is not None:
            out[t["peer_id"]] = ts
    return recs, out


def dedup_seeds(primary, extras=()):
    """``primary`` then each distinct extra, normalised to ``(host, int(port))``."""
    out = [(primary[0], int(primary[1]))]
    for s in extras or []:
        a = (s[0], int(s[1]))
        if a not in out:
            out.append(a)
    return out


def fetch_directory_multi(seeds, *, roles=None, reachability=None, auth_key=None, tls=None, timeout: float = 10.0,
                          seed_quorum: int = 1):
    """Union of verified records over several trackers; returns ``(records, seeds_answered)``."""
    addrs = list(dict.fromkeys((s[0], int(s[1])) for s in seeds))

    def fetch(a):
        return fetch_directory_and_tombstones(a, roles=roles, reachability=reachability, auth_key=auth_key,
                                              tls=tls, timeout=timeout)

    results = []
    if addrs:
        with ThreadPoolExecutor(max_workers=len(addrs)) as ex:
            for fut in [ex.submit(fetch, a) for a in addrs]:
                try:
                    results.append(fut.result())
                except Exception:
                    continue
    best, tombs, served = {}, {}, {}
    for recs, t in results:
        for pid, ts in t.items():
            tombs[pid] = max(ts, tombs.get(pid, ts))
        here = set()
        for r in recs:
            pid, ts = r.get("peer_id"), record_issued_at(r)
            if not isinstance(pid, str) or ts is None:
                continue
            if pid not in here:
                here.add(pid)
                served[pid] = served.get(pid, 0) + 1
            if pid not in best or ts > best[pid][0]:
                best[pid] = (ts, r)
    out = [r for pid, (ts, r) in best.items() if served[pid] >= seed_quorum and (pid not in tombs or ts > tombs[pid])]
    return out, len(results)


def import_records(addr, records, *, auth_key=None, tls=None, timeout: float = 10.0) -> dict:
    return tracker_rpc(addr, {"type": "import", "records": list(records)}, auth_key=auth_key, tls=tls,
                       timeout=timeout)


def put_epoch(addr, record, *, auth_key=None, tls=None, timeout: float = 10.0) -> dict:
    return tracker_rpc(addr, {"type": "epoch_put", "record": record}, auth_key=auth_key, tls=tls, timeout=timeout)


def get_epoch(addr, *, signer_pub=None, auth_key=None, tls=None, timeout: float = 10.0) -> dict | None:
    """The cached epoch, re-verified here (optionally pinned to the scheduler's key)."""
    reply = tracker_rpc(addr, {"type": "epoch_get"}, auth_key=auth_key, tls=tls, timeout=timeout) or {}
    rec = reply.get("record")
    return rec if rec is not None and verify_epoch_record(rec, signer_pub=signer_pub) else None
