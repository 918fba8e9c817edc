"""Sharded asynchronous DiLoCo: a weight-less scheduler + parameter servers (owners)
(reference ``src/opendipaco/schedule/sharded.py``).

* ``Scheduler`` hands out path-tasks (least-completed path, warm preference), tracks
  staleness and, on ``commit``, mints a single-use *grant* (HMAC- or Ed25519-signed)
  carrying the push weight ``alpha * 1/(1 + staleness)`` and the allowed keys. It
  never holds weights. Optional: throughput-measured task sizing (EMA rate, shrink
  batch then inner steps toward ``task_seconds``, park too-slow workers), redundant
  execution audits (replicas' pseudo-gradient digests, majority credits / debits
  reputation), trusted-probe screening, epochs published to owners, checkpoints.
* ``ParameterServer`` owns module keys: versioned ``(epoch, counter)`` weights and
  per-key outer optimizers. ``fetch`` ships only changed keys (optionally as an int8/
  int4 delta against a retained keyframe, or at a pinned version); ``push`` verifies
  the grant (single use, replay window), checks declared shapes before decoding,
  rejects non-finite data, optionally clips, then applies one outer step per key
  (or buffers ``quorum`` contributions and applies a robust aggregate). Under an
  epoch only the primary writes; backups pull exact state (``include_state``) from
  the primary; a gracefully leaving primary drains to its successor.
* ``run_sharded_worker`` / ``run_decentralized_worker`` are the worker loops.

Wire field names and the grant's canonical signed bytes match the reference.
"""

from __future__ import annotations

import collections
import hashlib
import hmac
import json
import logging
import os
import random
import threading
import time
import uuid
from collections import OrderedDict

import torch

from ..models.path import build_module_bank
from ..optim.diloco import apply_outer_grads, make_outer_optimizer
from ..parallel.backend.local import LocalBackend
from ..topology import is_private_key
from ..train.loop import _opt_state_cpu, _state_cpu
from .aggregate import check_aggregate, robust_delta
from .assignment import coordinator_key, is_assignee, version_lag
from .compress import (apply_state_delta, check_mode, compress_delta, compress_shard, compress_state,
                       declared_shape, encode_state_delta, maybe_dequantize, pseudograd_digest, restore_shard,
                       state_digest)
from .guard import all_finite, clip_norm_, loss_ok
from .identity import peer_id_of, sign_record, verify_record
from .ownership import (EpochManager, derive_epoch, epoch_newer, make_epoch_record, owners_for,
                        verify_epoch_record)
from .probe import TrustedProbe, as_finite_float, is_harmful
from .quorum import confirm_version, divergent_peers, read_quorum_versions
from .ratelimit import RateLimiter
from .reactor import ReactorServer
from .reputation import Reputation
from .rpc import connect, record_issued_at, rpc
from .scheduler import AsyncScheduler
from .throttle import tailor_encoding
from .wire import DEFAULT_MAX_MSG_BYTES, _kb

logger = logging.getLogger("opendipaco_b200.schedule")
_RATE_EMA = 0.3


# ============================================================================ helpers
def assign_shards(keys, num_shards: int) -> dict:
    """Round-robin placement of ``sorted(keys)`` over ``num_shards`` servers."""
    return {k: i % num_shards for i, k in enumerate(sorted(keys))}


def _grant_payload(grant: dict) -> bytes:
    return json.dumps({"path": list(grant["path"]), "token": grant["token"], "weight": grant["weight"],
                       "keys": list(grant["keys"])}, sort_keys=True, separators=(",", ":")).encode()


def make_grant(path, keys, weight: float, token: str, grant_key=None, *, identity=None) -> dict:
    g = {"path": list(path), "token": token, "weight": float(weight), "keys": sorted(keys)}
    if identity is not None:
        return sign_record(identity, {"kind": "grant", **g})
    if grant_key is not None:
        g["mac"] = hmac.new(_kb(grant_key), _grant_payload(g), hashlib.sha256).hexdigest()
    return g


def verify_grant(grant, grant_key, *, scheduler_pub: str | None = None) -> bool:
    if not isinstance(grant, dict) or not grant.get("token"):
        return False
    if scheduler_pub is not None:
        return verify_record(grant) and grant.get("kind") == "grant" and \
            grant.get("pub", "").lower() == scheduler_pub.lower()
    try:
        payload = _grant_payload(grant)
    except (KeyError, TypeError):
        return False
    if grant_key is None:
        return True
    return hmac.compare_digest(grant.get("mac", ""), hmac.new(_kb(grant_key), payload, hashlib.sha256).hexdigest())


def grant_signed_by(grant, expected_peer_id: str | None) -> bool:
    """Decentralized grant check: Ed25519-signed by exactly the expected owner."""
    if not isinstance(grant, dict) or not grant.get("token") or expected_peer_id is None:
        return False
    if not (verify_record(grant) and grant.get("kind") == "grant"):
        return False
    try:
        return peer_id_of(grant.get("pub", "")) == expected_peer_id
    except (ValueError, TypeError):
        return False


def _opt_to_wire(sd: dict) -> dict:
    return {"state": {str(i): s for i, s in sd["state"].items()}, "param_groups": sd["param_groups"]}


def _opt_from_wire(sd: dict) -> dict:
    return {"state": {int(i): s for i, s in sd["state"].items()}, "param_groups": sd["param_groups"]}


def _version_pair(v) -> tuple:
    return tuple(v) if isinstance(v, (tuple, list)) else (0, int(v))


def _safe_version(v):
    if isinstance(v, (list, tuple)) and len(v) == 2 and all(isinstance(x, int) and not isinstance(x, bool) for x in v):
        return int(v[0]), int(v[1])
    return None


_declared_shape = declared_shape


def _addr(a):
    return tuple(a) if isinstance(a, (list, tuple)) else a


# ===================================================================== parameter server
class ParameterServer(ReactorServer):
    _SEEN_GRANTS_MAX = 4096
    _PROPOSALS_MAX = 16       # live private-state proposals kept per key

    def __init__(self, config, owned_keys, diloco, *, host="0.0.0.0", port=0, auth_key=None, device="cpu",
                 resume_dir=None, grant_key=None, scheduler_pub=None, max_update_norm=None, compress="none",
                 identity=None, epoch_record=None, replicate_interval=10.0, peer_auth=None, bank_seed=0,
                 robustness="off", quorum_target=3, quorum_timeout=30.0, aggregate="trimmed_mean",
                 version_history=1, private_policy="overwrite", schedule_mode="central", down="full",
                 coordinates=None, scheduler_addr=None, peer_tls=None, private_quorum=2, salt="", k=3,
                 lease_ttl=20.0, read_quorum=1, directory_ttl=30.0, reputation=None, rate_limiter=None,
                 min_owner_reputation=0.0, corpus_weights=None, worker_set=None, staleness_bound=None,
                 staleness_weight="inverse", replica_audit_interval=30.0, sync_timeout=60.0, **kw):
        super().__init__(host=host, port=port, auth_key=auth_key, **kw)
        self.config, self.diloco, self.device = config, diloco, torch.device(device)
        self._topology = config.build_topology()
        self._paths = set(self._topology.paths())
        # an owner with an identity and no fixed keys is dynamic: it holds the whole seeded
        # bank and serves/writes only the keys the current epoch places on it
        self.dynamic = not owned_keys and identity is not None
        self.owned_keys = set(self._topology.module_keys()) if self.dynamic else set(owned_keys)
        self.grant_key, self.scheduler_pub = grant_key, scheduler_pub
        self.max_update_norm = max_update_norm
        self.compress = check_mode(compress)
        self.identity = identity
        self.peer_id = identity.peer_id if identity is not None else None
        self.peer_auth = peer_auth
        self.robust = robustness
        self.quorum_target, self.quorum_timeout = quorum_target, quorum_timeout
        self.aggregate = check_aggregate(aggregate)
        # delta-down needs past versions to diff against: a ring of 8 unless one was given
        self.version_history = max(1, int(version_history)) if down != "delta" or version_history > 1 else 8
        self.private_policy = private_policy
        if schedule_mode not in ("central", "decentralized"):
            raise ValueError(f"schedule_mode must be 'central' or 'decentralized', got {schedule_mode!r}")
        if schedule_mode == "decentralized" and self.compress != "none":
            # a worker's base must be the exact replica state that quorum reads confirm by
            # digest, so the down-link carries full-precision weights
            raise ValueError("schedule_mode='decentralized' needs compress='none'")
        self.schedule_mode = schedule_mode
        # decentralized coordination: the live worker set for the HRW-assignee check (a
        # callable; else the workers of the last tracker directory), the staleness bound in
        # base-version lag, and how often co-owner replicas are audited by digest
        self.worker_set = worker_set
        self.staleness_bound = 2 * self._topology.num_paths if staleness_bound is None else staleness_bound
        self.staleness_weight = staleness_weight
        self.replica_audit_interval = replica_audit_interval
        self._dir_workers: list = []
        self._last_audit = time.monotonic()
        self.down = down
        self.replicate_interval = replicate_interval
        self.scheduler_addr = _addr(scheduler_addr) if scheduler_addr is not None else None
        self.peer_tls, self.private_quorum = peer_tls, max(1, int(private_quorum))
        self.salt, self.k, self.lease_ttl, self.read_quorum = salt, k, lease_ttl, read_quorum
        self.directory_ttl = directory_ttl
        self.reputation = reputation or Reputation()
        self.rate_limiter = rate_limiter
        self.min_owner_reputation = min_owner_reputation
        self.corpus_weights = dict(corpus_weights) if corpus_weights else None
        self._tracker = None
        self._directory: dict = {}       # decentralized gossip: peer id -> newest signed record
        self._self_record = None
        self._hb_paused = threading.Event()  # set: stop refreshing the tracker record (suspend)
        full = build_module_bank(config, seed=bank_seed)
        self.bank = {k: full[k].to(self.device) for k in self.owned_keys}
        self._versions = {k: (0, 0) for k in self.bank}
        self._outer_opts = {k: make_outer_optimizer({k: m}, diloco) for k, m in self.bank.items()
                            if not is_private_key(k)}
        self._lock = threading.RLock()
        self._seen_grants: OrderedDict = OrderedDict()
        self._buffers: dict = {}
        self._buffer_ts: dict = {}
        self._history: dict = {k: collections.deque(maxlen=self.version_history) for k in self.bank}
        self._proposals: dict = {}
        self._saved: dict = {}
        self._epoch = None
        self._epoch_num = 0
        self._active = set() if self.dynamic else set(self.bank)
        self._draining = False
        self._repl_stop = threading.Event()
        self._repl_thread = None
        self._gen_counters: dict = {}   # path -> [open generation, monotonic time it opened]
        # a server without any authentication trusts every session (a closed test cluster);
        # otherwise exact state (weights + momentum) only goes to, and drains only come
        # from, sessions identity-authenticated as owners of the key
        self._open = self.auth_keys is None and self.admitted_peers is None
        # keys gained in a non-bootstrap epoch, waiting for a previous replica's state:
        # key -> (monotonic time of the first attempt, the epoch to sync from)
        self._syncing: dict = {}
        self.sync_timeout = sync_timeout
        self._coordinates = set(coordinates or [])
        # restarted from disk: before serving its first epoch's keys, this owner reconciles
        # them with their other replicas (the newest version wins), since a backup may have
        # trained past this owner's checkpoint
        self._resumed = bool(resume_dir)
        if resume_dir:
            if os.path.exists(os.path.join(resume_dir, self._shard_name())):
                self.load_shard(resume_dir)
            else:
                for k in list(self.bank):
                    self._load_module(k, resume_dir)
        if epoch_record is not None:
            self.apply_epoch(epoch_record)

    # -- dispatch -------------------------------------------------------------
    def _handle(self, msg: dict, nbytes: int, peer_id: str | None = None):
        kind = msg.get("type")
        if kind == "fetch":
            return self._fetch(msg, peer_id)
        if kind == "push":
            return self._push(msg, peer_id)
        if kind == "drain":
            return self._drain_recv(msg, peer_id)
        if kind == "digest":
            return self._digests(msg)
        if kind == "directory":
            return self._directory_rpc(msg)
        if kind == "commit":
            return self._commit(msg, peer_id)
        if kind == "generation":
            return self._generation(msg)
        if kind == "epoch":
            rec = msg.get("record")
            if not verify_epoch_record(rec, signer_pub=self.scheduler_pub,
                                       allow_deterministic=self.schedule_mode == "decentralized"):
                return {"type": "refused", "reason": "bad epoch record"}
            if self._epoch is not None and not epoch_newer(rec, self._epoch):
                return {"type": "ack", "stale": True}
            self.apply_epoch(rec)
            return {"type": "ack"}
        if kind == "checkpoint":
            if self._epoch is not None:
                return {"type": "ack", "versions": self.save_modules(msg["dir"])}
            self.save_shard(msg["dir"])
            return {"type": "ack"}
        if kind == "status":
            with self._lock:
                return {"type": "status", "epoch": self._epoch_num,
                        "versions": {k: self._versions[k] for k in self._active if k in self._versions}}
        return None

    # -- ownership ---------------------------------------------------------------
    def _primary(self, key) -> bool:
        if self._epoch is None:
            return not self.dynamic
        if self._draining or key not in self._active:
            return False
        owners = owners_for(key, self._epoch)
        return bool(owners) and owners[0]["peer_id"] == self.peer_id

    def _may_write(self, key) -> bool:
        if self.schedule_mode == "decentralized" and self._epoch is not None and not self._draining:
            return key in self.owned_keys and key in self._active
        return self._primary(key)

    def apply_epoch(self, record, *, bootstrap: bool | None = None) -> None:
        """Adopt an epoch: keys this peer is a replica of become active. Keys gained in a
        non-bootstrap epoch are first synced (highest version wins) from the replicas of
        the previous epoch, so a joining owner never serves its freshly seeded bank."""
        if not record:
            return
        boot = bool(record.get("bootstrap")) if bootstrap is None else bootstrap
        if not self._open:
            # the owners of a verified epoch may dial this server by identity
            for o in record.get("owners") or []:
                if isinstance(o.get("peer_id"), str):
                    self.admit_peer_id(o["peer_id"])
        with self._lock:
            prev = self._epoch
            act = {k for k in self.bank if self.peer_id in {o["peer_id"] for o in owners_for(k, record)}}
            gained = act - self._active
        pending = set()
        if gained and not boot and prev is not None:
            pending = set(gained) - self._sync_keys(sorted(gained), prev, record)
        elif gained and prev is None and self._resumed:
            # a restart: reconcile with the co-owners of the epoch it rejoins
            prev = record
            pending = set(gained) - self._sync_keys(sorted(gained), record, record)
        with self._lock:
            self._epoch = record
            self._epoch_num = int(record.get("epoch", 0))
            now = time.monotonic()
            self._syncing = {k: self._syncing.get(k, (now, prev)) for k in pending}
            self._active = act - pending

    def _sync_keys(self, keys, epoch, claim=None) -> set:
        """Pull the newest state of ``keys`` from their other replicas under ``epoch``,
        presenting ``claim`` (the epoch in which this owner holds them); returns the keys
        some replica answered for, and the keys no other replica holds (nothing to wait for)."""
        plan: dict = {}
        answered = set()
        for k in keys:
            others = [o for o in owners_for(k, epoch) if o["peer_id"] != self.peer_id]
            if not others:
                answered.add(k)
            for o in others:
                plan.setdefault(_addr(o["addr"]), []).append(k)
        for addr, ks in plan.items():
            msg = {"type": "fetch", "keys": ks, "include_state": True, "have": {}}
            if claim is not None:
                msg["epoch"] = claim
            try:
                reply = self._peer_rpc(addr, msg)
            except (OSError, ConnectionError, PermissionError):
                continue
            self._adopt(reply)
            answered |= set(reply.get("versions") or {}) & set(ks)
        return answered

    def _retry_sync(self) -> None:
        """Keys still syncing: ask the previous replicas again; a key none of them has
        answered for ``sync_timeout`` seconds is served from the local state (its
        replicas are gone, and waiting longer cannot bring the state back)."""
        with self._lock:
            todo, claim = dict(self._syncing), self._epoch
        if not todo:
            return
        done = set()
        for src in {id(e): e for _, e in todo.values()}.values():
            keys = sorted(k for k, (_, e) in todo.items() if e is src)
            done |= self._sync_keys(keys, src, claim)
        now = time.monotonic()
        expired = {k for k, (t0, _) in todo.items() if k not in done and now - t0 >= self.sync_timeout}
        if expired:
            logger.warning("no previous replica answered for %s within %.0fs: serving the local state",
                           sorted(expired), self.sync_timeout)
        with self._lock:
            for k in done | expired:
                if self._syncing.pop(k, None) is not None and claim is self._epoch and \
                        self.peer_id in {o["peer_id"] for o in owners_for(k, self._epoch)}:
                    self._active.add(k)

    def _state_allowed(self, key, peer_id, claim=None) -> bool:
        """May this session pull exact state of ``key`` or drain it here? Without an
        epoch (a fixed shard) or on an open server: yes. Otherwise only a session
        authenticated as an owner of the key, under this server's epoch or under a newer
        valid epoch the session presents (a new owner syncing before this server has
        seen that epoch)."""
        if self._epoch is None or self._open:
            return True
        if peer_id is None:
            return False
        if peer_id in {o["peer_id"] for o in owners_for(key, self._epoch)}:
            return True
        return (isinstance(claim, dict) and not epoch_newer(self._epoch, claim)
                and verify_epoch_record(claim, signer_pub=self.scheduler_pub,
                                        allow_deterministic=self.schedule_mode == "decentralized")
                and peer_id in {o["peer_id"] for o in owners_for(key, claim)})

    def _adopt(self, reply) -> dict:
        """Take every key of an ``include_state`` fetch reply that is newer than ours."""
        pulled = {}
        with self._lock:
            for k, sd in (reply.get("weights") or {}).items():
                v = _safe_version((reply.get("versions") or {}).get(k))
                if k in self.bank and v is not None and v > self._versions[k]:
                    self.bank[k].load_state_dict({n: t.to(self.device) for n, t in sd.items()})
                    st = (reply.get("state") or {}).get(k)
                    if st is not None and k in self._outer_opts:
                        self._outer_opts[k].load_state_dict(_opt_from_wire(st))
                    self._versions[k] = v
                    pulled[k] = v
        return pulled

    def _bump(self, key) -> None:
        e, c = self._versions[key]
        self._versions[key] = (self._epoch_num, c + 1 if e == self._epoch_num else 1)

    def _record_history(self, key) -> None:
        self._history[key].append((self._versions[key], _state_cpu(self.bank[key].state_dict())))

    def _pinned_state(self, key, version):
        if self._versions[key] == tuple(version):
            return _state_cpu(self.bank[key].state_dict())
        for v, sd in self._history[key]:
            if v == tuple(version):
                return sd
        return None

    # -- fetch ----------------------------------------------------------------
    def _down_payload(self, key, have):
        cur = _state_cpu(self.bank[key].state_dict())
        if self.down == "delta" and have:
            base = self._pinned_state(key, have)
            if base is not None:
                return {"delta": encode_state_delta(cur, base, "int4" if self.compress == "int4" else "int8"),
                        "base": list(have)}
        return compress_state(cur, self.compress)

    def _fetch(self, msg: dict, peer_id: str | None = None) -> dict:
        have, cold = msg.get("have", {}), msg.get("cold", False)
        want_state, pin = bool(msg.get("include_state")), msg.get("pin") or {}
        weights, versions, state, missing = {}, {}, {}, []
        with self._lock:
            for k in msg.get("keys", []):
                if k not in self.bank:
                    missing.append(k)
                    continue
                if k in pin:
                    snap = self._pinned_state(k, tuple(pin[k]))
                    if snap is None:
                        missing.append(k)
                    else:
                        weights[k], versions[k] = compress_state(snap, self.compress), tuple(pin[k])
                    continue
                if want_state:
                    if not self._state_allowed(k, peer_id, msg.get("epoch")):
                        missing.append(k)
                        continue
                    versions[k] = self._versions[k]
                    if tuple(have.get(k) or ()) != self._versions[k]:
                        weights[k] = _state_cpu(self.bank[k].state_dict())
                        if k in self._outer_opts:
                            state[k] = _opt_to_wire(_opt_state_cpu(self._outer_opts[k].state_dict()))
                    continue
                if k not in self._active:
                    missing.append(k)
                    continue
                if is_private_key(k):
                    if cold:
                        weights[k] = compress_state(_state_cpu(self.bank[k].state_dict()), self.compress)
                        versions[k] = self._versions[k]
                else:
                    versions[k] = self._versions[k]
                    if tuple(have.get(k) or ()) != self._versions[k]:
                        weights[k] = self._down_payload(k, tuple(have.get(k) or ()))
                    if self.version_history > 1:
                        self._record_keyframe(k)
        out = {"type": "weights", "weights": weights, "versions": versions}
        if want_state:
            out["state"] = state
        if missing:
            out["missing"] = missing
        return out

    def _record_keyframe(self, key) -> None:
        v = self._versions[key]
        if not any(hv == v for hv, _ in self._history[key]):
            self._record_history(key)

    # -- push -----------------------------------------------------------------
    def _expected_signer(self, grant):
        if self._epoch is None or not isinstance(grant, dict):
            return None
        path = grant.get("path")
        try:
            keys = self._topology.path_module_keys(tuple(path))
        except Exception:
            return None
        owners = owners_for(coordinator_key(keys), self._epoch)
        return owners[0]["peer_id"] if owners else None

    def _quorum_c(self, key) -> int:
        return max(1, min(self._topology.sharing_count(key), self.quorum_target))

    def _apply_outer(self, key, weight, grad) -> None:
        self._record_history(key)
        apply_outer_grads(self.bank[key], [weight * g.to(self.device) for g in grad])
        self._outer_opts[key].step()
        self._outer_opts[key].zero_grad(set_to_none=True)
        self._bump(key)

    def _flush_buffer(self, key) -> None:
        contribs = self._buffers.pop(key, None)
        self._buffer_ts.pop(key, None)
        if not contribs:
            return
        delta, wsum = robust_delta(contribs, aggregate=self.aggregate)
        self._record_history(key)
        apply_outer_grads(self.bank[key], [wsum * d.to(self.device) for d in delta])
        self._outer_opts[key].step()
        self._outer_opts[key].zero_grad(set_to_none=True)
        self._bump(key)

    def _sweep_buffers(self) -> None:
        if self.robust == "off":
            return
        now = time.monotonic()
        with self._lock:
            due = [k for k, ts in self._buffer_ts.items() if self._buffers.get(k) and now - ts >= self.quorum_timeout]
            for k in due:
                self._flush_buffer(k)

    def _private_ok(self, private) -> bool:
        for k, sd in private.items():
            if k not in self.bank or not isinstance(sd, dict):
                continue
            ref = self.bank[k].state_dict()
            if set(sd) != set(ref) or any(not torch.is_tensor(sd[n]) or sd[n].shape != ref[n].shape for n in ref):
                return False
        return True

    def _push(self, msg: dict, peer_id: str | None = None) -> dict:
        grant = msg.get("grant")
        ok = (grant_signed_by(grant, self._expected_signer(grant)) if self.schedule_mode == "decentralized"
              else verify_grant(grant, self.grant_key, scheduler_pub=self.scheduler_pub))
        if not ok:
            return {"type": "ack", "applied": False}
        raw, private = msg.get("updates") or {}, msg.get("private") or {}
        if not (isinstance(raw, dict) and isinstance(private, dict)):
            self.metrics.record_invalid_reject()
            return {"type": "ack", "applied": False}
        with self._lock:
            expected = {k: [tuple(p.shape) for p in self.bank[k].parameters()] for k in raw if k in self.bank}
        try:
            updates = {}
            for k, u in raw.items():
                shapes = expected.get(k)
                if shapes is None or not isinstance(u, dict):
                    continue
                grad = u.get("grad")
                if not isinstance(grad, list) or len(grad) != len(shapes) or any(
                        _declared_shape(p) != s for p, s in zip(grad, shapes)):
                    raise ValueError("grad payload shape mismatch")
                updates[k] = maybe_dequantize(grad)
        except (TypeError, KeyError, ValueError):
            self.metrics.record_invalid_reject()
            return {"type": "ack", "applied": False}
        weight, allowed = float(grant["weight"]), set(grant["keys"])
        skipped, applied = [], 0
        with self._lock:
            if grant["token"] in self._seen_grants:
                return {"type": "ack", "applied": False}
            self._seen_grants[grant["token"]] = True
            while len(self._seen_grants) > self._SEEN_GRANTS_MAX:
                self._seen_grants.popitem(last=False)
            if not (all_finite(updates) and all_finite(private) and self._private_ok(private)):
                self.metrics.record_invalid_reject()
                return {"type": "ack", "applied": False}
            for k, grad in updates.items():
                if is_private_key(k) or k not in allowed:
                    continue
                if k not in self.owned_keys or not self._may_write(k):
                    skipped.append(k)
                    continue
                if self.max_update_norm is not None and clip_norm_(grad, self.max_update_norm) > self.max_update_norm:
                    self.metrics.record_norm_clip()
                if self.robust == "off":
                    self._apply_outer(k, weight, grad)
                else:
                    buf = self._buffers.setdefault(k, [])
                    buf.append((weight, [g.to(self.device) for g in grad]))
                    self._buffer_ts.setdefault(k, time.monotonic())
                    if len(buf) >= self._quorum_c(k):
                        self._flush_buffer(k)
                applied += 1
            for k, sd in private.items():
                if k not in allowed:
                    continue
                if k not in self.owned_keys or not self._may_write(k):
                    skipped.append(k)
                    continue
                if self.private_policy == "proposal":
                    # apply only once private_quorum distinct proposers (peer identity, or the
                    # single-use grant without one) agree byte for byte; one live proposal per
                    # proposer, at most _PROPOSALS_MAX per key (the oldest are dropped)
                    dg = state_digest(sd)
                    props = self._proposals.setdefault(k, collections.OrderedDict())
                    who = peer_id or grant["token"]
                    props[who] = (dg, sd)
                    props.move_to_end(who)
                    while len(props) > self._PROPOSALS_MAX:
                        props.popitem(last=False)
                    if sum(1 for d, _ in props.values() if d == dg) >= self.private_quorum:
                        self._record_history(k)
                        self.bank[k].load_state_dict({n: v.to(self.device) for n, v in sd.items()})
                        self._bump(k)
                        self._proposals.pop(k, None)
                    applied += 1
                    continue
                self._record_history(k)
                self.bank[k].load_state_dict({n: v.to(self.device) for n, v in sd.items()})
                self._bump(k)
                applied += 1
            ep = self._epoch_num
        if skipped:
            return {"type": "ack", "applied": applied > 0, "skipped": sorted(skipped), "reason": "not_primary",
                    "epoch": ep}
        return {"type": "ack", "applied": True}

    # -- decentralized coordination (path primary mints grants) ----------------
    def _path_or_none(self, raw):
        try:
            path = tuple(int(i) for i in raw)
        except (TypeError, ValueError):
            return None
        return path if path in self._paths else None

    def _coordinates_path(self, path) -> bool:
        """Decentralized: this owner coordinates ``path`` when it is the active primary of
        the path's coordinator key (the path's private key when it has one)."""
        if self.schedule_mode != "decentralized" or self._epoch is None:
            return False
        return self._primary(coordinator_key(self._topology.path_module_keys(path)))

    def generation_of(self, path) -> int:
        """The open generation of ``path`` on this owner (its coordinator's is the truth)."""
        with self._lock:
            return self._gen_counters.get(tuple(path), (0, 0.0))[0]

    def _worker_ids(self) -> list:
        if self.worker_set is not None:
            return sorted(set(self.worker_set() or []))
        return list(self._dir_workers)

    def _generation(self, msg: dict) -> dict:
        """The path's open generation and how long it has been open (``age``): a worker
        feeds the age to the same takeover rule the coordinator applies at commit, so the
        two agree without sharing a clock."""
        path = self._path_or_none(msg.get("path"))
        if path is None:
            return {"type": "generation", "ok": False}
        with self._lock:
            if not self._coordinates_path(path):
                return {"type": "generation", "ok": False, "reason": "not_coordinator", "epoch": self._epoch_num}
            gen, opened = self._gen_counters.setdefault(path, [0, time.monotonic()])
            return {"type": "generation", "ok": True, "generation": gen, "age": max(0.0, time.monotonic() - opened),
                    "epoch": self._epoch_num, "lease_ttl": self.lease_ttl, "staleness_bound": self.staleness_bound}

    def _commit(self, msg: dict, peer_id: str | None = None) -> dict:
        """Decentralized commit of ``(path, gen_id)`` to the path's coordinating owner.

        Gates, in order: this owner coordinates the path; the generation is the open one
        (a version fence: the slot closes at the first accepted commit); the committer is
        the HRW assignee of the slot over the live worker set, or its successor once the
        slot has been open ``lease_ttl`` per rank (skipped without a worker set); the rate
        limit at the committer's reputation; a finite loss; the lag of the committer's
        base versions behind this owner's (same epoch, at most ``staleness_bound``). An
        accepted commit advances the generation and returns a grant signed with this
        owner's identity, which the path's co-owners check against the epoch. Reference
        behaviour: ``src/opendipaco/schedule/sharded.py:1328-1408``."""
        def nack(reason, **extra):
            return {"type": "commit_ack", "accepted": False, "reason": reason, **extra}

        if self.schedule_mode != "decentralized" or self.identity is None:
            return nack("not_decentralized")
        path = self._path_or_none(msg.get("path"))
        if path is None:
            return nack("bad_path")
        member = peer_id or msg.get("worker_id")
        outcome = None
        try:
            with self._lock:
                if not self._coordinates_path(path):
                    return nack("not_coordinator", epoch=self._epoch_num)
                slot = self._gen_counters.setdefault(path, [0, time.monotonic()])
                gen, opened = slot
                if msg.get("gen_id") != gen:
                    return nack("stale_generation", generation=gen)
                workers = self._worker_ids()
                if workers and not is_assignee(member, path, gen, workers, salt=self.salt,
                                               elapsed=time.monotonic() - opened, lease_ttl=self.lease_ttl):
                    return nack("not_assignee")
                if self.rate_limiter is not None and not self.rate_limiter.allow(
                        peer_id, reputation=self.reputation.get(peer_id)):
                    return nack("throttled")
                if not loss_ok(msg.get("loss"), empty=bool(msg.get("empty"))):
                    self.metrics.record_invalid_reject()
                    outcome = False
                    return nack("bad_loss")
                base = msg.get("base_versions")
                base = base if isinstance(base, dict) else {}
                held = {k: self._versions[k] for k in base if k in self._active}
                theirs = {k: _safe_version(base[k]) for k in held}
                lag = None if any(v is None for v in theirs.values()) else version_lag(theirs, held)
                if lag is None or lag > self.staleness_bound:
                    self.metrics.record_stale_reject()
                    return nack("stale")
                slot[0], slot[1] = gen + 1, time.monotonic()
                if self.corpus_weights is not None:
                    w = float(self.corpus_weights.get(self._topology.path_index(path), 0.0))
                else:
                    w = as_finite_float(msg.get("weight"))
                    w = 1.0 if w is None else min(max(w, 0.0), 1.0)
                if self.staleness_weight == "inverse":
                    w /= 1.0 + lag
                grant = make_grant(path, self._topology.path_module_keys(path), w, uuid.uuid4().hex,
                                   identity=self.identity)
                self.metrics.record_update(lag)
                outcome = True
                return {"type": "commit_ack", "accepted": True, "generation": gen + 1, "grant": grant,
                        "push_weight": w}
        finally:
            if outcome is True:
                self.reputation.credit(peer_id)
            elif outcome is False:
                self.reputation.debit(peer_id)

    def audit_replicas_once(self) -> dict:
        """Decentralized: compare this owner's ``(version, digest)`` of every active key
        with its co-owners'. A replica whose digest at the version a quorum confirms
        differs loses reputation -- with ``min_owner_reputation`` set it then drops out of
        the next derived epoch. A co-owner that does not answer is not blamed, nor is one
        that is only behind. Returns ``{key: flagged peer ids}``."""
        if self.schedule_mode != "decentralized" or self._epoch is None or self.peer_id is None:
            return {}
        with self._lock:
            keys, epoch = sorted(self._active), self._epoch
        reports = {k: {self.peer_id: (tuple(v), d)} for k, (v, d) in self._digests({"keys": keys})["digests"].items()}
        asks: dict = {}
        for k in keys:
            for o in owners_for(k, epoch):
                if o["peer_id"] != self.peer_id and o.get("addr"):
                    asks.setdefault((o["peer_id"], _addr(o["addr"])), []).append(k)
        for (pid, addr), ks in asks.items():
            try:
                reply = self._peer_rpc(addr, {"type": "digest", "keys": ks})
            except (OSError, ConnectionError, PermissionError):
                continue
            for k, rep in (reply.get("digests") or {}).items():
                if k in reports and k in ks and isinstance(rep, (list, tuple)) and len(rep) == 2:
                    v = _safe_version(rep[0])
                    if v is not None and isinstance(rep[1], str):
                        reports[k][pid] = (v, rep[1])
        return self.apply_replica_audit(reports)

    def apply_replica_audit(self, reports: dict) -> dict:
        """The audit rule on gathered ``{key: {peer_id: (version, digest)}}`` reports."""
        flagged = {}
        q = max(2, self.read_quorum)
        for k, by_peer in reports.items():
            bad = divergent_peers(by_peer, confirm_version(list(by_peer.values()), q))
            for pid in bad:
                self.reputation.debit(pid)
            if bad:
                flagged[k] = bad
        return flagged

    def _digests(self, msg: dict) -> dict:
        out = {}
        with self._lock:
            for k in msg.get("keys", []):
                if k in self.bank:
                    out[k] = [list(self._versions[k]), state_digest(_state_cpu(self.bank[k].state_dict()))]
        return {"type": "digests", "digests": out}

    # -- replication ------------------------------------------------------------
    def _drain_recv(self, msg: dict, peer_id: str | None = None) -> dict:
        """A leaving primary's newest state, adopted when strictly newer and sent by an
        owner of the key. Refused in decentralized mode: a pushed version is not
        quorum-confirmed there, so a Byzantine owner could poison its co-owners."""
        adopted = []
        if self.schedule_mode == "decentralized":
            return {"type": "drained", "adopted": adopted}
        with self._lock:
            for k, p in (msg.get("states") or {}).items():
                if k not in self.bank or not isinstance(p, dict) or not self._state_allowed(k, peer_id):
                    continue
                v, sd = _safe_version(p.get("version")), p.get("weights")
                if v is None or sd is None or v <= self._versions[k]:
                    continue
                self.bank[k].load_state_dict({n: t.to(self.device) for n, t in sd.items()})
                if p.get("state") is not None and k in self._outer_opts:
                    self._outer_opts[k].load_state_dict(_opt_from_wire(p["state"]))
                self._versions[k] = v
                adopted.append(k)
        return {"type": "drained", "adopted": adopted}

    def _peer_cred(self):
        """What this owner presents when dialing another owner: ``peer_auth`` when given,
        else its identity (so the other side can gate exact state on the session), else
        the shared key; nothing towards open servers."""
        if self.peer_auth is not None:
            return self.peer_auth
        if self._open:
            return None
        return self.identity if self.identity is not None else self.auth_key

    def _peer_rpc(self, addr, msg, timeout: float = 5.0):
        cred = self._peer_cred()
        s = connect(_addr(addr), cred, timeout=timeout, tls=self.peer_tls)
        try:
            return rpc(s, msg)
        finally:
            s.close()

    def _replicate_once(self) -> dict:
        """Pull exact state (weights + momentum) for keys this peer backs up."""
        pulled = {}
        if self._epoch is None:
            return pulled
        with self._lock:
            plan = {}
            for k in self._active:
                owners = owners_for(k, self._epoch)
                if owners and owners[0]["peer_id"] != self.peer_id:
                    plan.setdefault(_addr(owners[0]["addr"]), []).append(k)
            have = dict(self._versions)
        for addr, keys in plan.items():
            try:
                reply = self._peer_rpc(addr, {"type": "fetch", "keys": keys, "include_state": True,
                                              "have": {k: list(have[k]) for k in keys}, "epoch": self._epoch})
            except (OSError, ConnectionError, PermissionError):
                continue
            if self.schedule_mode == "decentralized" and self.read_quorum > 1:
                reply = self._quorum_filter(reply, addr)
            pulled.update(self._adopt(reply))
        return pulled

    def _quorum_filter(self, reply: dict, source) -> dict:
        """Decentralized: keep only pulled states that ``read_quorum`` replicas (the
        source included) report at the same ``(version, digest)``, so one Byzantine
        primary cannot poison its backups through replication."""
        weights = dict(reply.get("weights") or {})
        with self._lock:
            epoch = self._epoch
        for k in list(weights):
            v = _safe_version((reply.get("versions") or {}).get(k))
            want = (v, state_digest(weights[k])) if v is not None else None
            votes = 1 if want is not None else 0
            for o in owners_for(k, epoch):
                if want is None or votes >= self.read_quorum:
                    break
                if o["peer_id"] == self.peer_id or _addr(o["addr"]) == _addr(source):
                    continue
                try:
                    rep = (self._peer_rpc(o["addr"], {"type": "digest", "keys": [k]}).get("digests") or {}).get(k)
                except (OSError, ConnectionError, PermissionError):
                    continue
                if isinstance(rep, (list, tuple)) and len(rep) == 2 and (_safe_version(rep[0]), rep[1]) == want:
                    votes += 1
            if votes < self.read_quorum:
                weights.pop(k)
        return dict(reply, weights=weights)

    def _poll_scheduler_epoch(self) -> None:
        if self.scheduler_addr is None:
            return
        try:
            cred = self.auth_key if self.auth_key is not None else self.identity
            s = connect(self.scheduler_addr, cred, timeout=5.0, tls=self.peer_tls)
            try:
                rec = rpc(s, {"type": "epoch_get"}).get("record")
            finally:
                s.close()
        except (OSError, ConnectionError, PermissionError):
            return
        if rec and verify_epoch_record(rec, signer_pub=self.scheduler_pub) and epoch_newer(rec, self._epoch):
            self.apply_epoch(rec)

    def import_directory(self, records) -> int:
        """Merge signed peer records into this owner's directory (gossip): a record
        replaces its peer's held one only when newer, and records older than
        ``directory_ttl`` are not taken. Returns how many were taken."""
        now, taken = time.time(), 0
        with self._lock:
            for r in records or []:
                if not (verify_record(r) and r.get("kind") == "peer"):
                    continue
                ts = record_issued_at(r)
                if ts is None or now - ts > self.directory_ttl:
                    continue
                held = self._directory.get(r["peer_id"])
                if held is None or ts > record_issued_at(held):
                    self._directory[r["peer_id"]] = r
                    taken += 1
        return taken

    def directory(self) -> list:
        """The live records this owner knows (its own first), stale ones dropped."""
        now = time.time()
        with self._lock:
            for pid in [p for p, r in self._directory.items() if now - record_issued_at(r) > self.directory_ttl]:
                del self._directory[pid]
            recs = [r for p, r in self._directory.items() if p != self.peer_id]
        own = self._self_record
        return ([own] if own is not None else []) + recs

    def _directory_rpc(self, msg: dict) -> dict:
        return {"type": "directory", "records": self.directory()}

    def _derive_from_directory(self) -> None:
        """Decentralized: gather signed peer records from the trackers (bootstrap seeds)
        and from the current co-owners' directories (gossip), then derive the epoch that
        every owner derives from the same records. With the trackers gone the owners
        keep converging through one another."""
        if self._tracker is None or self.schedule_mode != "decentralized":
            return
        from .tracker import fetch_directory

        wait = min(2.0, self.directory_ttl / 4)  # a dead seed or peer must not stall the pass
        for a in self._tracker["all"]:
            try:
                self.import_directory(fetch_directory(a, auth_key=self._tracker["auth"], tls=self._tracker["tls"],
                                                      timeout=wait))
            except (OSError, ConnectionError, PermissionError):
                continue
        with self._lock:
            peers = {o["peer_id"]: o["addr"] for o in (self._epoch or {}).get("owners", []) if o.get("addr")}
        for pid, addr in peers.items():
            if pid == self.peer_id:
                continue
            try:
                self.import_directory(self._peer_rpc(addr, {"type": "directory"}, timeout=wait).get("records"))
            except (OSError, ConnectionError, PermissionError):
                continue
        everyone = self.directory()
        if not everyone:
            return
        self._dir_workers = _worker_directory_ids(everyone)
        recs = [r for r in everyone if "owner" in (r.get("roles") or [])]
        eligible = (lambda pid: self.reputation.get(pid) >= self.min_owner_reputation) \
            if self.min_owner_reputation else None
        prev = self._epoch if self._epoch is not None and self._epoch.get("deterministic") else None
        nxt = derive_epoch(recs, k=self.k, salt=self.salt, prev=prev, is_eligible=eligible)
        if nxt is not prev and nxt["owners"]:
            self.apply_epoch(nxt)

    def _replicate_loop(self) -> None:
        while not self._repl_stop.wait(self.replicate_interval):
            try:
                self._sweep_buffers()
                self._poll_scheduler_epoch()
                self._derive_from_directory()
                self._retry_sync()
                self._replicate_once()
                if (self.schedule_mode == "decentralized"
                        and time.monotonic() - self._last_audit >= self.replica_audit_interval):
                    self._last_audit = time.monotonic()
                    self.audit_replicas_once()
            except Exception:
                logger.exception("replication pass failed")

    def start(self) -> None:
        super().start()
        if self._epoch is not None or self.robust != "off" or self.dynamic or self.scheduler_addr is not None:
            self._repl_thread = threading.Thread(target=self._replicate_loop, daemon=True)
            self._repl_thread.start()
            if self.scheduler_addr is not None:
                threading.Thread(target=self._poll_scheduler_epoch, daemon=True).start()

    def start_tracker_heartbeat(self, tracker_addr, advertise_host, *, interval=10.0, auth_key=None, tls=None,
                                seeds=(), circuit_addrs=None):
        """Keep this owner's signed record registered on the tracker(s) (re-register every
        ``interval`` s, below the tracker's TTL); deregistered on a graceful shutdown.
        With ``circuit_addrs`` (from :func:`relay.serve_via_relays`) the owner registers
        as a ``nat`` peer reachable through those relays instead of at
        ``advertise_host``."""
        from .tracker import dedup_seeds

        if self.identity is None:
            raise ValueError("a tracker heartbeat needs an owner identity")
        addrs = dedup_seeds(tuple(tracker_addr), seeds)
        self._tracker = {"addr": addrs[0], "all": addrs, "auth": auth_key, "tls": tls}
        stop = self._repl_stop

        from .tracker import make_peer_record, tracker_rpc

        def beat():
            while True:
                if not self._hb_paused.is_set():
                    # a fresh signed record each beat: registered on the trackers and served to
                    # co-owners that gossip directories (decentralized mode)
                    if circuit_addrs:
                        rec = make_peer_record(self.identity, reachability="nat", circuit_addrs=list(circuit_addrs),
                                               roles=["owner"])
                    else:
                        rec = make_peer_record(self.identity, reachability="public",
                                               addr=(advertise_host, self.port), roles=["owner"])
                    self._self_record = rec
                    for a in addrs:  # a dead tracker must not hold back the next beat
                        try:
                            tracker_rpc(a, {"type": "register", "record": rec}, auth_key=auth_key, tls=tls,
                                        timeout=min(5.0, max(0.5, interval)))
                        except (OSError, ConnectionError, PermissionError):
                            continue
                if stop.wait(interval):
                    return

        threading.Thread(target=beat, daemon=True).start()

    def pause_heartbeat(self) -> None:
        """Stop re-registering on the tracker while the server keeps serving: a
        deterministic suspend for failure tests. The record lapses after the tracker's
        TTL, as a sleeping laptop's would."""
        self._hb_paused.set()

    def resume_heartbeat(self) -> None:
        """Re-register again after :meth:`pause_heartbeat` (the machine woke up)."""
        self._hb_paused.clear()

    def _drain_to_backups(self) -> dict:
        """A leaving primary pushes its latest state to each key's next owner."""
        sent = {}
        if self._epoch is None:
            return sent
        with self._lock:
            plan = {}
            for k in self._active:
                owners = owners_for(k, self._epoch)
                if owners and owners[0]["peer_id"] == self.peer_id and len(owners) > 1:
                    plan.setdefault(_addr(owners[1]["addr"]), {})[k] = {
                        "version": list(self._versions[k]), "weights": _state_cpu(self.bank[k].state_dict()),
                        "state": _opt_to_wire(_opt_state_cpu(self._outer_opts[k].state_dict()))
                        if k in self._outer_opts else None}
            self._draining = True
        for addr, states in plan.items():
            try:
                sent[addr] = self._peer_rpc(addr, {"type": "drain", "states": states}).get("adopted", [])
            except (OSError, ConnectionError, PermissionError):
                continue
        return sent

    def shutdown(self, *, graceful: bool = False) -> None:
        if graceful:
            with self._lock:
                for k in list(self._buffers):
                    self._flush_buffer(k)
            self._drain_to_backups()
            if self._tracker is not None:
                from .tracker import deregister_peer

                for a in self._tracker["all"]:
                    try:
                        deregister_peer(a, self.identity, auth_key=self._tracker["auth"], tls=self._tracker["tls"],
                                        timeout=5.0)
                    except (OSError, ConnectionError, PermissionError):
                        continue
        self._repl_stop.set()
        super().shutdown()

    def simulate_crash(self) -> None:
        """A killed owner: connections drop, and with the process gone its replication
        loop and tracker heartbeat stop too (no drain, no deregistration), so the record
        lapses after the tracker's TTL."""
        self._repl_stop.set()
        super().simulate_crash()

    # -- persistence ------------------------------------------------------------
    @staticmethod
    def _module_file(key: str) -> str:
        return f"module_{hashlib.sha256(key.encode()).hexdigest()[:16]}.pt"

    def save_modules(self, dirpath: str) -> dict:
        os.makedirs(dirpath, exist_ok=True)
        saved, blobs = {}, {}
        with self._lock:
            for k in list(self._buffers):
                self._flush_buffer(k)
            for k in self.bank:
                v = self._versions[k]
                saved[k] = v
                if self._saved.get((dirpath, k)) == v:
                    continue
                opt = self._outer_opts.get(k)
                blobs[k] = {"key": k, "version": list(v), "weights": _state_cpu(self.bank[k].state_dict()),
                            "outer_opt": _opt_state_cpu(opt.state_dict()) if opt is not None else None}
        for k, blob in blobs.items():
            tmp = os.path.join(dirpath, self._module_file(k) + ".tmp")
            torch.save(blob, tmp)
            os.replace(tmp, os.path.join(dirpath, self._module_file(k)))
            self._saved[(dirpath, k)] = tuple(blob["version"])
        return saved

    def _load_module(self, key: str, dirpath: str) -> bool:
        p = os.path.join(dirpath, self._module_file(key))
        if not os.path.exists(p):
            return False
        blob = torch.load(p, map_location=self.device, weights_only=True)
        self.bank[key].load_state_dict({n: v.to(self.device) for n, v in blob["weights"].items()})
        self._versions[key] = _version_pair(blob["version"])
        if blob.get("outer_opt") is not None and key in self._outer_opts:
            self._outer_opts[key].load_state_dict(blob["outer_opt"])
        return True

    def _shard_name(self) -> str:
        return f"shard_{hashlib.sha256(','.join(sorted(self.owned_keys)).encode()).hexdigest()[:16]}.pt"

    def save_shard(self, dirpath: str) -> None:
        os.makedirs(dirpath, exist_ok=True)
        with self._lock:
            for k in list(self._buffers):
                self._flush_buffer(k)
            blob = {"weights": {k: _state_cpu(m.state_dict()) for k, m in self.bank.items()},
                    "versions": dict(self._versions),
                    "outer_opts": {k: _opt_state_cpu(o.state_dict()) for k, o in self._outer_opts.items()}}
        tmp = os.path.join(dirpath, self._shard_name() + ".tmp")
        torch.save(blob, tmp)
        os.replace(tmp, os.path.join(dirpath, self._shard_name()))

    def load_shard(self, dirpath: str) -> None:
        blob = torch.load(os.path.join(dirpath, self._shard_name()), map_location=self.device, weights_only=True)
        with self._lock:
            for k, sd in blob["weights"].items():
                if k in self.bank:
                    self.bank[k].load_state_dict({n: v.to(self.device) for n, v in sd.items()})
            self._versions.update({k: _version_pair(v) for k, v in blob["versions"].items() if k in self._versions})
            for k, sd in blob.get("outer_opts", {}).items():
                if k in self._outer_opts:
                    self._outer_opts[k].load_state_dict(sd)


# ============================================================================ scheduler
class Scheduler(ReactorServer):
    """Task queue + clock + staleness + grants; holds no weights."""

    def __init__(self, config, corpus, ps_addrs, diloco, batch_size, *, host="0.0.0.0", port=0, auth_key=None,
                 seed=0, staleness_bound=None, staleness_weight="inverse", heartbeat_timeout=30.0, grant_key=None,
                 identity=None, compress="none", idle_backoff=None, reputation=None, rate_limiter=None,
                 redundancy=3, redundancy_rate=0.0, audit_timeout=60.0, private_policy="overwrite", down="full",
                 up_density=1.0, task_seconds=None, park_factor=3.0, min_task_rate=None, tailor_bandwidth=False,
                 probe=None, probe_quorum=0, probe_abs_margin=0.05, probe_rel_margin=0.02, probe_debit=False,
                 ps_tls=None, min_owner_reputation=0.0, **kw):
        super().__init__(host=host, port=port, auth_key=auth_key, **kw)
        self.config, self.corpus, self.diloco, self.batch_size = config, corpus, diloco, batch_size
        self.topology = config.build_topology()
        self.seed = seed
        npaths = self.topology.num_paths
        self.staleness_bound = staleness_bound if staleness_bound is not None else 2 * npaths
        self.staleness_weight, self.heartbeat_timeout = staleness_weight, heartbeat_timeout
        self.grant_key, self.identity = grant_key, identity
        self.compress = check_mode(compress)
        self.idle_backoff, self.down, self.up_density = idle_backoff, down, up_density
        self.reputation = reputation or Reputation()
        self.rate_limiter = rate_limiter or RateLimiter(capacity=1e9, refill_per_sec=1e9)
        self.redundancy, self.redundancy_rate, self.audit_timeout = redundancy, redundancy_rate, audit_timeout
        self.private_policy = private_policy
        self.task_seconds, self.park_factor, self.min_task_rate = task_seconds, park_factor, min_task_rate
        self.tailor_bandwidth = tailor_bandwidth
        self._probe = probe if isinstance(probe, TrustedProbe) or probe is None else TrustedProbe(probe)
        self.probe_quorum, self.probe_debit = probe_quorum, probe_debit
        self.probe_margin = {"abs_margin": probe_abs_margin, "rel_margin": probe_rel_margin}
        self.ps_tls, self.min_owner_reputation = ps_tls, min_owner_reputation
        self._ps_addrs = [_addr(a) for a in ps_addrs or []]
        keys = self.topology.module_keys()
        self._static_routing = ({k: self._ps_addrs[i] for k, i in assign_shards(keys, len(self._ps_addrs)).items()}
                                if self._ps_addrs else {})
        self._routing = dict(self._static_routing)
        self._epoch_record = None
        self._lock = threading.RLock()
        self._serving = False
        self._T = self._target = 0
        self.total_rounds = None
        self._completed: dict = {}
        self._inflight: dict = {}
        self._issued: dict = {}
        self._lease: dict = {}
        self._owner: dict = {}
        self._lease_at: dict = {}
        self._lease_work: dict = {}
        self._worker_caps: dict = {}
        self._worker_rate: dict = {}
        self._parked: dict = {}
        self._audits: dict = {}
        self._manifest = None          # run manifest served to `opendipaco join`
        self._recovery = None          # signed recovery manifest of the last cluster checkpoint
        self._epoch_floor = 0          # epochs published after a restart number from here

    def _handle(self, msg: dict, nbytes: int, peer_id: str | None = None):
        kind = msg.get("type")
        if kind == "request":
            return self._next_task(msg, peer_id)
        if kind == "commit":
            return self._commit(msg, peer_id)
        if kind == "nack":
            return self._nack(msg)
        if kind == "heartbeat":
            self._heartbeat(msg)
            return None
        if kind == "routing":
            return self._fresh_routing(msg)
        if kind == "manifest":
            return {"type": "manifest", "manifest": self._manifest}
        if kind == "epoch_get":
            with self._lock:
                return {"type": "epoch", "record": self._epoch_record}
        return None

    def serve_manifest(self, manifest) -> None:
        self._manifest = manifest

    # -- epochs ----------------------------------------------------------------
    def publish_epoch(self, owner_records, *, k=3, salt="", bootstrap=None) -> dict:
        """Sign an epoch over ``owner_records`` and route future tasks by it."""
        if self.identity is None:
            raise ValueError("publishing an epoch needs a scheduler identity")
        with self._lock:
            num = max(self._epoch_floor, 0 if self._epoch_record is None else self._epoch_record["epoch"] + 1)
            rec = make_epoch_record(self.identity, epoch=num, owner_records=owner_records, k=k, salt=salt,
                                    bootstrap=bool(bootstrap) if bootstrap is not None else num == 0)
            self._epoch_record = rec
            self._routing = {}
        for o in rec["owners"]:
            try:
                s = connect(_addr(o["addr"]), self.auth_key, timeout=5.0, tls=self.ps_tls)
                try:
                    rpc(s, {"type": "epoch", "record": rec})
                finally:
                    s.close()
            except (OSError, ConnectionError, PermissionError):
                continue
        return rec

    def watch_tracker(self, tracker_addr, *, k=3, salt="", owner_grace=240.0, min_epoch_interval=60.0,
                      poll_interval=5.0, tracker_auth=None, tracker_tls=None):
        """Publish a signed epoch whenever the tracker's live owner set changes
        (hysteresis and rate limit of ``EpochManager``; owners below
        ``min_owner_reputation`` are left out)."""
        from .tracker import fetch_directory_and_tombstones

        eligible = (lambda pid: self.reputation.get(pid) >= self.min_owner_reputation) \
            if self.min_owner_reputation else None
        mgr = EpochManager(owner_grace=owner_grace, min_epoch_interval=min_epoch_interval, is_eligible=eligible)
        stop = threading.Event()

        def watch():
            while not self._stop:
                try:
                    recs, tombs = fetch_directory_and_tombstones(tuple(tracker_addr), roles=["owner"],
                                                                 auth_key=tracker_auth, tls=tracker_tls)
                    nxt = mgr.observe(recs, tombstoned=tombs)
                    if nxt:
                        self.publish_epoch(nxt, k=k, salt=salt)
                except Exception:
                    logger.exception("tracker watch pass failed")
                if stop.wait(poll_interval):
                    return

        threading.Thread(target=watch, daemon=True).start()
        return stop

    def _routing_locked(self, keys) -> dict:
        if self._epoch_record is not None:
            return {k: [o["addr"] for o in owners_for(k, self._epoch_record)] for k in keys}
        return {k: [self._routing[k]] for k in keys}

    def _fresh_routing(self, msg: dict) -> dict:
        with self._lock:
            keys = [k for k in msg.get("keys", []) if k in set(self.topology.module_keys())]
            return {"type": "routing", "routing": self._routing_locked(keys)}

    def _idle(self) -> dict:
        return {"type": "idle", **({"retry_in": self.idle_backoff} if self.idle_backoff is not None else {})}

    # -- task sizing (EMA effective rate) ---------------------------------------
    def _record_rate(self, wid, work, elapsed) -> None:
        if wid is None or not work or work <= 0 or elapsed <= 0:
            return
        r = work / elapsed
        prev = self._worker_rate.get(wid)
        self._worker_rate[wid] = r if prev is None else (1 - _RATE_EMA) * prev + _RATE_EMA * r

    def worker_rate(self, wid):
        with self._lock:
            return self._worker_rate.get(wid)

    def _size_task(self, wid, batch_cap):
        inner = self.diloco.inner_steps
        rate = self._worker_rate.get(wid)
        if not self.task_seconds or not rate:
            return batch_cap, inner
        budget = rate * self.task_seconds / self.config.sequence_length  # sequences in the window
        batch = max(1, min(batch_cap, int(budget // max(inner, 1))))
        if batch * inner > budget and batch == 1:
            inner = max(1, int(budget))
        return batch, inner

    def _too_slow(self, wid) -> bool:
        rate = self._worker_rate.get(wid)
        return self.min_task_rate is not None and rate is not None and rate < self.min_task_rate

    # -- tasks ---------------------------------------------------------------------
    def _next_task(self, req: dict, peer_id: str | None = None) -> dict:
        wid = req.get("worker_id")
        warm = {tuple(p) for p in req.get("warm_paths", [])}
        cached = {tuple(p) for p in req.get("cached_shards", [])}
        caps = req.get("capabilities") or {}
        check_only = audit = False
        base = None
        with self._lock:
            if caps:
                self._worker_caps[wid] = caps
            if not self._serving or self._T >= self._target:
                return {"type": "stop"} if self._stop else self._idle()
            if not self._routing and self._epoch_record is None:
                return self._idle()
            self._reclaim_locked()
            member = peer_id or wid
            rep = self.reputation.get(peer_id)
            cap = max(1, min(self.batch_size, int(caps["max_batch"]))) if caps.get("max_batch") else self.batch_size
            batch, inner = self._size_task(wid, cap)
            if self._too_slow(wid):
                now = time.monotonic()
                last = self._parked.get(wid)
                t_task = batch * inner * self.config.sequence_length / self._worker_rate[wid]
                if last is not None and now - last < self.park_factor * t_task:
                    return self._idle()
                self._parked[wid] = now
            eligible = [p for p in self._completed if p not in self._inflight]
            if not self.rate_limiter.allow(peer_id, reputation=rep):
                return self._idle()
            if not eligible:
                cand = next((k for k, a in self._audits.items() if a["base"] is not None and
                             member not in a["members"] and len(a["members"]) - 1 < a["target"]), None)
                if cand is None:
                    return self._idle()
                a = self._audits[cand]
                a["members"].add(member)
                path, generation = cand
                lease = uuid.uuid4().hex
                a.setdefault("check_leases", {})[member] = lease
                base, check_only = a["base"], True
                batch, inner = a["batch"], a["inner"]
            else:
                path = min(eligible, key=lambda p: (self._completed[p], p not in warm, p))
                lease = uuid.uuid4().hex
                self._owner[path], self._lease[path] = wid, lease
                self._inflight[path] = time.monotonic() + self.heartbeat_timeout
                self._issued[path] = self._T
                self._lease_at[path] = time.monotonic()
                self._lease_work[path] = batch * inner * self.config.sequence_length
                generation = self._completed[path]
                if (self.redundancy > 1 and self.redundancy_rate > 0 and random.random() < self.redundancy_rate
                        and (path, generation) not in self._audits):
                    audit = True
                    self._audits[(path, generation)] = {"target": self.redundancy - 1, "base": None,
                                                        "primary_digest": None, "primary_peer": None, "checks": [],
                                                        "members": {member}, "batch": batch, "inner": inner,
                                                        "deadline": time.monotonic() + self.audit_timeout,
                                                        "probes": []}
            routing = self._routing_locked(self.topology.path_module_keys(path))
        shard = spec = None
        if check_only or path not in cached:
            if hasattr(self.corpus, "spec"):
                spec = {"path_index": self.topology.path_index(path), "spec": self.corpus.spec}
            else:
                shard = self.corpus.shard(self.topology.path_index(path))
        comp, dens = self.compress, self.up_density
        mbps = caps.get("max_mbps")
        if self.tailor_bandwidth and not check_only and isinstance(mbps, (int, float)) and not isinstance(mbps, bool):
            comp, dens = tailor_encoding(mbps, base_compress=self.compress, base_density=self.up_density)
        task = {"type": "task", "gen_id": generation, "lease": lease, "path": path, "routing": routing,
                "compress": comp, "density": dens, "down": self.down, "shard": compress_shard(shard, comp),
                "shard_spec": spec, "batch_size": batch, "total_rounds": self.total_rounds, "seed": self.seed}
        if self.task_seconds or check_only:
            task["inner_steps"] = inner
        if check_only:
            task["check_only"], task["base"] = True, base
            if self._probe is not None and not self._probe.empty:
                task["probe"], task["probe_batch"] = self._probe.sequences, self._probe.batch_size
        elif audit:
            task["audit"] = True
        return task

    def _commit(self, msg: dict, peer_id: str | None = None) -> dict:
        path = tuple(msg.get("path") or ())
        if msg.get("check_only"):
            key, member = (path, msg.get("gen_id")), peer_id or msg.get("worker_id")
            with self._lock:
                a = self._audits.get(key)
                if a is not None and a.get("check_leases", {}).get(member) == msg.get("lease") and \
                        member not in a.setdefault("checked", set()):
                    a["checked"].add(member)
                    a["checks"].append((peer_id, msg.get("digest")))
                    pb, pa = as_finite_float(msg.get("probe_before")), as_finite_float(msg.get("probe_after"))
                    if pb is not None and pa is not None:
                        a["probes"].append((peer_id, pb, pa))
                    if len(a["checks"]) >= a["target"]:
                        self._resolve_audit(key)
            return {"type": "commit_ack", "check": True}
        verdict = None
        try:
            with self._lock:
                if path not in self._inflight or msg.get("lease") != self._lease.get(path):
                    return {"type": "commit_ack", "accepted": False}
                staleness = self._T - self._issued.get(path, self._T)
                self._inflight.pop(path, None)
                self._lease.pop(path, None)
                wid = self._owner.get(path)
                t0, work = self._lease_at.pop(path, None), self._lease_work.pop(path, None)
                if staleness > self.staleness_bound:
                    self.metrics.record_stale_reject()
                    return {"type": "commit_ack", "accepted": False}
                if not loss_ok(msg.get("loss"), empty=bool(msg.get("empty"))):
                    self.metrics.record_invalid_reject()
                    verdict = False
                    return {"type": "commit_ack", "accepted": False}
                gen = self._completed.get(path, 0)
                self._T += 1
                self._completed[path] = gen + 1
                if t0 is not None and not msg.get("empty"):
                    self._record_rate(wid, work, time.monotonic() - t0)
                damp = 1.0 / (1.0 + staleness) if self.staleness_weight == "inverse" else 1.0
                w = self.corpus.shard_weight(self.topology.path_index(path)) * damp
                self.metrics.record_update(staleness)
                grant = make_grant(path, self.topology.path_module_keys(path), w, msg.get("lease"), self.grant_key,
                                   identity=self.identity)
                a = self._audits.get((path, gen))
                if a is not None and a["base"] is None:
                    a.update(base=msg.get("base"), primary_digest=msg.get("digest"), primary_peer=peer_id,
                             deadline=time.monotonic() + self.audit_timeout)
                    if a["base"] is None:
                        self._audits.pop((path, gen), None)
                verdict = True
                return {"type": "commit_ack", "accepted": True, "push_weight": w, "grant": grant}
        finally:
            if verdict is True:
                self.reputation.credit(peer_id)
            elif verdict is False:
                self.reputation.debit(peer_id)

    def _resolve_audit(self, key) -> None:
        a = self._audits.pop(key, None)
        if a is None:
            return
        present = ([(a["primary_peer"], a["primary_digest"])] if a["primary_digest"] is not None else []) + \
            [(p, d) for p, d in a["checks"] if d is not None]
        digests = [d for _, d in present]
        if len(digests) >= 2:
            top, n = collections.Counter(digests).most_common(1)[0]
            if n >= 2:
                for peer, d in present:
                    if peer is None:
                        continue
                    if d == top:
                        self.reputation.credit(peer)
                    else:
                        self.reputation.debit(peer)
                        self.metrics.record_invalid_reject()
        if self.probe_quorum and a.get("primary_digest") is not None:
            bad = sum(1 for _, b, af in a.get("probes", []) if is_harmful(b, af, **self.probe_margin))
            if bad >= self.probe_quorum:
                self.metrics.record_poison_flag()
                if self.probe_debit and a.get("primary_peer") is not None:
                    self.reputation.debit(a["primary_peer"])

    def _nack(self, msg: dict) -> dict:
        path = tuple(msg.get("path") or ())
        with self._lock:
            if path in self._inflight and msg.get("lease") == self._lease.get(path):
                for d in (self._inflight, self._lease, self._lease_at, self._lease_work):
                    d.pop(path, None)
                return {"type": "nack_ack", "freed": True}
        return {"type": "nack_ack", "freed": False}

    def _heartbeat(self, msg: dict) -> None:
        path = tuple(msg.get("path") or ())
        with self._lock:
            if path in self._inflight and msg.get("lease") == self._lease.get(path):
                self._inflight[path] = time.monotonic() + self.heartbeat_timeout

    def _reclaim_locked(self) -> None:
        now = time.monotonic()
        for path, dl in list(self._inflight.items()):
            if now >= dl:
                del self._inflight[path]
                self._lease.pop(path, None)
                self._owner[path] = None
                self.metrics.reclaims += 1
        for key in [k for k, a in self._audits.items() if a["deadline"] is not None and now >= a["deadline"]]:
            self._resolve_audit(key)

    def fit(self, num_generations: int, *, total_generations=None, log_every=0, reclaim_interval=0.05,
            checkpoint_dir=None, checkpoint_every=0, resume=False, recovery_poll: float = 0.5):
        """Serve until every path has had about ``num_generations`` more updates. With
        ``resume`` the scheduler state of ``checkpoint_dir`` is restored and, when that
        checkpoint has a signed recovery manifest, no task is served until some live
        owner holds at least the manifest's version of every key (owners catch up by
        replication meanwhile): tasks served earlier would train on state older than the
        recovery point."""
        if resume and checkpoint_dir and os.path.exists(os.path.join(checkpoint_dir, "scheduler.pt")):
            self._load_state(checkpoint_dir)
            while self._recovery is not None and not (self._stop or self._dead) and not self._recovery_ready():
                time.sleep(recovery_poll)
        self.total_rounds = total_generations or self.total_rounds or num_generations
        paths = list(self.topology.paths())
        with self._lock:
            self._completed = {p: self._completed.get(p, 0) for p in paths}
            self._inflight, self._issued = {}, {}
            self._target = self._T + num_generations * len(paths)
            self._serving = True
        t0, last = time.monotonic(), self._T
        while True:
            with self._lock:
                self._reclaim_locked()
                done = self._T >= self._target
            if done or self._stop or self._dead:
                break
            if checkpoint_dir and checkpoint_every and self._T - last >= checkpoint_every:
                self._checkpoint_cluster(checkpoint_dir)
                last = self._T
                if log_every:
                    print(f"[sharded] T={self._T}/{self._target}", flush=True)
            time.sleep(reclaim_interval)
        with self._lock:
            self._serving = False
        self.metrics._wall += time.monotonic() - t0
        if checkpoint_dir and checkpoint_every:
            self._checkpoint_cluster(checkpoint_dir)
        return dict(self._completed)

    def _checkpoint_cluster(self, dirpath: str) -> None:
        """Cluster checkpoint: every owner persists its modules, the scheduler writes
        ``scheduler.pt`` and, with an identity and an owner epoch, a signed recovery
        manifest (``manifest.json``: per key the highest version an owner persisted),
        the floor a restarted cluster must reach before it serves tasks again. File
        names and contents are the reference's, so either framework resumes the other's
        checkpoint."""
        os.makedirs(dirpath, exist_ok=True)
        with self._lock:
            record = self._epoch_record
        owners = ([_addr(o["addr"]) for o in record["owners"]] if record is not None else sorted(set(self._ps_addrs)))
        held: dict = {}
        for a in owners:
            try:
                s = connect(a, self.auth_key, timeout=5.0, tls=self.ps_tls)
                try:
                    reply = rpc(s, {"type": "checkpoint", "dir": dirpath})
                finally:
                    s.close()
            except (OSError, ConnectionError, PermissionError):
                continue  # an owner out of reach now is checkpointed next time
            for k, v in (reply.get("versions") or {}).items():
                held[k] = max(held.get(k, (0, 0)), _version_pair(v))
        if record is not None and self.identity is not None and held:
            manifest = sign_record(self.identity, {"kind": "manifest", "epoch": record["epoch"],
                                                   "keys": {k: list(v) for k, v in held.items()},
                                                   "issued_at": time.time()})
            tmp = os.path.join(dirpath, "manifest.json.tmp")
            with open(tmp, "w", encoding="utf-8") as f:
                json.dump(manifest, f)
            os.replace(tmp, os.path.join(dirpath, "manifest.json"))
            with self._lock:
                self._recovery = manifest
        with self._lock:
            state = {"T": self._T, "completed": dict(self._completed),
                     "epoch": -1 if record is None else int(record["epoch"]), "reputation": self.reputation.snapshot()}
        tmp = os.path.join(dirpath, "scheduler.pt.tmp")
        torch.save(state, tmp)
        os.replace(tmp, os.path.join(dirpath, "scheduler.pt"))

    def _load_state(self, dirpath: str) -> None:
        state = torch.load(os.path.join(dirpath, "scheduler.pt"), weights_only=True)
        with self._lock:
            self._T = state["T"]
            self._completed = dict(state["completed"])
            self._epoch_floor = max(self._epoch_floor, int(state.get("epoch", -1)) + 1)
        self.reputation.restore(state.get("reputation") or {})
        mpath = os.path.join(dirpath, "manifest.json")
        if self.identity is not None and os.path.exists(mpath):
            with open(mpath, encoding="utf-8") as f:
                manifest = json.load(f)
            # only this scheduler's own signature counts: a planted manifest could lower
            # (or inflate) the recovery floor
            if (verify_record(manifest) and manifest.get("kind") == "manifest"
                    and str(manifest.get("pub", "")).lower() == self.identity.public_key_hex):
                with self._lock:
                    self._recovery = manifest

    def _recovery_ready(self) -> bool:
        """True when, among the current epoch's owners that answer, some owner holds at
        least the recovery manifest's version of every key."""
        with self._lock:
            record, manifest = self._epoch_record, self._recovery
        if manifest is None:
            return True
        if record is None:
            return False  # the owner set is not known yet (the tracker watch publishes it)
        held: dict = {}
        for a in sorted({_addr(o["addr"]) for o in record["owners"]}):
            try:
                s = connect(a, self.auth_key, timeout=5.0, tls=self.ps_tls)
                try:
                    reply = rpc(s, {"type": "status"})
                finally:
                    s.close()
            except (OSError, ConnectionError, PermissionError):
                continue
            for k, v in ((reply or {}).get("versions") or {}).items():
                held[k] = max(held.get(k, (-1, -1)), _version_pair(v))
        return all(held.get(k, (-1, -1)) >= _version_pair(v) for k, v in manifest["keys"].items())

    def shutdown(self) -> None:
        with self._lock:
            self._serving = False
        super().shutdown()


# ================================================================================ workers
class _WorkerLink:
    """A worker's connections: one to the scheduler (re-dialled after a drop when
    ``reconnect``), cached ones to owners; all optionally TLS and bandwidth-throttled."""

    def __init__(self, sch_addr, *, auth_key, max_msg_bytes=DEFAULT_MAX_MSG_BYTES, connect_timeout=10.0, tls=None,
                 tls_hostname=None, bucket=None, reconnect=False, reconnect_timeout=30.0):
        self.auth_key, self.max_msg_bytes = auth_key, max_msg_bytes
        self.timeout, self.tls, self.tls_hostname, self.bucket = connect_timeout, tls, tls_hostname, bucket
        self.reconnect, self.reconnect_timeout = reconnect, reconnect_timeout
        self._sch_lock = threading.Lock()
        self._ps: dict = {}
        self.sch_addr = _addr(sch_addr) if sch_addr is not None else None
        self.sch = self._dial(self.sch_addr, connect_timeout) if self.sch_addr is not None else None

    def _dial(self, addr, timeout):
        from .throttle import throttled

        s = connect(addr, self.auth_key, self.max_msg_bytes, timeout, tls=self.tls,
                    server_hostname=self.tls_hostname)
        return throttled(s, self.bucket)

    def _redial(self) -> None:
        try:
            self.sch.close()
        except OSError:
            pass
        self.sch = self._dial(self.sch_addr, self.reconnect_timeout)

    def sch_send(self, msg) -> None:
        from .wire import send_msg

        with self._sch_lock:
            send_msg(self.sch, msg)

    def sch_rpc(self, msg):
        with self._sch_lock:
            try:
                return rpc(self.sch, msg, self.max_msg_bytes)
            except (OSError, ConnectionError):
                if not self.reconnect:
                    raise
                self._redial()
                return rpc(self.sch, msg, self.max_msg_bytes)

    def ps_rpc(self, addr, msg):
        a = _addr(addr)
        if a not in self._ps:
            self._ps[a] = self._dial(a, self.timeout)
        try:
            return rpc(self._ps[a], msg, self.max_msg_bytes)
        except (OSError, ConnectionError):
            self._drop(a)
            raise

    def _drop(self, a) -> None:
        s = self._ps.pop(a, None)
        if s is not None:
            try:
                s.close()
            except OSError:
                pass

    def close(self) -> None:
        for a in list(self._ps):
            self._drop(a)
        if self.sch is not None:
            try:
                self.sch.close()
            except OSError:
                pass


def _fetch_keys(link, routing, keys, versions, cold_keys, keyframes, pin=None):
    """Fetch the listed keys from their owners, primary first: a key an owner reports
    missing (not active there yet, or an aged-out pinned version) or an owner that does
    not answer falls back to the key's next replica. Returns {key: state_dict}; raises
    ConnectionError when no replica serves some key."""
    out: dict = {}
    pending = list(keys)
    rank = 0
    while pending:
        by_owner: dict = {}
        unserved = []
        for k in pending:
            owners = routing[k]
            if rank < len(owners):
                by_owner.setdefault(_addr(owners[rank]), []).append(k)
            else:
                unserved.append(k)
        if unserved:
            raise ConnectionError(f"no replica served {sorted(unserved)}")
        retry = []
        for addr, ks in by_owner.items():
            msg = {"type": "fetch", "keys": ks, "have": {k: list(versions[k]) for k in ks if k in versions},
                   "cold": any(k in cold_keys for k in ks)}
            if pin:
                msg["pin"] = {k: pin[k] for k in ks if k in pin}
            try:
                reply = link.ps_rpc(addr, msg)
            except (OSError, ConnectionError):
                retry += ks
                continue
            retry += [k for k in (reply.get("missing") or []) if k in ks]
            for k, payload in (reply.get("weights") or {}).items():
                if isinstance(payload, dict) and "delta" in payload:
                    held = keyframes.get(k)
                    if held is None or held[0] != tuple(payload["base"]):
                        versions.pop(k, None)  # ask for full weights next time
                        raise ValueError(f"delta for {k} against a keyframe this worker does not hold")
                    payload = apply_state_delta(held[1], payload["delta"])
                out[k] = payload
                v = _version_pair(reply["versions"][k])
                versions[k] = v
                # one keyframe per key: the state at the version this worker reports as held
                keyframes[k] = (v, {n: t.float() if t.is_floating_point() else t for n, t in payload.items()})
        pending, rank = retry, rank + 1
    return out


def _push_group(routing, grant, shared_payload, private_payload, link) -> set:
    """Push each key's update to its primary; returns keys refused as not-primary."""
    by_owner: dict = {}
    for k, p in shared_payload.items():
        by_owner.setdefault(_addr(routing[k][0]), ({}, {}))[0][k] = {"grad": p}
    for k, sd in (private_payload or {}).items():
        by_owner.setdefault(_addr(routing[k][0]), ({}, {}))[1][k] = sd
    refused = set()
    for addr, (upd, priv) in by_owner.items():
        try:
            ack = link.ps_rpc(addr, {"type": "push", "grant": grant, "updates": upd, "private": priv})
        except (OSError, ConnectionError):
            refused |= set(upd) | set(priv)
            continue
        if ack.get("reason") == "not_primary":
            refused |= set(ack.get("skipped") or [])
    return refused


def _build_engine(config, diloco, device, seed):
    from ..train.loop import DiPaCoEngine, ExecOptions

    return DiPaCoEngine(config, diloco, LocalBackend(config.build_topology()), device=device, seed=seed,
                        materialize="serial", exec_options=ExecOptions(fused=False))


def run_sharded_worker(config, diloco, scheduler_addr, *, device="cpu", seed=0, auth_key=None,
                       max_msg_bytes=DEFAULT_MAX_MSG_BYTES, connect_timeout=10.0, heartbeat_interval=3.0,
                       poll_interval=0.02, max_tasks=None, fault_hook=None, tls=None, tls_hostname=None,
                       stop_event=None, max_batch_size=None, max_shards=None, reconnect=True,
                       reconnect_timeout=30.0, data_dir=None, data_source=None, data_tokenizer=None,
                       verify_routing=False, bucket=None, identity=None, contribution_hook=None):
    """Lease -> fetch from owners -> train -> commit (grant) -> push to owners.

    ``auth_key`` (or ``identity``) is the credential; ``bucket`` a shared
    ``throttle.TokenBucket`` capping this worker's bandwidth; ``data_dir`` caches
    shards materialised from shipped specs (``verify_routing`` re-fits the shipped
    router from the public source first and refuses to train on a mismatch).
    ``contribution_hook(path, contribution) -> contribution`` rewrites each finished
    task before it is committed (adversary and fault injection in harnesses)."""
    from .distributed import ShardCache, heartbeats, materialize_shard_spec

    engine = _build_engine(config, diloco, device, seed)
    worker = AsyncScheduler(engine, num_workers=1)
    wid = uuid.uuid4().hex
    topo = engine.topology
    cred = auth_key if auth_key is not None else identity
    try:
        link = _WorkerLink(scheduler_addr, auth_key=cred, max_msg_bytes=max_msg_bytes,
                           connect_timeout=connect_timeout, tls=tls, tls_hostname=tls_hostname, bucket=bucket,
                           reconnect=reconnect, reconnect_timeout=reconnect_timeout)
    except ConnectionError:
        return
    data_ctx = {"dir": data_dir, "source": data_source, "tokenizer": data_tokenizer, "verify": verify_routing}
    warm, cache = set(), ShardCache(max_shards)
    versions, keyframes, residuals = {}, {}, {}
    caps = {"device": str(device), **({"max_batch": int(max_batch_size)} if max_batch_size else {})}
    done = 0
    try:
        while stop_event is None or not stop_event.is_set():
            try:
                msg = link.sch_rpc({"type": "request", "worker_id": wid, "warm_paths": list(warm),
                                    "cached_shards": list(cache), "capabilities": caps})
            except (OSError, ConnectionError):
                return          # the scheduler is gone (and did not come back within reconnect_timeout)
            if msg["type"] == "stop":
                return
            if msg["type"] == "idle":
                time.sleep(msg.get("retry_in") or poll_interval)
                continue
            path, lease, routing = tuple(msg["path"]), msg["lease"], msg["routing"]
            worker.seed, engine.total_rounds = msg["seed"], msg["total_rounds"]
            keys = topo.path_module_keys(path)
            try:
                with heartbeats(link.sch_send, heartbeat_interval,
                                {"type": "heartbeat", "lease": lease, "path": path, "worker_id": wid}):
                    if fault_hook is not None:
                        fault_hook(path, 1)
                    pin = msg.get("base") if msg.get("check_only") else None
                    cold = {k for k in keys if is_private_key(k) and path not in warm}
                    fetched = _fetch_keys(link, routing, keys, versions, cold, keyframes, pin=pin)
                    for k, sd in fetched.items():
                        engine.bank[k].load_state_dict({n: v.to(engine.device) for n, v in sd.items()})
                    base = {k: list(versions[k]) for k in keys if k in versions and not is_private_key(k)}
                    if msg.get("shard") is not None:
                        cache[path] = restore_shard(msg["shard"])
                    elif msg.get("shard_spec") is not None and path not in cache:
                        cache[path] = materialize_shard_spec(msg["shard_spec"], data_ctx)
                    if path not in warm:
                        engine._opt_state.pop(path, None)
                    probe = (TrustedProbe(msg["probe"], batch_size=msg.get("probe_batch", 8))
                             if msg.get("probe") is not None else None)
                    contrib = worker._train_path(path, cache[path], msg["batch_size"], msg["gen_id"],
                                                 inner_steps=msg.get("inner_steps"), probe=probe)
                    if contribution_hook is not None:  # fault / adversary injection in harnesses
                        contrib = contribution_hook(path, contrib)
            except Exception as exc:
                try:
                    link.sch_rpc({"type": "nack", "lease": lease, "path": path, "error": repr(exc)})
                except (OSError, ConnectionError):
                    return      # the scheduler is gone as well
                continue
            digest = pseudograd_digest(contrib.shared_delta) if (msg.get("audit") or msg.get("check_only")) else None
            commit = {"type": "commit", "lease": lease, "path": path, "gen_id": msg["gen_id"], "loss": contrib.loss,
                      "empty": contrib.empty, "worker_id": wid, "digest": digest, "base": base,
                      "check_only": bool(msg.get("check_only")), "probe_before": contrib.probe_before,
                      "probe_after": contrib.probe_after}
            try:
                ack = link.sch_rpc(commit)
            except (OSError, ConnectionError):
                return          # the scheduler went away while this task trained
            if msg.get("check_only") or not ack.get("accepted"):
                continue
            engine._opt_state[path] = contrib.opt_state
            for k, sd in contrib.private_state.items():
                engine.bank[k].load_state_dict({n: v.to(engine.device) for n, v in sd.items()})
            warm.add(path)
            mode, dens = msg.get("compress") or "none", float(msg.get("density") or 1.0)
            carry = residuals.get(path) or {}
            shared_p, pending = {}, {}
            for k, d in contrib.shared_delta.items():
                shared_p[k], pending[k] = compress_delta(d, mode, carry=carry.get(k), density=dens)
            private_p = {k: compress_state(sd, mode) for k, sd in contrib.private_state.items()}
            refused = _push_group(routing, ack["grant"], shared_p, private_p, link)
            if refused:
                try:
                    fresh = link.sch_rpc({"type": "routing", "keys": sorted(refused)}).get("routing", {})
                except (OSError, ConnectionError):
                    return
                routing = {**routing, **fresh}
                refused = _push_group(routing, ack["grant"], {k: v for k, v in shared_p.items() if k in refused},
                                      {k: v for k, v in private_p.items() if k in refused}, link)
            if not refused and (mode != "none" or dens < 1.0):
                residuals.setdefault(path, {}).update({k: v for k, v in pending.items() if v is not None})
            done += 1
            if max_tasks is not None and done >= max_tasks:
                return
    finally:
        link.close()


# ====================================================================== decentralized
def _verified_peers(records) -> list:
    return [r for r in records if verify_record(r) and r.get("kind") == "peer"]


def _owner_directories(link, epoch) -> list:
    """The newest verified record of every peer the owners of ``epoch`` know."""
    best: dict = {}
    for o in epoch.get("owners") or []:
        try:
            recs = link.ps_rpc(o["addr"], {"type": "directory"}).get("records") or []
        except (OSError, ConnectionError, PermissionError):
            continue
        for r in _verified_peers(recs):
            ts = record_issued_at(r)
            if ts is not None and (r["peer_id"] not in best or ts > record_issued_at(best[r["peer_id"]])):
                best[r["peer_id"]] = r
    return list(best.values())


def _worker_directory_ids(records) -> list[str]:
    return sorted(r["peer_id"] for r in _verified_peers(records) if "worker" in (r.get("roles") or []))


def _decentralized_routing(topology, path, epoch) -> dict:
    return {k: [o["addr"] for o in owners_for(k, epoch)] for k in topology.path_module_keys(path)}


def run_decentralized_worker(config, diloco, tracker, corpus, *, identity, auth_key=None, device="cpu", seed=0,
                             batch_size=8, workers_fn=None, k=3, salt="", lease_ttl=30.0, read_quorum=1,
                             max_tasks=None, stop_event=None, poll_interval=0.05, total_rounds=None, tls=None,
                             bucket=None, heartbeat_interval=10.0, seeds=(), seed_quorum=1):
    """Scheduler-less worker: self-assign ``(path, generation)`` slots by HRW over the
    live worker set, read bases with quorum reads, commit to the path's coordinating
    owner (which mints an Ed25519 grant), push to every owner of each key.

    ``tracker`` is the tracker's ``(host, port)`` -- the worker then registers itself
    (role ``worker``) every ``heartbeat_interval`` s and derives the owner epoch and
    the worker set from the (multi-seed) directory each pass -- or a callable that
    returns the current epoch record (tests, embedded use). With ``total_rounds``
    the worker stops taking a path once its generation reaches it."""
    from .tracker import dedup_seeds, fetch_directory_multi, register_peer

    engine = _build_engine(config, diloco, device, seed)
    engine.total_rounds = total_rounds
    worker = AsyncScheduler(engine, num_workers=1)
    topo = engine.topology
    link = _WorkerLink(None, auth_key=auth_key if auth_key is not None else identity, connect_timeout=5.0,
                       tls=tls, bucket=bucket)
    beat_stop = threading.Event()
    state = {"epoch": None}
    if callable(tracker):
        epoch_fn = tracker
    else:
        seed_list = dedup_seeds(tuple(tracker), seeds)

        def beat():
            while True:
                for a in seed_list:
                    try:
                        register_peer(a, identity, roles=["worker"], auth_key=auth_key, tls=tls, timeout=5.0)
                    except (OSError, ConnectionError, PermissionError):
                        continue
                if beat_stop.wait(heartbeat_interval):
                    return

        threading.Thread(target=beat, daemon=True).start()

        def epoch_fn():
            recs, answered = fetch_directory_multi(seed_list, auth_key=auth_key, tls=tls, seed_quorum=seed_quorum,
                                                   timeout=2.0)
            if not answered and state["epoch"] is not None:
                # every seed is gone: read the directories the last epoch's owners gossip
                recs = _owner_directories(link, state["epoch"])
            owners = [r for r in recs if "owner" in (r.get("roles") or [])]
            state["workers"] = _worker_directory_ids(recs)
            if owners:
                state["epoch"] = derive_epoch(owners, k=k, salt=salt, prev=state["epoch"])
            return state["epoch"]

        if workers_fn is None:
            workers_fn = lambda: state.get("workers")  # noqa: E731
    done, t_open, finished = 0, {}, set()
    try:
        while (stop_event is None or not stop_event.is_set()) and (max_tasks is None or done < max_tasks):
            try:
                epoch = epoch_fn()
            except (OSError, ConnectionError, PermissionError):
                epoch = None
            if not epoch or not epoch.get("owners"):
                time.sleep(poll_interval)
                continue
            workers = sorted(set((workers_fn() if workers_fn else None) or []) | {identity.peer_id})
            picked = None
            for path in topo.paths():
                keys = topo.path_module_keys(path)
                coord = owners_for(coordinator_key(keys), epoch)[0]
                try:
                    reply = link.ps_rpc(coord["addr"], {"type": "generation", "path": path})
                except (OSError, ConnectionError, PermissionError):
                    continue
                if not reply.get("ok", "generation" in reply):
                    continue  # not the coordinator under its epoch (yet): ask again next pass
                gen = reply["generation"]
                if total_rounds is not None and gen >= total_rounds:
                    finished.add(path)
                    continue
                # the coordinator's age of the open slot drives takeover on both sides
                t0 = t_open.setdefault((path, gen), time.monotonic())
                age = as_finite_float(reply.get("age"))
                elapsed = age if age is not None else time.monotonic() - t0
                if is_assignee(identity.peer_id, path, gen, workers, salt=salt, elapsed=elapsed,
                               lease_ttl=lease_ttl):
                    picked = (path, gen, coord)
                    break
            if picked is None:
                if total_rounds is not None and len(finished) == topo.num_paths:
                    return
                time.sleep(poll_interval)
                continue
            path, gen, coord = picked
            try:
                if _decentralized_task(engine, worker, link, topo, corpus, epoch, path, gen, coord, batch_size,
                                       read_quorum, identity.peer_id):
                    done += 1
            except (OSError, ConnectionError, PermissionError, ValueError):
                time.sleep(poll_interval)
    finally:
        beat_stop.set()
        link.close()


def _decentralized_task(engine, worker, link, topo, corpus, epoch, path, gen, coord, batch_size, read_quorum,
                        worker_id=None) -> bool:
    routing = _decentralized_routing(topo, path, epoch)
    keys = topo.path_module_keys(path)
    shared = [k for k in keys if not is_private_key(k)]
    confirmed = read_quorum_versions(list({_addr(a) for k in shared for a in routing[k]}), shared, read_quorum,
                                     lambda a, m: link.ps_rpc(a, m)) if read_quorum > 1 else {}
    base: dict = {}
    fetched = _fetch_keys(link, routing, keys, base, {k for k in keys if is_private_key(k)}, {},
                          pin={k: list(v[0]) for k, v in confirmed.items()} or None)
    for k, sd in fetched.items():
        engine.bank[k].load_state_dict({n: v.to(engine.device) for n, v in sd.items()})
    contrib = worker._train_path(path, corpus.shard(topo.path_index(path)), batch_size, gen)
    ack = link.ps_rpc(coord["addr"], {"type": "commit", "path": path, "gen_id": gen, "loss": contrib.loss,
                                     "empty": contrib.empty, "weight": corpus.shard_weight(topo.path_index(path)),
                                     "worker_id": worker_id, "base_versions": {k: list(v) for k, v in base.items()}})
    if not ack.get("accepted"):
        return False
    # one push per owner (a grant token is single-use per owner), carrying every key it replicates
    by_owner: dict = {}
    for k in keys:
        for a in routing[k]:
            upd, priv = by_owner.setdefault(_addr(a), ({}, {}))
            if k in contrib.shared_delta:
                upd[k] = {"grad": contrib.shared_delta[k]}
            if k in contrib.private_state:
                priv[k] = contrib.private_state[k]
    for a, (upd, priv) in by_owner.items():
        try:
            link.ps_rpc(a, {"type": "push", "grant": ack["grant"], "updates": upd, "private": priv})
        except (OSError, ConnectionError):
            continue
    return True


__all__ = ["ParameterServer", "Scheduler", "assign_shards", "make_grant", "verify_grant", "grant_signed_by",
           "run_sharded_worker", "run_decentralized_worker"]
