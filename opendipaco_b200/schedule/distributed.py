"""Single-node asynchronous coordinator and stateful TCP worker
(reference ``src/opendipaco/schedule/distributed.py``).

Coordinator (``CoordinatorServer``) holds the whole bank and serves tasks:

* ``request`` -> ``task``: the least-completed path not in flight (ties broken toward
  paths the worker already holds warm), with a fresh lease token; only shared weights
  whose version differs from what the worker holds, private weights only for cold
  paths, the shard (or a shard *spec* in spec mode) unless cached.
* ``submit`` -> ``ack``: rejected unless the lease token matches the live lease;
  rejected when staler than ``staleness_bound`` updates or when the guard finds
  non-finite values; otherwise each shared key takes its own SGD-Nesterov step with
  weight ``alpha * 1/(1 + staleness)`` (optionally x sqrt(sharing)), bumping its
  version.
* ``heartbeat`` refreshes a lease; leases whose deadline passed are reclaimed.

Worker (``run_worker``): keeps its private modules, inner-optimizer state and shards
warm across tasks (optimizer state never crosses the wire), heartbeats during
training, compresses its upload per the coordinator's mode with error feedback whose
residuals are adopted only when the server applied the update, reconnects with
exponential backoff. Message schema and field names follow the reference so either
framework's peers can talk to the other's.
"""

from __future__ import annotations

import math
import os
import socket
import ssl
import threading
import time
import uuid
from collections import OrderedDict

import torch

from ..checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
from ..data.spec import materialize_shard, spec_fingerprint, verify_routing
from ..optim.diloco import apply_outer_grads, make_outer_optimizer
from ..parallel.backend.local import LocalBackend
from ..topology import is_private_key
from ..train.loop import _opt_state_cpu, _state_cpu
from .compress import check_mode, compress_delta, compress_shard, compress_state, maybe_dequantize, restore_shard
from .guard import clip_norm_, contribution_ok
from .reactor import ReactorServer
from .scheduler import AsyncScheduler
from .wire import DEFAULT_MAX_MSG_BYTES, client_handshake, recv_msg, send_msg


class CoordinatorServer(ReactorServer):
    def __init__(self, scheduler: AsyncScheduler, corpus, batch_size: int, *, host: str = "0.0.0.0",
                 port: int = 0, heartbeat_timeout: float | None = None, auth_key=None, accept_keys=None,
                 admitted_peers=None, max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES, staleness_bound: int | None = None,
                 staleness_weight: str = "inverse", rescale_by_sqrt_sharing: bool = False,
                 max_update_norm: float | None = None, compress: str = "none", idle_backoff: float | None = None,
                 io_threads: int = 4, max_connections: int = 1024, tls=None):
        super().__init__(host=host, port=port, auth_key=auth_key, accept_keys=accept_keys,
                         admitted_peers=admitted_peers, max_msg_bytes=max_msg_bytes, io_threads=io_threads,
                         max_connections=max_connections, tls=tls)
        self.sched, self.engine, self.corpus, self.batch_size = scheduler, scheduler.engine, corpus, batch_size
        npaths = len(self.engine.topology.paths())
        self.staleness_bound = staleness_bound if staleness_bound is not None else 2 * npaths
        self.staleness_weight = staleness_weight
        self.rescale_by_sqrt_sharing = rescale_by_sqrt_sharing
        self.max_update_norm = max_update_norm
        self.compress = check_mode(compress)
        self.idle_backoff = idle_backoff
        self.heartbeat_timeout = heartbeat_timeout if heartbeat_timeout is not None else scheduler.lease_timeout
        self._lock = threading.Lock()
        self._serving = False
        self._versions = {k: 0 for k in self.engine.topology.module_keys() if not is_private_key(k)}
        self._worker_caps: dict = {}
        self._owner: dict = {}
        self._T = 0
        self._target = 0
        self._completed: dict = {}
        self._inflight: dict = {}
        self._issued: dict = {}
        self._lease: dict = {}
        self._outer_opts: dict = {}

    # -- dispatch -------------------------------------------------------------
    def _handle(self, msg: dict, nbytes: int, peer_id: str | None = None):
        kind = msg.get("type")
        if kind == "request":
            return self._next_task(msg)
        if kind == "submit":
            return {"type": "ack", "applied": self._receive(msg)}
        if kind == "manifest":
            return {"type": "manifest", "manifest": getattr(self, "_manifest", None)}
        if kind == "nack":
            self._nack(msg)
        elif kind == "heartbeat":
            self._heartbeat(msg)
        return None

    def serve_manifest(self, manifest) -> None:
        """Publish the run manifest that ``opendipaco join`` clients fetch."""
        self._manifest = manifest

    def shutdown(self) -> None:
        with self._lock:
            self._serving = False
        super().shutdown()

    def simulate_crash(self) -> None:
        with self._lock:
            self._serving = False
        super().simulate_crash()

    def _idle(self) -> dict:
        return {"type": "idle", **({"retry_in": self.idle_backoff} if self.idle_backoff is not None else {})}

    def _task_batch_size(self, caps: dict) -> int:
        cap = (caps or {}).get("max_batch")
        return max(1, min(self.batch_size, int(cap))) if cap else self.batch_size

    def _next_task(self, req: dict) -> dict:
        wid = req.get("worker_id")
        warm = {tuple(p) for p in req.get("warm_paths", [])}
        cached = {tuple(p) for p in req.get("cached_shards", [])}
        have = req.get("have_shared", {})
        caps = req.get("capabilities") or {}
        e = self.engine
        with self._lock:
            if caps:
                self._worker_caps[wid] = caps
            if not self._serving or self._T >= self._target:
                return {"type": "stop"} if self._stop else self._idle()
            self._reclaim_inflight_locked()
            eligible = [p for p in self._completed if p not in self._inflight]
            if not eligible:
                return self._idle()
            path = min(eligible, key=lambda p: (self._completed[p], p not in warm, p))
            lease = uuid.uuid4().hex
            self._owner[path] = wid
            self._inflight[path] = time.monotonic() + self.heartbeat_timeout
            self._issued[path] = self._T
            self._lease[path] = lease
            generation = self._completed[path]
            versions = dict(self._versions)
            keys = e.topology.path_module_keys(path)
            shared_keys = [k for k in keys if not is_private_key(k)]
            shared_w = {k: compress_state(_state_cpu(e.bank[k].state_dict()), self.compress)
                        for k in shared_keys if have.get(k) != versions[k]}
            private_w = None if path in warm else {
                k: compress_state(_state_cpu(e.bank[k].state_dict()), self.compress)
                for k in keys if is_private_key(k)}
        shard = spec = None
        if path not in cached:
            if hasattr(self.corpus, "spec"):
                spec = {"path_index": e.topology.path_index(path), "spec": self.corpus.spec}
            else:
                shard = self.corpus.shard(e.topology.path_index(path))
        return {"type": "task", "gen_id": generation, "lease": lease, "generation": generation, "path": path,
                "compress": self.compress, "shared_weights": shared_w,
                "shared_versions": {k: versions[k] for k in shared_keys}, "private_weights": private_w,
                "shard": compress_shard(shard, self.compress), "shard_spec": spec,
                "batch_size": self._task_batch_size(caps), "total_rounds": e.total_rounds, "seed": self.sched.seed}

    def _receive(self, msg: dict) -> bool:
        path = tuple(msg["path"])
        e = self.engine
        try:
            shared = {k: maybe_dequantize(v) for k, v in (msg.get("shared_grad") or {}).items() if k in self._versions}
        except (TypeError, KeyError, ValueError):
            shared = None
        private = {k: v for k, v in (msg.get("private_weights") or {}).items() if is_private_key(k) and k in e.bank}
        valid = shared is not None and contribution_ok(msg.get("loss"), msg.get("empty"), shared, private)
        with self._lock:
            if path not in self._inflight or msg.get("lease") != self._lease.get(path):
                return False
            staleness = self._T - self._issued.get(path, self._T)
            self._inflight.pop(path, None)
            self._lease.pop(path, None)
            if staleness > self.staleness_bound:
                self.metrics.record_stale_reject()
                return False
            if not valid:
                self.metrics.record_invalid_reject()
                return False
            keys = set(e.topology.path_module_keys(path))
            shared = {k: v for k, v in shared.items() if k in keys}
            private = {k: v for k, v in private.items() if k in keys}
            if self.max_update_norm is not None:
                for delta in shared.values():
                    if clip_norm_(delta, self.max_update_norm) > self.max_update_norm:
                        self.metrics.record_norm_clip()
            self._T += 1
            self._completed[path] = self._completed.get(path, 0) + 1
            damp = 1.0 / (1.0 + staleness) if self.staleness_weight == "inverse" else 1.0
            for key, sd in private.items():
                e.bank[key].load_state_dict({n: v.to(e.device) for n, v in sd.items()})
            pidx = e.topology.path_index(path)
            for key, delta in shared.items():
                w = e._outer_weight(key, pidx, self.corpus) * damp
                if self.rescale_by_sqrt_sharing:
                    w *= math.sqrt(e.topology.sharing_count(key))
                apply_outer_grads(e.bank[key], [w * d.to(e.device) for d in delta])
                self._outer_opts[key].step()
                self._outer_opts[key].zero_grad(set_to_none=True)
                self._versions[key] += 1
            self.metrics.record_update(staleness)
            return True

    def _nack(self, msg: dict) -> None:
        path = tuple(msg["path"])
        with self._lock:
            if path in self._inflight and msg.get("lease") == self._lease.get(path):
                self.sched.errors[path] = msg.get("error", "worker nack")
                self._inflight.pop(path, None)
                self._lease.pop(path, None)

    def _heartbeat(self, msg: dict) -> None:
        path = tuple(msg["path"])
        with self._lock:
            if path in self._inflight and msg.get("lease") == self._lease.get(path):
                self._inflight[path] = time.monotonic() + self.heartbeat_timeout

    def _reclaim_inflight_locked(self) -> None:
        now = time.monotonic()
        for path, deadline in list(self._inflight.items()):
            if now >= deadline:
                del self._inflight[path]
                self._lease.pop(path, None)
                self._owner[path] = None
                self.metrics.reclaims += 1

    def fit(self, num_generations: int, *, total_generations: int | None = None, log_every: int = 0,
            reclaim_interval: float = 0.05, checkpoint_dir: str | None = None, checkpoint_every: int = 0,
            resume: bool = False):
        """Serve until every path has had ~``num_generations`` more accepted updates."""
        e = self.engine
        restore = None
        if resume and checkpoint_dir and latest_checkpoint(checkpoint_dir):
            restore = load_checkpoint(e, latest_checkpoint(checkpoint_dir)).get("extra")
        if total_generations is not None:
            e.total_rounds = total_generations
        elif e.total_rounds is None:
            e.total_rounds = num_generations
        paths = list(e.topology.paths())
        self.sched._last_batch_size = self.batch_size
        self._outer_opts = {k: make_outer_optimizer({k: e.bank[k]}, e.diloco) for k in self._versions}
        if restore is not None:
            with self._lock:
                self._T = restore["T"]
                self._completed = dict(restore["completed"])
                self._versions.update(restore["versions"])
            for k, sd in restore["outer_opts"].items():
                if k in self._outer_opts:
                    self._outer_opts[k].load_state_dict(sd)
        with self._lock:
            self._completed = {p: self._completed.get(p, 0) for p in paths}
            self._inflight, self._issued = {}, {}
            self._target = self._T + num_generations * len(paths)
            self._serving = True
        t0 = time.monotonic()
        last = self._T
        while True:
            with self._lock:
                self._reclaim_inflight_locked()
                done = self._T >= self._target
            if done or self._stop or self._dead:
                break
            if checkpoint_dir and checkpoint_every and self._T - last >= checkpoint_every:
                last = self._save_cluster_checkpoint(checkpoint_dir)
                if log_every:
                    print(f"[async] T={last}/{self._target} {self.metrics.report().splitlines()[0]}", flush=True)
            time.sleep(reclaim_interval)
        with self._lock:
            self._serving = False
        self.metrics._wall += time.monotonic() - t0
        if checkpoint_dir and checkpoint_every:
            self._save_cluster_checkpoint(checkpoint_dir)
        return dict(self._completed)

    def _save_cluster_checkpoint(self, checkpoint_dir: str) -> int:
        with self._lock:
            extra = {"T": self._T, "completed": dict(self._completed), "versions": dict(self._versions),
                     "outer_opts": {k: _opt_state_cpu(o.state_dict()) for k, o in self._outer_opts.items()}}
            save_checkpoint(self.engine, os.path.join(checkpoint_dir, f"upd{self._T:08d}"), extra=extra)
            return self._T


# ============================================================================== worker
class RoutingVerificationError(RuntimeError):
    """A shipped router does not reproduce from its declared public source."""


class _ShardCache:
    """Bounded LRU ``path -> shard tensor``."""

    def __init__(self, maxsize: int | None = 4):
        maxsize = 4 if maxsize is None else int(maxsize)
        if maxsize < 1:
            raise ValueError(f"shard cache maxsize must be >= 1, got {maxsize}")
        self._max, self._d = maxsize, OrderedDict()

    def __contains__(self, path) -> bool:
        return path in self._d

    def __getitem__(self, path):
        self._d.move_to_end(path)
        return self._d[path]

    def __setitem__(self, path, shard) -> None:
        self._d[path] = shard
        self._d.move_to_end(path)
        while len(self._d) > self._max:
            self._d.popitem(last=False)

    def __iter__(self):
        return iter(tuple(self._d))

    def __len__(self) -> int:
        return len(self._d)


def _build_worker_engine(config, diloco, device, seed):
    from ..train.loop import DiPaCoEngine, ExecOptions

    return DiPaCoEngine(config, diloco, LocalBackend(config.build_topology()), device=device, seed=seed,
                        materialize="serial", exec_options=ExecOptions(fused=False))


def _compress_contribution(contrib, mode, residuals, path, density: float = 1.0):
    if mode == "none" and density >= 1.0:
        return contrib.shared_delta, contrib.private_state, None
    carry = residuals.get(path) or {}
    payload, pending = {}, {}
    for key, delta in contrib.shared_delta.items():
        payload[key], pending[key] = compress_delta(delta, mode, carry=carry.get(key), density=density)
    private = {k: compress_state(sd, mode) for k, sd in contrib.private_state.items()}
    return payload, private, pending


def _commit_residuals(residuals, path, pending) -> None:
    if pending:
        residuals.setdefault(path, {}).update(pending)


def _load_into(engine, key, sd) -> None:
    engine.bank[key].load_state_dict({n: v.to(engine.device) for n, v in sd.items()})


def _load_private(engine, private_state) -> None:
    for key, sd in (private_state or {}).items():
        _load_into(engine, key, sd)


def _materialize_from_spec(shard_spec, ctx) -> torch.Tensor:
    ctx = ctx or {}
    spec = shard_spec["spec"]
    if ctx.get("verify"):
        fp = spec_fingerprint(spec)
        seen = ctx.setdefault("verified", set())
        if fp not in seen:
            try:
                ok = verify_routing(spec, source=ctx.get("source"), tokenizer=ctx.get("tokenizer"))
            except ValueError as exc:
                print(f"WARNING: cannot verify spec {fp}: {exc}. Proceeding unverified.", flush=True)
                ok = True
            if not ok:
                raise RoutingVerificationError(f"shipped router for spec {fp} does not reproduce from its public "
                                               "source -- refusing to train")
            seen.add(fp)
    return materialize_shard(spec, shard_spec["path_index"], source=ctx.get("source"),
                             tokenizer=ctx.get("tokenizer"), cache_dir=ctx.get("dir"))


def _apply_task(engine, msg, shard_cache, versions, warm, residuals, data_ctx=None) -> torch.Tensor:
    path = tuple(msg["path"])
    for key, sd in (msg.get("shared_weights") or {}).items():
        _load_into(engine, key, sd)
    versions.update(msg.get("shared_versions", {}))
    if msg.get("private_weights"):
        _load_private(engine, msg["private_weights"])
    if path not in warm:
        engine._opt_state.pop(path, None)
        residuals.pop(path, None)
    if msg.get("shard") is not None:
        shard_cache[path] = restore_shard(msg["shard"])
    elif msg.get("shard_spec") is not None and path not in shard_cache:
        shard_cache[path] = _materialize_from_spec(msg["shard_spec"], data_ctx)
    return shard_cache[path]


def _connect(host: str, port: int, timeout: float, *, tls=None, server_hostname: str | None = None):
    deadline, last = time.monotonic() + timeout, None
    while time.monotonic() < deadline:
        s = None
        try:
            s = socket.create_connection((host, port), timeout=timeout)
            s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            return tls.wrap_socket(s, server_hostname=server_hostname or host) if tls is not None else s
        except ssl.SSLError:
            if s is not None:
                s.close()
            raise
        except OSError as exc:
            last = exc
            time.sleep(0.05)
    raise ConnectionError(f"could not connect to coordinator at {host}:{port}: {last}")


def _heartbeat_loop(send, stop, interval, wid, lease, path) -> None:
    while not stop.wait(interval):
        try:
            send({"type": "heartbeat", "lease": lease, "path": path, "worker_id": wid})
        except OSError:
            return


def _serve_connection(conn, engine, worker, wid, warm, cache, versions, attempts, residuals, data_ctx, caps,
                      state, poll_interval, heartbeat_interval, max_msg_bytes, max_tasks, fault_hook) -> bool:
    lock = threading.Lock()

    def send(m):
        with lock:
            send_msg(conn, m)

    while True:
        try:
            send({"type": "request", "worker_id": wid, "have_shared": versions, "warm_paths": list(warm),
                  "cached_shards": list(cache), "capabilities": caps})
            msg = recv_msg(conn, max_msg_bytes)
        except (OSError, ValueError):
            return False
        if msg is None:
            return False
        if msg["type"] == "stop":
            return True
        if msg["type"] == "idle":
            time.sleep(msg.get("retry_in") or poll_interval)
            continue
        path, lease = tuple(msg["path"]), msg.get("lease")
        worker.seed = msg["seed"]
        engine.total_rounds = msg["total_rounds"]
        stop_beat = threading.Event()
        beat = threading.Thread(target=_heartbeat_loop, args=(send, stop_beat, heartbeat_interval, wid, lease, path),
                                daemon=True)
        beat.start()
        try:
            if fault_hook is not None:
                attempts[path] = attempts.get(path, 0) + 1
                fault_hook(path, attempts[path])
            shard = _apply_task(engine, msg, cache, versions, warm, residuals, data_ctx)
            contrib = worker._train_path(path, shard, msg["batch_size"], msg["generation"])
            engine._opt_state[path] = contrib.opt_state
            _load_private(engine, contrib.private_state)
            warm.add(path)
        except RoutingVerificationError:
            stop_beat.set()
            beat.join(timeout=1)
            raise
        except Exception as exc:
            stop_beat.set()
            beat.join(timeout=1)
            try:
                send({"type": "nack", "gen_id": msg["gen_id"], "lease": lease, "path": path, "error": repr(exc)})
            except OSError:
                return False
            continue
        stop_beat.set()
        beat.join(timeout=1)
        shared_p, private_p, pending = _compress_contribution(contrib, msg.get("compress") or "none", residuals, path)
        try:
            send({"type": "submit", "gen_id": msg["gen_id"], "lease": lease, "path": path, "loss": contrib.loss,
                  "empty": contrib.empty, "shared_grad": shared_p, "private_weights": private_p})
            ack = recv_msg(conn, max_msg_bytes)
        except OSError:
            return False
        if ack and ack.get("applied"):
            _commit_residuals(residuals, path, pending)
        state["done"] += 1
        if max_tasks is not None and state["done"] >= max_tasks:
            return True


def run_worker(config, diloco, host: str, port: int, *, device: str = "cpu", seed: int = 0,
               poll_interval: float = 0.02, connect_timeout: float = 10.0, reconnect: bool = True,
               reconnect_timeout: float = 30.0, heartbeat_interval: float = 3.0, auth_key=None,
               max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES, max_tasks: int | None = None, fault_hook=None, tls=None,
               tls_hostname: str | None = None, data_dir: str | None = None, data_source=None,
               data_tokenizer=None, max_batch_size: int | None = None, max_shards: int = 4,
               verify_routing: bool = False):
    """Train leased path-tasks from a coordinator until told to stop."""
    engine = _build_worker_engine(config, diloco, device, seed)
    worker = AsyncScheduler(engine, num_workers=1)
    wid = uuid.uuid4().hex
    warm, cache = set(), _ShardCache(max_shards)
    versions, attempts, residuals = {}, {}, {}
    ctx = {"dir": data_dir, "source": data_source, "tokenizer": data_tokenizer, "verify": verify_routing}
    caps = {"device": str(device)}
    if max_batch_size is not None:
        caps["max_batch"] = int(max_batch_size)
    state, first, backoff = {"done": 0}, True, 0.05
    while True:
        try:
            conn = _connect(host, port, connect_timeout if first else reconnect_timeout, tls=tls,
                            server_hostname=tls_hostname)
        except ConnectionError:
            return
        first = False
        if not client_handshake(conn, auth_key):
            conn.close()
            raise PermissionError("coordinator rejected auth (wrong or missing key)")
        try:
            done = _serve_connection(conn, engine, worker, wid, warm, cache, versions, attempts, residuals, ctx,
                                     caps, state, poll_interval, heartbeat_interval, max_msg_bytes, max_tasks,
                                     fault_hook)
        finally:
            try:
                conn.close()
            except OSError:
                pass
        if done or not reconnect:
            return
        time.sleep(backoff)
        backoff = min(backoff * 2, 1.0)
