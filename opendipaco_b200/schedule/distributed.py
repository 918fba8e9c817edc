"""Single-node asynchronous coordinator and stateful TCP workers.

The coordinator (:class:`CoordinatorServer`) holds the whole module bank and hands out
path tasks; workers (:func:`run_worker`) train them and send back pseudo-gradients. There
are no generations: every accepted update moves the global modules at once.

Coordinator, per message type:

* ``request``: the path with the fewest accepted updates that is not in flight (ties:
  paths the worker already holds warm, then path order) under a fresh lease token.
  The task carries only the shared modules whose version differs from the worker's
  copy, the private modules only for a cold path, and the token shard (or, in spec
  mode, the shard's recipe) unless the worker caches it.
* ``submit``: accepted only under the live lease, at most ``staleness_bound`` updates
  stale, and with finite values (the guard); each shared key then takes its own
  SGD-Nesterov step with weight ``alpha / (1 + staleness)`` (times sqrt(sharing) on
  request) and its version advances. Answered with ``ack`` (``applied``).
* ``heartbeat`` extends a lease; ``nack`` releases it; expired leases are reclaimed.

Worker: keeps its private modules, inner-optimizer states and shards warm across tasks
(optimizer state never crosses the wire), heartbeats while training, compresses its
upload in the coordinator's mode with error feedback (a residual is kept only when the
server applied the update) and reconnects with exponential backoff.

The message types, their fields and the checkpoint ``extra`` record follow the
reference's ``src/opendipaco/schedule/distributed.py``, so peers and checkpoints of
either framework interoperate; the structure of this module is its own.
"""

from __future__ import annotations

import math
import os
import threading
import time
import uuid
from collections import OrderedDict
from contextlib import contextmanager
from dataclasses import dataclass

import torch

from ..checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
from ..data.spec import materialize_shard, spec_fingerprint, verify_routing
from ..optim.diloco import apply_outer_grads, make_outer_optimizer
from ..parallel.backend.local import LocalBackend
from ..topology import Path, is_private_key
from ..train.loop import _opt_state_cpu, _state_cpu
from .compress import check_mode, compress_delta, compress_shard, compress_state, decode_checked, restore_shard
from .guard import clip_norm_, contribution_ok
from .reactor import ReactorServer
from .rpc import connect
from .scheduler import AsyncScheduler
from .wire import DEFAULT_MAX_MSG_BYTES, recv_msg, send_msg


# ============================================================================ coordinator
@dataclass
class _PathRecord:
    completed: int = 0            # accepted updates of this path
    lease: str | None = None      # live lease token (None: not in flight)
    deadline: float = 0.0         # lease expiry (monotonic seconds)
    issued_at: int = 0            # global update count T when the task was issued
    owner: str | None = None      # worker id of the lease


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
        topo = self.engine.topology
        self.staleness_bound = staleness_bound if staleness_bound is not None else 2 * len(topo.paths())
        self.staleness_weight = staleness_weight
        self.rescale_by_sqrt_sharing = rescale_by_sqrt_sharing
        self.max_update_norm = max_update_norm
        self.compress = check_mode(compress)
        self.idle_backoff = idle_backoff
        self.heartbeat_timeout = heartbeat_timeout if heartbeat_timeout is not None else scheduler.lease_timeout
        self._lock = threading.Lock()
        self._serving = False
        self._versions = {k: 0 for k in topo.module_keys() if not is_private_key(k)}
        self._records: dict[Path, _PathRecord] = {p: _PathRecord() for p in topo.paths()}
        self._worker_caps: dict = {}
        self._T = 0        # accepted updates so far
        self._target = 0   # stop serving once T reaches it
        self._outer_opts: dict = {}
        self._manifest = None
        self._routes = {"request": self._on_request, "submit": self._on_submit, "manifest": self._on_manifest,
                        "nack": self._on_nack, "heartbeat": self._on_heartbeat}

    # -- messages
    def _handle(self, msg: dict, nbytes: int, peer_id: str | None = None):
        route = self._routes.get(msg.get("type"))
        return route(msg) if route is not None else None

    def _on_manifest(self, msg: dict) -> dict:
        return {"type": "manifest", "manifest": self._manifest}

    def serve_manifest(self, manifest) -> None:
        """Publish the run manifest that ``opendipaco join`` clients fetch."""
        self._manifest = manifest

    def _idle(self) -> dict:
        return {"type": "idle", **({"retry_in": self.idle_backoff} if self.idle_backoff is not None else {})}

    def _task_batch_size(self, caps: dict) -> int:
        cap = (caps or {}).get("max_batch")
        return max(1, min(self.batch_size, int(cap))) if cap else self.batch_size

    def _expire_locked(self) -> None:
        now = time.monotonic()
        for rec in self._records.values():
            if rec.lease is not None and now >= rec.deadline:
                rec.lease, rec.owner = None, None
                self.metrics.reclaims += 1

    def _lease_of(self, msg: dict) -> _PathRecord | None:
        """The record of the message's path when the message holds its live lease."""
        rec = self._records.get(tuple(msg.get("path", ())))
        return rec if rec is not None and rec.lease is not None and msg.get("lease") == rec.lease else None

    def _on_request(self, req: dict) -> dict:
        wid = req.get("worker_id")
        warm = {tuple(p) for p in req.get("warm_paths", [])}
        cached = {tuple(p) for p in req.get("cached_shards", [])}
        held = req.get("have_shared", {})
        caps = req.get("capabilities") or {}
        e = self.engine
        with self._lock:
            if caps:
                self._worker_caps[wid] = caps
            if not self._serving or self._T >= self._target:
                return {"type": "stop"} if self._stop else self._idle()
            self._expire_locked()
            free = [p for p, r in self._records.items() if r.lease is None]
            if not free:
                return self._idle()
            path = min(free, key=lambda p: (self._records[p].completed, p not in warm, p))
            rec = self._records[path]
            rec.lease, rec.owner, rec.issued_at = uuid.uuid4().hex, wid, self._T
            rec.deadline = time.monotonic() + self.heartbeat_timeout
            keys = e.topology.path_module_keys(path)
            shared_keys = [k for k in keys if not is_private_key(k)]
            snapshot = lambda k: compress_state(_state_cpu(e.bank[k].state_dict()), self.compress)  # noqa: E731
            shared_w = {k: snapshot(k) for k in shared_keys if held.get(k) != self._versions[k]}
            private_w = None if path in warm else {k: snapshot(k) for k in keys if is_private_key(k)}
            versions = {k: self._versions[k] for k in shared_keys}
            lease, generation = rec.lease, rec.completed
        shard = spec = None
        if path not in cached:
            if hasattr(self.corpus, "spec"):
                spec = {"path_index": e.topology.path_index(path), "spec": self.corpus.spec}
            else:
                shard = self.corpus.shard(e.topology.path_index(path))
        return {"type": "task", "gen_id": generation, "lease": lease, "generation": generation, "path": path,
                "compress": self.compress, "shared_weights": shared_w, "shared_versions": versions,
                "private_weights": private_w, "shard": compress_shard(shard, self.compress), "shard_spec": spec,
                "batch_size": self._task_batch_size(caps), "total_rounds": e.total_rounds, "seed": self.sched.seed}

    def _decode_upload(self, msg: dict):
        """(shared pseudo-gradients or None when malformed, private states, valid)."""
        e = self.engine
        raw, priv = msg.get("shared_grad") or {}, msg.get("private_weights") or {}
        if not (isinstance(raw, dict) and isinstance(priv, dict)):
            return {}, {}, False
        try:  # declared shapes are screened before any payload is decoded
            shared = {k: decode_checked(v, [tuple(p.shape) for p in e.bank[k].parameters()])
                      for k, v in raw.items() if k in self._versions}
        except (TypeError, KeyError, ValueError):
            shared = None
        private = {k: v for k, v in priv.items() if is_private_key(k) and k in e.bank}
        for k, sd in private.items():
            ref = e.bank[k].state_dict()
            if not isinstance(sd, dict) or set(sd) != set(ref) or any(
                    not torch.is_tensor(sd[n]) or sd[n].shape != ref[n].shape for n in ref):
                return {}, {}, False
        valid = shared is not None and contribution_ok(msg.get("loss"), msg.get("empty"), shared, private)
        return shared or {}, private, valid

    def _on_submit(self, msg: dict) -> dict:
        return {"type": "ack", "applied": self._accept(msg)}

    def _accept(self, msg: dict) -> bool:
        shared, private, valid = self._decode_upload(msg)
        path = tuple(msg["path"])
        e = self.engine
        with self._lock:
            rec = self._lease_of(msg)
            if rec is None:
                return False
            staleness = self._T - rec.issued_at
            rec.lease, rec.owner = None, None
            if staleness > self.staleness_bound:
                self.metrics.record_stale_reject()
                return False
            if not valid:
                self.metrics.record_invalid_reject()
                return False
            mine = set(e.topology.path_module_keys(path))
            if self.max_update_norm is not None:
                for key, delta in shared.items():
                    if key in mine and clip_norm_(delta, self.max_update_norm) > self.max_update_norm:
                        self.metrics.record_norm_clip()
            self._T += 1
            rec.completed += 1
            for key, sd in private.items():
                if key in mine:
                    e.bank[key].load_state_dict({n: v.to(e.device) for n, v in sd.items()})
            damp = 1.0 / (1.0 + staleness) if self.staleness_weight == "inverse" else 1.0
            pidx = e.topology.path_index(path)
            for key, delta in shared.items():
                if key not in mine:
                    continue
                w = e._outer_weight(key, pidx, self.corpus) * damp
                if self.rescale_by_sqrt_sharing:
                    w *= math.sqrt(e.topology.sharing_count(key))
                apply_outer_grads(e.bank[key], [w * d.to(e.device) for d in delta])
                opt = self._outer_opts[key]
                opt.step()
                opt.zero_grad(set_to_none=True)
                self._versions[key] += 1
            self.metrics.record_update(staleness)
            return True

    def _on_nack(self, msg: dict) -> None:
        with self._lock:
            rec = self._lease_of(msg)
            if rec is not None:
                self.sched.errors[tuple(msg["path"])] = msg.get("error", "worker nack")
                rec.lease, rec.owner = None, None

    def _on_heartbeat(self, msg: dict) -> None:
        with self._lock:
            rec = self._lease_of(msg)
            if rec is not None:
                rec.deadline = time.monotonic() + self.heartbeat_timeout

    # -- lifecycle
    def shutdown(self) -> None:
        with self._lock:
            self._serving = False
        super().shutdown()

    def simulate_crash(self) -> None:
        with self._lock:
            self._serving = False
        super().simulate_crash()

    def _restore(self, extra: dict) -> None:
        """Coordinator state of a cluster checkpoint (the engine's own state is loaded
        before the outer optimizers are built on its parameters)."""
        with self._lock:
            self._T = extra["T"]
            for p, n in extra["completed"].items():
                self._records.setdefault(tuple(p), _PathRecord()).completed = n
            self._versions.update(extra["versions"])
        for k, sd in extra["outer_opts"].items():
            if k in self._outer_opts:
                self._outer_opts[k].load_state_dict(sd)

    def fit(self, num_generations: int, *, total_generations: int | None = None, log_every: int = 0,
            reclaim_interval: float = 0.05, checkpoint_dir: str | None = None, checkpoint_every: int = 0,
            resume: bool = False):
        """Serve until every path has had about ``num_generations`` more accepted updates;
        returns path -> accepted updates."""
        e = self.engine
        if total_generations is not None:
            e.total_rounds = total_generations
        elif e.total_rounds is None:
            e.total_rounds = num_generations
        self.sched._last_batch_size = self.batch_size
        extra = None
        if resume and checkpoint_dir and latest_checkpoint(checkpoint_dir):
            extra = load_checkpoint(e, latest_checkpoint(checkpoint_dir)).get("extra")
        self._outer_opts = {k: make_outer_optimizer({k: e.bank[k]}, e.diloco) for k in self._versions}
        if extra is not None:
            self._restore(extra)
        with self._lock:
            for rec in self._records.values():
                rec.lease, rec.owner = None, None
            self._target = self._T + num_generations * len(self._records)
            self._serving = True
        started, saved_at = time.monotonic(), self._T
        while not (self._stop or self._dead):
            with self._lock:
                self._expire_locked()
                if self._T >= self._target:
                    break
            if checkpoint_dir and checkpoint_every and self._T - saved_at >= checkpoint_every:
                saved_at = self._save_cluster_checkpoint(checkpoint_dir)
                if log_every:
                    print(f"[async] T={saved_at}/{self._target} {self.metrics.report().splitlines()[0]}", flush=True)
            time.sleep(reclaim_interval)
        with self._lock:
            self._serving = False
        self.metrics._wall += time.monotonic() - started
        if checkpoint_dir and checkpoint_every:
            self._save_cluster_checkpoint(checkpoint_dir)
        return {p: r.completed for p, r in self._records.items()}

    def _save_cluster_checkpoint(self, checkpoint_dir: str) -> int:
        with self._lock:
            extra = {"T": self._T, "completed": {p: r.completed for p, r in self._records.items()},
                     "versions": dict(self._versions),
                     "outer_opts": {k: _opt_state_cpu(o.state_dict()) for k, o in self._outer_opts.items()}}
            save_checkpoint(self.engine, os.path.join(checkpoint_dir, f"upd{self._T:08d}"), extra=extra)
            return self._T


# ============================================================================ worker
class RoutingVerificationError(RuntimeError):
    """A shipped router does not reproduce from its declared public source."""


class ShardCache(OrderedDict):
    """``path -> token shard`` keeping the ``maxsize`` most recently used entries."""

    def __init__(self, maxsize: int | None = 4):
        super().__init__()
        self.maxsize = 4 if maxsize is None else int(maxsize)
        if self.maxsize < 1:
            raise ValueError(f"shard cache maxsize must be >= 1, got {self.maxsize}")

    def __getitem__(self, path):
        self.move_to_end(path)
        return super().__getitem__(path)

    def __setitem__(self, path, shard) -> None:
        super().__setitem__(path, shard)
        self.move_to_end(path)
        while len(self) > self.maxsize:
            self.popitem(last=False)


_ShardCache = ShardCache


def materialize_shard_spec(shard_spec: dict, ctx: dict | None) -> torch.Tensor:
    """Build a path's shard from a shipped recipe ``{"path_index", "spec"}``; with
    ``ctx["verify"]`` the recipe's router must first reproduce from its declared public
    source (checked once per recipe fingerprint)."""
    ctx = ctx if ctx is not None else {}
    spec = shard_spec["spec"]
    if ctx.get("verify"):
        fp = spec_fingerprint(spec)
        checked = ctx.setdefault("verified", set())
        if fp not in checked:
            try:
                ok = verify_routing(spec, source=ctx.get("source"), tokenizer=ctx.get("tokenizer"))
            except ValueError as exc:
                print(f"WARNING: cannot verify spec {fp}: {exc}. Proceeding unverified.", flush=True)
                ok = True
            if not ok:
                raise RoutingVerificationError(f"shipped router for spec {fp} does not reproduce from its public "
                                               "source -- refusing to train")
            checked.add(fp)
    return materialize_shard(spec, shard_spec["path_index"], source=ctx.get("source"),
                             tokenizer=ctx.get("tokenizer"), cache_dir=ctx.get("dir"))


def _build_worker_engine(config, diloco, device, seed):
    from ..train.loop import DiPaCoEngine, ExecOptions

    return DiPaCoEngine(config, diloco, LocalBackend(config.build_topology()), device=device, seed=seed,
                        materialize="serial", exec_options=ExecOptions(fused=False))


def _load_states(engine, states) -> None:
    for key, sd in (states or {}).items():
        engine.bank[key].load_state_dict({n: v.to(engine.device) for n, v in sd.items()})


class _WorkerState:
    """Everything a worker keeps across tasks and reconnects."""

    def __init__(self, engine, *, shards: int, data_ctx: dict, caps: dict, fault_hook=None):
        self.engine = engine
        self.trainer = AsyncScheduler(engine, num_workers=1)
        self.wid = uuid.uuid4().hex
        self.warm: set = set()
        self.shards = ShardCache(shards)
        self.versions: dict = {}
        self.residuals: dict = {}   # path -> key -> residual list (error feedback)
        self.attempts: dict = {}
        self.data_ctx, self.caps, self.fault_hook = data_ctx, caps, fault_hook
        self.done = 0

    def request(self) -> dict:
        return {"type": "request", "worker_id": self.wid, "have_shared": self.versions, "warm_paths": list(self.warm),
                "cached_shards": list(self.shards), "capabilities": self.caps}

    def adopt(self, task: dict) -> torch.Tensor:
        """Load the task's weights into the local bank; return its shard."""
        path = tuple(task["path"])
        _load_states(self.engine, task.get("shared_weights"))
        self.versions.update(task.get("shared_versions", {}))
        _load_states(self.engine, task.get("private_weights"))
        if path not in self.warm:  # a cold path starts its inner optimizer and residuals afresh
            self.engine._opt_state.pop(path, None)
            self.residuals.pop(path, None)
        if task.get("shard") is not None:
            self.shards[path] = restore_shard(task["shard"])
        elif task.get("shard_spec") is not None and path not in self.shards:
            self.shards[path] = materialize_shard_spec(task["shard_spec"], self.data_ctx)
        return self.shards[path]

    def train(self, task: dict):
        path = tuple(task["path"])
        self.trainer.seed = task["seed"]
        self.engine.total_rounds = task["total_rounds"]
        if self.fault_hook is not None:
            self.attempts[path] = self.attempts.get(path, 0) + 1
            self.fault_hook(path, self.attempts[path])
        contrib = self.trainer._train_path(path, self.adopt(task), task["batch_size"], task["generation"])
        self.engine._opt_state[path] = contrib.opt_state
        _load_states(self.engine, contrib.private_state)
        self.warm.add(path)
        return contrib

    def package(self, contrib, mode: str, density: float = 1.0):
        """(shared payload, private payload, residuals to keep if the update is applied)."""
        if mode == "none" and density >= 1.0:
            return contrib.shared_delta, contrib.private_state, None
        carry = self.residuals.get(contrib.path) or {}
        shared, keep = {}, {}
        for key, delta in contrib.shared_delta.items():
            shared[key], keep[key] = compress_delta(delta, mode, carry=carry.get(key), density=density)
        private = {k: compress_state(sd, mode) for k, sd in contrib.private_state.items()}
        return shared, private, keep

    def applied(self, path, keep) -> None:
        if keep:
            self.residuals.setdefault(path, {}).update(keep)


@contextmanager
def heartbeats(send, interval: float, beat: dict):
    """Send ``beat`` every ``interval`` seconds while the block runs."""
    halt = threading.Event()

    def loop():
        while not halt.wait(interval):
            try:
                send(beat)
            except OSError:
                return

    t = threading.Thread(target=loop, name="odp-heartbeat", daemon=True)
    t.start()
    try:
        yield
    finally:
        halt.set()
        t.join(timeout=1.0)


def _session(conn, st: _WorkerState, *, poll_interval: float, heartbeat_interval: float, max_msg_bytes: int,
             max_tasks: int | None) -> bool:
    """Serve tasks over one connection; True when the work is over, False when the
    connection was lost (the caller reconnects)."""
    wlock = threading.Lock()

    def send(m):
        with wlock:
            send_msg(conn, m)

    while True:
        try:
            send(st.request())
            task = recv_msg(conn, max_msg_bytes)
        except (OSError, ValueError):
            return False
        if task is None:
            return False
        if task["type"] == "stop":
            return True
        if task["type"] == "idle":
            time.sleep(task.get("retry_in") or poll_interval)
            continue
        path, lease = tuple(task["path"]), task.get("lease")
        try:
            with heartbeats(send, heartbeat_interval,
                             {"type": "heartbeat", "lease": lease, "path": path, "worker_id": st.wid}):
                contrib = st.train(task)
        except RoutingVerificationError:
            raise
        except Exception as exc:
            try:
                send({"type": "nack", "gen_id": task["gen_id"], "lease": lease, "path": path, "error": repr(exc)})
            except OSError:
                return False
            continue
        shared, private, keep = st.package(contrib, task.get("compress") or "none")
        try:
            send({"type": "submit", "gen_id": task["gen_id"], "lease": lease, "path": path, "loss": contrib.loss,
                  "empty": contrib.empty, "shared_grad": shared, "private_weights": private})
            ack = recv_msg(conn, max_msg_bytes)
        except OSError:
            return False
        if ack and ack.get("applied"):
            st.applied(path, keep)
        st.done += 1
        if max_tasks is not None and st.done >= max_tasks:
            return True


def run_worker(config, diloco, host: str, port: int, *, device: str = "cpu", seed: int = 0,
               poll_interval: float = 0.02, connect_timeout: float = 10.0, reconnect: bool = True,
               reconnect_timeout: float = 30.0, heartbeat_interval: float = 3.0, auth_key=None,
               max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES, max_tasks: int | None = None, fault_hook=None, tls=None,
               tls_hostname: str | None = None, data_dir: str | None = None, data_source=None,
               data_tokenizer=None, max_batch_size: int | None = None, max_shards: int = 4,
               verify_routing: bool = False):
    """Train leased path tasks from a coordinator until it says stop (or, with
    ``reconnect=False``, until the connection drops)."""
    caps = {"device": str(device), **({"max_batch": int(max_batch_size)} if max_batch_size is not None else {})}
    st = _WorkerState(_build_worker_engine(config, diloco, device, seed), shards=max_shards, caps=caps,
                      data_ctx={"dir": data_dir, "source": data_source, "tokenizer": data_tokenizer,
                                "verify": verify_routing}, fault_hook=fault_hook)
    timeout, backoff = connect_timeout, 0.05
    while True:
        try:
            conn = connect((host, port), auth_key, max_msg_bytes, timeout, tls=tls, server_hostname=tls_hostname)
        except PermissionError:
            raise PermissionError("coordinator rejected auth (wrong or missing key)") from None
        except ConnectionError:
            return
        timeout = reconnect_timeout
        try:
            finished = _session(conn, st, poll_interval=poll_interval, heartbeat_interval=heartbeat_interval,
                                max_msg_bytes=max_msg_bytes, max_tasks=max_tasks)
        finally:
            try:
                conn.close()
            except OSError:
                pass
        if finished or not reconnect:
            return
        time.sleep(backoff)
        backoff = min(2 * backoff, 1.0)
