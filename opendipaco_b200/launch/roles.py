"""Cluster roles stood up from a ``LaunchConfig`` (reference ``src/opendipaco/launch/roles.py``).

* ``run_coordinator`` -- single-node async coordinator (holds the weights).
* ``run_scheduler`` -- weight-less sharded scheduler; with ``ownership.mode:
  rendezvous`` it signs owner epochs from the tracker's live owner set.
* ``run_parameter_server`` -- a static shard (``assign_shards`` slice) or a dynamic
  owner (heartbeats the tracker; its keys follow the epochs).
* ``run_worker_role`` -- coordinator, sharded or decentralized worker.
* ``run_tracker`` / ``run_relay`` / ``run_ingest``.
* ``run_local`` -- a whole cluster in one process (coordinator, static-sharded,
  rendezvous or decentralized), ephemeral ports, for smoke runs and tests.

Servers block until SIGINT/SIGTERM (or a given ``stop_event``); a graceful owner
shutdown hands its latest state to its successors within a 10 s deadline.
"""

from __future__ import annotations

import os
import signal
import threading
import time

import torch

from ..data import (ShardedCorpus, SpecCorpus, c4_source, fit_routing_from_source, kmeans_routing,
                    make_shard_spec, pack_sequences, round_robin_routing, synthetic_documents, synthetic_source)
from ..data.spec import iter_spec_documents
from ..parallel.backend.local import LocalBackend
from ..routing import BagOfTokensFeaturizer, KMeansRouter
from ..schedule import (AsyncScheduler, CoordinatorServer, ParameterServer, PeerIdentity, RateLimiter,
                        Reputation, Scheduler, Tracker, assign_shards, client_context, derive_epoch,
                        make_peer_record, owners_for, path_primary, run_decentralized_worker, run_sharded_worker,
                        run_worker, server_context)
from ..schedule.throttle import TokenBucket, rate_from_mbps
from ..train.loop import DiPaCoEngine
from .config import LaunchConfig, dipaco_config, diloco_config
from .manifest import build_manifest

SHUTDOWN_DEADLINE = 10.0
DECENTRALIZED_RUN_TIMEOUT = 120.0


# ------------------------------------------------------------------- shared builders
def build_tls_server(cfg: LaunchConfig):
    t = cfg.tls
    return server_context(t.certfile, t.keyfile, cafile=t.cafile,
                          require_client_cert=t.require_client_cert) if t.enabled else None


def build_tls_client(cfg: LaunchConfig):
    t = cfg.tls
    return client_context(cafile=t.cafile, insecure=t.insecure) if t.enabled else None


def _server_kw(cfg: LaunchConfig, extra_admitted=None) -> dict:
    t = cfg.transport
    kw = dict(auth_key=t.auth_key, accept_keys=list(t.accept_keys) or None, tls=build_tls_server(cfg))
    admitted = list(t.admitted_peers) + list(extra_admitted or [])
    if admitted:
        kw["admitted_peers"] = admitted
    if t.max_msg_bytes is not None:
        kw["max_msg_bytes"] = t.max_msg_bytes
    return kw


def _reputation(cfg: LaunchConfig) -> Reputation:
    r = cfg.robustness
    return Reputation(floor=r.reputation_floor, credit=r.reputation_credit, debit=r.reputation_debit,
                      decay_halflife=r.reputation_halflife)


def _rate_limiter(cfg: LaunchConfig) -> RateLimiter:
    return RateLimiter(capacity=cfg.robustness.rate_capacity, refill_per_sec=cfg.robustness.rate_refill_per_sec)


def _build_probe(cfg: LaunchConfig, model):
    """The trusted probe: the first ``robustness.probe_docs`` documents of the public
    source packed to the model's sequence length. A configured screen that cannot get
    its probe raises instead of running without it."""
    n = cfg.robustness.probe_docs
    if not n:
        return None
    docs = []
    try:
        for doc in iter_spec_documents({"source": _spec_source(cfg)}):
            docs.append(doc)
            if len(docs) >= n:
                break
    except Exception as exc:
        raise RuntimeError(f"could not read the public source for the poisoning probe ({exc}); "
                           "fix the source or unset robustness.probe_docs") from exc
    probe = pack_sequences(docs, model.sequence_length)
    if probe.numel() == 0:
        raise ValueError(f"robustness.probe_docs={n} gave an empty probe (documents too few or too short)")
    return probe


def _scheduler_robust_kw(cfg: LaunchConfig, model) -> dict:
    r = cfg.robustness
    return dict(reputation=_reputation(cfg), rate_limiter=_rate_limiter(cfg),
                min_owner_reputation=r.min_owner_reputation, redundancy=r.redundancy,
                redundancy_rate=r.redundancy_rate, audit_timeout=r.audit_timeout, private_policy=r.private_policy,
                probe=_build_probe(cfg, model), probe_quorum=r.probe_quorum, probe_abs_margin=r.probe_abs_margin,
                probe_rel_margin=r.probe_rel_margin, probe_debit=r.probe_debit)


def _ps_robust_kw(cfg: LaunchConfig) -> dict:
    r = cfg.robustness
    # audits pin the primary's base version, so owners must keep a few past versions
    history = 4 if r.version_history <= 1 and r.redundancy_rate > 0 else r.version_history
    return dict(robustness=r.mode, aggregate=r.aggregate, quorum_target=r.quorum_target,
                quorum_timeout=r.quorum_timeout, version_history=history, private_policy=r.private_policy,
                private_quorum=r.private_quorum)


def _decentralized_kw(cfg: LaunchConfig) -> dict:
    if cfg.schedule.mode != "decentralized":
        return {}
    s, own = cfg.schedule, cfg.ownership
    return dict(schedule_mode="decentralized", salt=own.salt, k=own.k, lease_ttl=s.lease_ttl,
                read_quorum=s.read_quorum, directory_ttl=cfg.tracker.ttl, reputation=_reputation(cfg),
                rate_limiter=_rate_limiter(cfg), min_owner_reputation=cfg.robustness.min_owner_reputation)


def _publish_manifest(server, cfg: LaunchConfig, identity) -> None:
    m = build_manifest(cfg, identity=identity)
    if "sig" not in m:
        print("NOTE: serving an unsigned run manifest (no transport.identity_key); joiners cannot pin it "
              "with --server-pub", flush=True)
    server.serve_manifest(m)


def _advertise_host(cfg: LaunchConfig) -> str:
    t = cfg.transport
    return cfg.ownership.advertise_host or t.connect_host or (t.host if t.host not in ("0.0.0.0", "::")
                                                               else "127.0.0.1")


def _identity(cfg: LaunchConfig, identity=None, *, generate=False):
    if identity is not None:
        return identity
    if cfg.transport.identity_key:
        return PeerIdentity.load(cfg.transport.identity_key)
    return PeerIdentity.generate() if generate else None


def _worker_credential(cfg: LaunchConfig):
    """A per-peer Ed25519 identity when configured (revocable), else the shared secret."""
    return PeerIdentity.load(cfg.transport.identity_key) if cfg.transport.identity_key else cfg.transport.auth_key


def _attach_metrics(server, cfg: LaunchConfig) -> None:
    t = cfg.transport
    if t.metrics_port is not None:
        server.start_metrics_server(host=t.metrics_host, port=t.metrics_port)
    if t.metrics_log_interval and t.metrics_log_interval > 0:
        server.start_metrics_logging(interval=t.metrics_log_interval)


def _signal_event() -> threading.Event:
    ev = threading.Event()
    for sig in (signal.SIGINT, signal.SIGTERM):
        try:
            signal.signal(sig, lambda *_: ev.set())
        except (ValueError, OSError):   # not the main thread
            pass
    return ev


def _graceful_shutdown(server, deadline: float = SHUTDOWN_DEADLINE) -> None:
    """``shutdown(graceful=True)``, but leave anyway if the hand-off hangs."""
    timer = threading.Timer(deadline, lambda: os._exit(0))
    timer.daemon = True
    timer.start()
    try:
        server.shutdown(graceful=True)
    finally:
        timer.cancel()


# ------------------------------------------------------------------------ data
def build_documents(cfg: LaunchConfig):
    d = cfg.data
    if d.source == "synthetic":
        return synthetic_documents(vocab_size=cfg.model.vocab_size, num_documents=d.num_documents,
                                   doc_len=d.synthetic_doc_len, topics=d.synthetic_topics, seed=cfg.run.seed)
    if d.source == "c4":
        from ..data import load_c4_documents

        return load_c4_documents(num_documents=d.num_documents, tokenizer_name=d.tokenizer or "t5-base",
                                 max_doc_tokens=d.max_doc_tokens, min_doc_tokens=d.min_doc_tokens,
                                 cache_path=d.cache_path)
    raise ValueError(f"unknown data source {d.source!r} (use 'c4' or 'synthetic')")


def _spec_source(cfg: LaunchConfig) -> dict:
    d = cfg.data
    if d.source == "synthetic":
        return synthetic_source(vocab_size=cfg.model.vocab_size, num_documents=d.num_documents,
                                doc_len=d.synthetic_doc_len, topics=d.synthetic_topics, seed=cfg.run.seed)
    if d.source == "c4":
        return c4_source(num_documents=d.num_documents, tokenizer=d.tokenizer or "t5-base",
                         max_doc_tokens=d.max_doc_tokens, min_doc_tokens=d.min_doc_tokens)
    raise ValueError(f"unknown data source {d.source!r}")


def _fit_router(cfg: LaunchConfig, model, docs):
    feat = BagOfTokensFeaturizer(cfg.model.vocab_size, feature_dim=min(256, cfg.model.vocab_size))
    router = KMeansRouter(model.num_paths, seed=cfg.data.router_seed).fit(
        feat([d[:model.sequence_length] for d in docs]))
    return feat, router


def build_corpus(cfg: LaunchConfig, model, docs):
    """Packed shards (``data.ship: bytes``) or a shard recipe + token counts (``spec``)."""
    if cfg.data.ship == "spec":
        return build_spec_corpus(cfg, model, docs)
    n, seq = model.num_paths, model.sequence_length
    if cfg.data.routing == "round_robin" or len(docs) < n:
        return ShardedCorpus.from_assignments(docs, torch.tensor([i % n for i in range(len(docs))]), n, seq)
    feat, router = _fit_router(cfg, model, docs)
    return ShardedCorpus.from_documents(docs, router, feat, n, seq)


def build_spec_corpus(cfg: LaunchConfig, model, docs) -> SpecCorpus:
    n, seq = model.num_paths, model.sequence_length
    if cfg.data.routing == "round_robin" or len(docs) < n:
        routing = round_robin_routing()
    else:
        feat, router = _fit_router(cfg, model, docs)
        routing = kmeans_routing(router.centroids, vocab_size=cfg.model.vocab_size, feature_dim=feat.feature_dim)
    spec = make_shard_spec(source=_spec_source(cfg), routing=routing, num_paths=n, seq_len=seq)
    return SpecCorpus.from_documents(spec, docs)


def build_spec_corpus_streaming(cfg: LaunchConfig, model) -> SpecCorpus:
    """Two streamed passes over the public source (sampled router fit, token counts):
    the server never holds the corpus."""
    n, seq = model.num_paths, model.sequence_length
    source = _spec_source(cfg)
    if cfg.data.routing == "round_robin":
        routing = round_robin_routing()
    else:
        routing = fit_routing_from_source(source, num_paths=n, vocab_size=cfg.model.vocab_size, seq_len=seq,
                                          sample=cfg.data.router_sample,
                                          feature_dim=min(256, cfg.model.vocab_size),
                                          router_seed=cfg.data.router_seed)
    return SpecCorpus.build(make_shard_spec(source=source, routing=routing, num_paths=n, seq_len=seq))


def build_server_corpus(cfg: LaunchConfig, model):
    if cfg.data.ship == "spec" and cfg.data.router_sample is not None:
        return build_spec_corpus_streaming(cfg, model)
    return build_corpus(cfg, model, build_documents(cfg))


# ------------------------------------------------------------------------ roles
def run_coordinator(cfg: LaunchConfig, *, on_start=None):
    """Train to ``run.generations`` behind a single coordinator; returns ``(server, completed)``."""
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    corpus = build_server_corpus(cfg, model)
    engine = DiPaCoEngine(model, diloco, LocalBackend(model.build_topology()), seed=cfg.run.seed,
                          materialize="serial")
    t = cfg.transport
    server = CoordinatorServer(AsyncScheduler(engine, lease_timeout=t.heartbeat_timeout), corpus,
                               batch_size=cfg.run.batch_size, host=t.host, port=t.port,
                               heartbeat_timeout=t.heartbeat_timeout, staleness_bound=t.staleness_bound,
                               staleness_weight=t.staleness_weight, max_update_norm=t.max_update_norm,
                               compress=t.compress, idle_backoff=t.idle_backoff, **_server_kw(cfg))
    server.start()
    _publish_manifest(server, cfg, _identity(cfg))
    _attach_metrics(server, cfg)
    if on_start:
        on_start(server)
    completed = server.fit(num_generations=cfg.run.generations, total_generations=cfg.run.generations,
                           checkpoint_dir=cfg.run.checkpoint_dir, checkpoint_every=cfg.run.checkpoint_every,
                           resume=cfg.run.resume)
    server.shutdown()
    return server, completed


def run_scheduler(cfg: LaunchConfig, *, ps_addrs=None, on_start=None, identity=None, tracker_addr=None,
                  extra_admitted=None):
    """The weight-less scheduler. Static ownership routes to ``sharded.parameter_servers``
    (or ``ps_addrs``); rendezvous ownership signs epochs from the tracker directory."""
    if cfg.transport.kind == "libp2p":
        from ..schedule.p2p import _require_libp2p

        _require_libp2p()
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    corpus = build_server_corpus(cfg, model)
    own, t = cfg.ownership, cfg.transport
    rendezvous = own.mode == "rendezvous"
    ident = _identity(cfg, identity, generate=rendezvous)
    if rendezvous:
        addrs = []
    else:
        addrs = list(ps_addrs) if ps_addrs is not None else [tuple(a) for a in cfg.sharded.parameter_servers]
        if not addrs:
            raise ValueError("sharded mode needs sharded.parameter_servers (or ps_addrs)")
    sched = Scheduler(model, corpus, addrs, diloco, cfg.run.batch_size, host=t.host, port=t.port,
                      seed=cfg.run.seed, staleness_bound=t.staleness_bound, staleness_weight=t.staleness_weight,
                      heartbeat_timeout=t.heartbeat_timeout, grant_key=t.grant_key, identity=ident,
                      compress=t.compress, down=t.down, up_density=t.up_density, idle_backoff=t.idle_backoff,
                      task_seconds=cfg.run.task_seconds, park_factor=cfg.run.park_factor,
                      min_task_rate=cfg.run.min_task_rate, tailor_bandwidth=t.tailor_bandwidth,
                      ps_tls=build_tls_client(cfg), **_scheduler_robust_kw(cfg, model),
                      **_server_kw(cfg, extra_admitted))
    sched.start()
    _publish_manifest(sched, cfg, ident)
    _attach_metrics(sched, cfg)
    if rendezvous:
        if cfg.run.resume and cfg.run.checkpoint_dir and os.path.exists(
                os.path.join(cfg.run.checkpoint_dir, "scheduler.pt")):
            sched._load_state(cfg.run.checkpoint_dir)
        sched.watch_tracker(tracker_addr or cfg.tracker_connect_addr(), k=own.k, salt=own.salt,
                            owner_grace=own.owner_grace, min_epoch_interval=own.min_epoch_interval,
                            poll_interval=own.epoch_poll_interval, tracker_auth=t.auth_key,
                            tracker_tls=build_tls_client(cfg))
    if on_start:
        on_start(sched)
    completed = sched.fit(cfg.run.generations, total_generations=cfg.run.generations,
                          checkpoint_dir=cfg.run.checkpoint_dir, checkpoint_every=cfg.run.checkpoint_every,
                          resume=cfg.run.resume and not rendezvous)
    sched.shutdown()
    return sched, completed


def _ps_port(cfg: LaunchConfig, shard_id: int, port) -> int:
    if port is not None:
        return port
    servers = cfg.sharded.parameter_servers
    return int(servers[shard_id][1]) if shard_id < len(servers) else 0


def run_parameter_server(cfg: LaunchConfig, shard_id: int = 0, *, port=None, on_start=None, stop_event=None,
                         identity=None, scheduler_addr=None, tracker_addr=None, scheduler_pub=None,
                         extra_admitted=None):
    """A parameter server until stopped: a fixed shard (``ownership.mode: static``) or a
    dynamic owner (``rendezvous``: tracker heartbeat, keys from epochs)."""
    if cfg.transport.kind == "libp2p":
        from ..schedule.p2p import _require_libp2p

        _require_libp2p()
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    own, t = cfg.ownership, cfg.transport
    common = dict(host=t.host, device=cfg.run.device, grant_key=t.grant_key, max_update_norm=t.max_update_norm,
                  compress=t.compress, down=t.down,
                  resume_dir=cfg.run.checkpoint_dir if cfg.run.resume else None, **_ps_robust_kw(cfg))
    if own.mode == "rendezvous":
        ident = _identity(cfg, identity, generate=True)
        central = cfg.schedule.mode != "decentralized"
        ps = ParameterServer(model, [], diloco, port=port if port is not None else 0, identity=ident,
                             scheduler_pub=scheduler_pub or t.scheduler_pub,
                             scheduler_addr=(scheduler_addr or cfg.connect_addr()) if central else None,
                             replicate_interval=own.replicate_interval, bank_seed=own.bank_seed,
                             peer_tls=build_tls_client(cfg), **_decentralized_kw(cfg), **common,
                             **_server_kw(cfg, extra_admitted))
        ps.start()
        circuits = None
        if t.relays and t.kind == "tcp":
            # behind NAT: reachable only through reservations on the configured relays
            from ..schedule.relay import serve_via_relays

            circuits = serve_via_relays(ps, t.relays, ident)
            if not circuits:
                raise RuntimeError(f"no relay of {t.relays} accepted a reservation")
        ps.start_tracker_heartbeat(tracker_addr or cfg.tracker_connect_addr(), _advertise_host(cfg),
                                   interval=own.heartbeat_interval, auth_key=t.auth_key, tls=build_tls_client(cfg),
                                   seeds=cfg.tracker.seeds, circuit_addrs=circuits)
    else:
        keys = sorted(model.build_topology().module_keys())
        owned = [k for k, s in assign_shards(keys, cfg.sharded.num_shards).items() if s == shard_id]
        ps = ParameterServer(model, owned, diloco, port=_ps_port(cfg, shard_id, port), **common,
                             **_server_kw(cfg, extra_admitted))
        ps.start()
    _attach_metrics(ps, cfg)
    if on_start:
        on_start(ps)
    (stop_event or _signal_event()).wait()
    if stop_event is None:
        _graceful_shutdown(ps)
    else:
        ps.shutdown(graceful=True)
    return ps


def run_worker_role(cfg: LaunchConfig, *, addr=None, scheduler_addr=None, max_tasks=None, stop_event=None,
                    bucket=None):
    """A worker for the configured mode; ``bucket`` (a shared ``TokenBucket``) caps its
    bandwidth, built from ``transport.max_mbps`` when not given."""
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    t, r = cfg.transport, cfg.run
    mt = max_tasks if max_tasks is not None else r.max_tasks
    if bucket is None and t.max_mbps:
        rate = rate_from_mbps(t.max_mbps)
        bucket = TokenBucket(rate) if rate else None
    if t.kind == "libp2p":
        from ..schedule.p2p import _require_libp2p

        _require_libp2p()
    if stop_event is None and (cfg.mode == "sharded" or cfg.schedule.mode == "decentralized"):
        # SIGINT / SIGTERM end these loops between tasks (a graceful leave); the
        # coordinator's worker keeps the default handlers, as nothing there would
        # consume the event and the signal would otherwise be swallowed
        stop_event = _signal_event()
    if cfg.schedule.mode == "decentralized":
        own = cfg.ownership
        corpus = build_corpus(cfg, model, build_documents(cfg))
        run_decentralized_worker(model, diloco, tuple(cfg.tracker_connect_addr()), corpus,
                                 identity=_identity(cfg, generate=True), device=r.device, seed=r.seed,
                                 auth_key=t.auth_key, k=own.k, salt=own.salt, read_quorum=cfg.schedule.read_quorum,
                                 lease_ttl=cfg.schedule.lease_ttl, batch_size=r.batch_size,
                                 total_rounds=r.generations, max_tasks=mt, heartbeat_interval=own.heartbeat_interval,
                                 tls=build_tls_client(cfg), stop_event=stop_event, bucket=bucket,
                                 seeds=cfg.tracker.seeds, seed_quorum=cfg.tracker.seed_quorum)
        return
    if cfg.mode == "sharded":
        run_sharded_worker(model, diloco, tuple(scheduler_addr or cfg.connect_addr()), device=r.device, seed=r.seed,
                           auth_key=_worker_credential(cfg), max_tasks=mt, reconnect=True,
                           heartbeat_interval=t.heartbeat_interval, tls=build_tls_client(cfg),
                           tls_hostname=cfg.tls.server_hostname, data_dir=cfg.data.shard_cache_dir,
                           max_batch_size=r.worker_max_batch, max_shards=r.worker_max_shards,
                           verify_routing=bool(r.verify_routing), stop_event=stop_event, bucket=bucket)
        return
    host, port = addr or cfg.connect_addr()
    run_worker(model, diloco, host, port, device=r.device, seed=r.seed, auth_key=_worker_credential(cfg),
               max_tasks=mt, heartbeat_interval=t.heartbeat_interval, tls=build_tls_client(cfg),
               tls_hostname=cfg.tls.server_hostname, data_dir=cfg.data.shard_cache_dir,
               max_batch_size=r.worker_max_batch, max_shards=r.worker_max_shards or 4,
               verify_routing=bool(r.verify_routing))


def run_tracker(cfg: LaunchConfig, *, on_start=None, stop_event=None):
    t = cfg.tracker
    tracker = Tracker(host=t.host, port=t.port, ttl=t.ttl, open_enrollment=t.open_enrollment,
                      enroll_peers=list(t.enroll_peers), **_server_kw(cfg))
    tracker.start()
    _publish_manifest(tracker, cfg, _identity(cfg))
    _attach_metrics(tracker, cfg)
    if on_start:
        on_start(tracker)
    (stop_event or _signal_event()).wait()
    tracker.shutdown()
    return tracker


def run_relay(cfg: LaunchConfig, *, on_start=None, stop_event=None, port=None):
    """A circuit relay for NAT peers on ``transport.host:port`` (``schedule/relay.py``);
    ``transport.admitted_peers`` (public keys), when set, limits who may reserve."""
    from ..schedule.identity import peer_id_of
    from ..schedule.relay import RelayServer

    t = cfg.transport
    admitted = [peer_id_of(p) for p in t.admitted_peers] or None
    relay = RelayServer(_identity(cfg, generate=True), host=t.host, port=t.port if port is None else port,
                        admitted=admitted).start()
    print(f"relay listening: {relay.multiaddr(_advertise_host(cfg))}", flush=True)
    if on_start:
        on_start(relay)
    (stop_event or _signal_event()).wait()
    relay.shutdown()
    return relay


def run_ingest(cfg: LaunchConfig, shard_id: int):
    """Resumably ingest this host's C4 shard into ``data.shard_cache_dir``."""
    from ..data import ingest_c4_shard, load_tokenizer

    d = cfg.data
    if not d.shard_cache_dir:
        raise ValueError("ingest needs data.shard_cache_dir")
    if d.source != "c4":
        raise ValueError("ingest is for the 'c4' data source")
    return ingest_c4_shard(d.shard_cache_dir, shard_id=shard_id, num_shards=cfg.sharded.num_shards,
                           target_docs=d.num_documents, tokenizer=load_tokenizer(d.tokenizer or "t5-base"),
                           max_doc_tokens=d.max_doc_tokens, min_doc_tokens=d.min_doc_tokens)


# ------------------------------------------------------------------ local clusters
def run_local(cfg: LaunchConfig):
    """The whole cluster in this process; returns ``(driving server, completed)``."""
    if cfg.schedule.mode == "decentralized":
        return _local_decentralized(cfg)
    if cfg.mode != "sharded":
        return _local_coordinator(cfg)
    return _local_rendezvous(cfg) if cfg.ownership.mode == "rendezvous" else _local_sharded(cfg)


def _start(target, **kw):
    """Run ``target(on_start=...)`` in a daemon thread; return (server, thread, result box)."""
    box, ready = {}, threading.Event()

    def on_start(s):
        box["server"] = s
        ready.set()

    th = threading.Thread(target=lambda: box.__setitem__("result", target(on_start=on_start, **kw)), daemon=True)
    th.start()
    if not ready.wait(timeout=120):
        raise RuntimeError(f"{getattr(target, '__name__', target)} did not start")
    return box["server"], th, box


def _workers(cfg, **kw):
    ws = [threading.Thread(target=run_worker_role, kwargs=dict(cfg=cfg, **kw), daemon=True)
          for _ in range(cfg.run.local_workers)]
    for w in ws:
        w.start()
    return ws


def _local_coordinator(cfg: LaunchConfig):
    server, th, box = _start(run_coordinator, cfg=cfg)
    ws = _workers(cfg, addr=("127.0.0.1", server.port))
    th.join()
    for w in ws:
        w.join(timeout=5)
    return box["result"]


def _local_sharded(cfg: LaunchConfig):
    n = cfg.sharded.num_shards
    stops = [threading.Event() for _ in range(n)]
    pss = [_start(run_parameter_server, cfg=cfg, shard_id=i, port=0, stop_event=stops[i]) for i in range(n)]
    sched, th, box = _start(run_scheduler, cfg=cfg, ps_addrs=[("127.0.0.1", ps.port) for ps, _, _ in pss])
    ws = _workers(cfg, scheduler_addr=("127.0.0.1", sched.port), stop_event=threading.Event())
    th.join()
    for s in stops:
        s.set()
    for _, t, _ in pss:
        t.join(timeout=10)
    for w in ws:
        w.join(timeout=5)
    sched, completed = box["result"]
    # the trained global modules, read from their owners (for evaluation after the run)
    sched.owner_banks = {k: ps.bank[k] for ps, _, _ in pss for k in ps.owned_keys}
    return sched, completed


def _local_rendezvous(cfg: LaunchConfig):
    n = cfg.sharded.num_shards
    if cfg.transport.auth_key is None:
        cfg.transport.auth_key = os.urandom(16).hex()
    sched_id = PeerIdentity.generate()
    owner_ids = [PeerIdentity.generate() for _ in range(n)]
    tracker = Tracker(host="127.0.0.1", port=0, open_enrollment=True, ttl=cfg.tracker.ttl,
                      auth_key=cfg.transport.auth_key)
    tracker.start()
    taddr = ("127.0.0.1", tracker.port)
    sched, th, box = _start(run_scheduler, cfg=cfg, identity=sched_id, tracker_addr=taddr)
    saddr = ("127.0.0.1", sched.port)
    stops = [threading.Event() for _ in range(n)]
    pts = [threading.Thread(target=run_parameter_server, kwargs=dict(
        cfg=cfg, port=0, identity=owner_ids[i], scheduler_addr=saddr, tracker_addr=taddr,
        scheduler_pub=sched_id.public_key_hex, stop_event=stops[i]), daemon=True) for i in range(n)]
    for t in pts:
        t.start()
    ws = _workers(cfg, scheduler_addr=saddr, stop_event=threading.Event())
    th.join()
    for s in stops:
        s.set()
    for t in pts:
        t.join(timeout=10)
    tracker.shutdown()
    for w in ws:
        w.join(timeout=5)
    return box["result"]


class DecentralizedCluster:
    """What a local decentralized run returns: a representative ``metrics`` and the
    merged bank read from each key's primary before shutdown."""

    def __init__(self, metrics, bank):
        self.metrics, self._bank = metrics, bank

    def merged_bank(self) -> dict:
        return self._bank


def _local_decentralized(cfg: LaunchConfig):
    n, own = cfg.sharded.num_shards, cfg.ownership
    if cfg.transport.auth_key is None:
        cfg.transport.auth_key = os.urandom(16).hex()
    auth = cfg.transport.auth_key
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    corpus = build_server_corpus(cfg, model)
    topo = model.build_topology()
    tracker = Tracker(host="127.0.0.1", port=0, open_enrollment=True, ttl=cfg.tracker.ttl, auth_key=auth)
    tracker.start()
    taddr = ("127.0.0.1", tracker.port)
    weights = {p: corpus.shard_weight(p) for p in range(model.num_paths)}
    t = cfg.transport
    owners = []
    for _ in range(n):
        ps = ParameterServer(model, [], diloco, host="127.0.0.1", port=0, identity=PeerIdentity.generate(),
                             replicate_interval=own.replicate_interval, bank_seed=own.bank_seed,
                             corpus_weights=weights, peer_tls=build_tls_client(cfg), device=cfg.run.device,
                             grant_key=t.grant_key, max_update_norm=t.max_update_norm, compress=t.compress,
                             down=t.down, **_decentralized_kw(cfg), **_ps_robust_kw(cfg), **_server_kw(cfg))
        ps.start()
        owners.append(ps)
    by_id = {ps.peer_id: ps for ps in owners}
    # cold start: every owner serves its identically seeded bank under one derived epoch
    recs = [make_peer_record(ps.identity, reachability="public", addr=("127.0.0.1", ps.port), roles=["owner"])
            for ps in owners]
    epoch0 = derive_epoch(recs, k=own.k, salt=own.salt)
    for ps in owners:
        ps.apply_epoch(epoch0, bootstrap=True)
        ps.start_tracker_heartbeat(taddr, "127.0.0.1", interval=own.heartbeat_interval, auth_key=auth,
                                   seeds=cfg.tracker.seeds)
    stop = threading.Event()
    ws = [threading.Thread(target=run_decentralized_worker, args=(model, diloco, taddr, corpus), kwargs=dict(
        identity=PeerIdentity.generate(), device=cfg.run.device, seed=cfg.run.seed, auth_key=auth, k=own.k,
        salt=own.salt, read_quorum=cfg.schedule.read_quorum, lease_ttl=cfg.schedule.lease_ttl,
        batch_size=cfg.run.batch_size, total_rounds=cfg.run.generations, heartbeat_interval=own.heartbeat_interval,
        stop_event=stop, seeds=cfg.tracker.seeds, seed_quorum=cfg.tracker.seed_quorum), daemon=True)
        for _ in range(cfg.run.local_workers)]
    for w in ws:
        w.start()
    target, completed = cfg.run.generations, {}
    deadline = time.monotonic() + DECENTRALIZED_RUN_TIMEOUT
    try:
        while time.monotonic() < deadline:
            for path in topo.paths():
                prim = path_primary(topo.path_module_keys(path), epoch0)
                ps = by_id.get(prim["peer_id"]) if prim else None
                completed[topo.path_index(path)] = ps.generation_of(path)
            if all(v >= target for v in completed.values()):
                break
            time.sleep(0.05)
    finally:
        stop.set()
        for w in ws:
            w.join(timeout=10)
        bank = {}
        for key in topo.module_keys():
            ps = by_id[owners_for(key, epoch0)[0]["peer_id"]]
            with ps._lock:
                bank[key] = {nm: v.detach().cpu().clone() for nm, v in ps.bank[key].state_dict().items()}
        for ps in owners:
            ps.shutdown(graceful=True)
        tracker.shutdown()
    if any(v < target for v in completed.values()):
        print(f"WARNING: local decentralized run stopped at the {DECENTRALIZED_RUN_TIMEOUT:.0f}s limit before "
              f"every path reached generation {target}: {completed}", flush=True)
    return DecentralizedCluster(owners[0].metrics, bank), completed
