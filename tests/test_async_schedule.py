"""Async scheduler and TCP coordinator/worker (failures injected on the host)."""

import threading

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig, DiPaCoEngine, LocalBackend
from opendipaco_b200.schedule.distributed import CoordinatorServer, run_worker
from opendipaco_b200.schedule.scheduler import AsyncScheduler, Preempt, TransientFault, task_seed

from helpers import rr_corpus, tiny_config


def _engine(cfg, **dl):
    d = dict(inner_steps=2, inner_lr=1e-3)
    d.update(dl)
    return DiPaCoEngine(cfg, DiLoCoConfig(**d), LocalBackend(cfg.build_topology()), seed=0, materialize="serial")


def _bank(e):
    return {k: torch.cat([p.detach().reshape(-1) for p in m.parameters()]) for k, m in e.bank.items()}


def test_results_independent_of_worker_count_and_faults():
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    a = AsyncScheduler(_engine(cfg), num_workers=1)
    a.fit(corpus, 2, 4, log_every=0)
    b = AsyncScheduler(_engine(cfg), num_workers=3, lease_timeout=0.2)
    hits = {}

    def hook(path, attempt):
        hits[path] = hits.get(path, 0) + 1
        if path == (0, 1) and attempt == 1:
            raise TransientFault()
        if path == (1, 0) and attempt == 1:
            raise Preempt()

    b.fit(corpus, 2, 4, log_every=0, fault_hook=hook)
    assert hits[(0, 1)] >= 2 and hits[(1, 0)] >= 2 and not b.dropped
    ba, bb = _bank(a.engine), _bank(b.engine)
    for k in ba:
        assert torch.allclose(ba[k], bb[k], atol=1e-5), k


def test_path_dropped_after_max_attempts():
    cfg = tiny_config()
    s = AsyncScheduler(_engine(cfg), num_workers=2, max_attempts=2)

    def hook(path, attempt):
        if path == (1, 1):
            raise TransientFault()

    m = s.fit(rr_corpus(cfg), 1, 4, log_every=0, fault_hook=hook)[0]
    assert s.dropped == {(1, 1)} and (1, 1) not in m.per_path_loss
    assert "TransientFault" in s.errors[(1, 1)]


def test_task_seed_constants():
    assert task_seed(0, 0, 0) == 0
    assert task_seed(1, 2, 3) == ((0x9E3779B1) ^ (2 * 0x85EBCA77) ^ (3 * 0xC2B2AE35)) & 0x7FFFFFFFFFFFFFFF


@pytest.mark.parametrize("compress", ["none", "int8", "int4"])
def test_coordinator_worker_over_tcp(compress):
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    coord_engine = _engine(cfg)
    server = CoordinatorServer(AsyncScheduler(coord_engine), corpus, 4, host="127.0.0.1", port=0,
                               auth_key="s3cret", compress=compress, heartbeat_timeout=5.0)
    server.start()
    before = _bank(coord_engine)
    done = {}

    def serve():
        done["completed"] = server.fit(1)

    th = threading.Thread(target=serve)
    th.start()
    workers = [threading.Thread(target=run_worker, kwargs=dict(config=cfg, diloco=coord_engine.diloco,
                                                               host="127.0.0.1", port=server.port,
                                                               auth_key="s3cret", max_tasks=3,
                                                               reconnect=False))
               for _ in range(2)]
    for w in workers:
        w.start()
    th.join(timeout=120)
    server.shutdown()
    for w in workers:
        w.join(timeout=30)
    s = server.metrics.summary()
    assert s["accepted_updates"] >= 4 and s["bytes_opt"] == 0
    assert all(v >= 1 for v in done["completed"].values())
    after = _bank(coord_engine)
    assert any(not torch.equal(before[k], after[k]) for k in before)
    assert "opendipaco_transport_bytes_opt_total 0" in server.metrics.prometheus()


def test_worker_with_wrong_key_is_refused():
    cfg = tiny_config()
    server = CoordinatorServer(AsyncScheduler(_engine(cfg)), rr_corpus(cfg), 4, host="127.0.0.1", port=0,
                               auth_key="right")
    server.start()
    try:
        with pytest.raises((PermissionError, ConnectionError)):
            run_worker(cfg, DiLoCoConfig(inner_steps=1), "127.0.0.1", server.port, auth_key="wrong",
                       reconnect=False, connect_timeout=2.0)
    finally:
        server.shutdown()
