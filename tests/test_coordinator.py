"""The TCP coordinator's policies, driven message by message (CPU): staleness bound,
fencing of a reclaimed lease, heartbeats, nack, warm shipping of private and unchanged
shared weights, update-norm clipping and non-finite rejection, idle backoff and batch
caps; plus the transport's
connection cap and a bounded handler pool serving many clients at once.

Behaviours of the reference's ``tests/test_scheduler_distributed.py``
(``src/opendipaco/schedule/distributed.py``).
"""

import socket
import threading
import time

import torch

from opendipaco_b200.schedule import AsyncScheduler, CoordinatorServer
from opendipaco_b200.schedule.reactor import ReactorServer
from opendipaco_b200.schedule.rpc import one_shot
from opendipaco_b200.topology import is_private_key

from helpers import engine, rr_corpus, tiny_config


def _coord(cfg=None, **kw):
    cfg = cfg or tiny_config()
    e = engine(cfg)
    c = CoordinatorServer(AsyncScheduler(e), rr_corpus(cfg), 4, host="127.0.0.1", **kw)
    from opendipaco_b200.optim.diloco import make_outer_optimizer

    c._outer_opts = {k: make_outer_optimizer({k: e.bank[k]}, e.diloco) for k in c._versions}
    with c._lock:  # what fit() sets up, without its serving loop
        c._target = 10 ** 6
        c._serving = True
    return c, e


def _req(c, w, **extra):
    return c._handle({"type": "request", "worker_id": w, **extra}, 0)


def _submit(c, t, e, scale=1e-3, **extra):
    keys = [k for k in e.topology.path_module_keys(tuple(t["path"])) if not is_private_key(k)]
    grad = {k: [torch.full_like(p, scale) for p in e.bank[k].parameters()] for k in keys}
    msg = {"type": "submit", "path": list(t["path"]), "lease": t["lease"], "shared_grad": grad,
           "private_weights": {}, "loss": 1.0, **extra}
    return c._handle(msg, 0)["applied"]


def test_staleness_bound_rejects_old_leases():
    c, e = _coord(staleness_bound=1)
    old = _req(c, "slow")
    for _ in range(2):  # two updates land while the slow worker trains
        t = _req(c, "fast")
        assert _submit(c, t, e)
    assert not _submit(c, old, e)
    assert c.metrics.summary()["stale_rejected"] == 1


def test_reclaimed_lease_is_fenced():
    """A worker whose lease ran out (no heartbeat) cannot submit once the path was handed
    to someone else; the new holder's submission lands."""
    c, e = _coord(heartbeat_timeout=0.05)
    paths = list(e.topology.paths())
    zombie = _req(c, "zombie")
    others = [_req(c, f"w{i}") for i in range(len(paths) - 1)]  # every other path busy
    time.sleep(0.1)
    with c._lock:
        c._expire_locked()
    fresh = _req(c, "fresh")
    assert tuple(fresh["path"]) == tuple(zombie["path"]) and fresh["lease"] != zombie["lease"]
    assert not _submit(c, zombie, e)
    assert _submit(c, fresh, e)
    assert c.metrics.reclaims >= 1 and others


def test_heartbeat_keeps_a_lease_alive_and_nack_frees_it():
    c, e = _coord(heartbeat_timeout=0.2)
    t = _req(c, "w")
    for _ in range(4):
        time.sleep(0.08)
        c._handle({"type": "heartbeat", "path": list(t["path"]), "lease": t["lease"]}, 0)
        with c._lock:
            c._expire_locked()
    assert c._records[tuple(t["path"])].lease == t["lease"]
    c._handle({"type": "nack", "path": list(t["path"]), "lease": t["lease"], "error": "oom"}, 0)
    assert c._records[tuple(t["path"])].lease is None and c.sched.errors[tuple(t["path"])] == "oom"
    assert not _submit(c, t, e)  # the lease is gone


def test_warm_worker_gets_neither_private_nor_unchanged_shared_weights():
    cfg = tiny_config(embedding="private", head="private")
    c, e = _coord(cfg)
    cold = _req(c, "w")
    path = tuple(cold["path"])
    assert set(cold["private_weights"]) == {k for k in e.topology.path_module_keys(path) if is_private_key(k)}
    assert set(cold["shared_weights"]) == set(cold["shared_versions"])
    c._handle({"type": "nack", "path": list(path), "lease": cold["lease"]}, 0)
    warm = _req(c, "w", warm_paths=[list(path)], have_shared=cold["shared_versions"])
    assert tuple(warm["path"]) == path
    assert warm["private_weights"] is None and warm["shared_weights"] == {}
    # no optimizer state is ever shipped
    assert not any("exp_avg" in str(k) or "momentum" in str(k) for k in warm)


def test_update_norm_is_clipped_and_non_finite_updates_rejected():
    c, e = _coord(max_update_norm=1e-3)
    t = _req(c, "w")
    assert _submit(c, t, e, scale=1.0)
    assert c.metrics.summary()["norm_clipped"] >= 1
    t = _req(c, "w")
    assert not _submit(c, t, e, scale=float("nan"))
    t = _req(c, "w")
    assert not _submit(c, t, e, loss=float("inf"))
    assert c.metrics.summary()["invalid_rejected"] == 2


def test_connection_cap_refuses_excess_clients():
    srv = ReactorServer(host="127.0.0.1", port=0, max_connections=1)
    srv._handle = lambda msg, nbytes, peer_id=None: {"type": "pong"}
    srv.start()
    try:
        first = socket.create_connection(("127.0.0.1", srv.port), timeout=5)
        time.sleep(0.1)  # the first session is registered
        second = socket.create_connection(("127.0.0.1", srv.port), timeout=5)
        second.settimeout(5)
        assert second.recv(1) == b""  # closed by the server without a byte
        first.close()
        second.close()
        time.sleep(0.1)
        assert one_shot(("127.0.0.1", srv.port), {"type": "ping"})["type"] == "pong"
    finally:
        srv.shutdown()


def test_bounded_handler_pool_serves_many_clients():
    srv = ReactorServer(host="127.0.0.1", port=0, io_threads=2)
    seen = set()

    def handle(msg, nbytes, peer_id=None):
        seen.add(threading.current_thread().name)
        time.sleep(0.02)
        return {"type": "echo", "i": msg["i"]}

    srv._handle = handle
    srv.start()
    out = {}
    try:
        def client(i):
            out[i] = one_shot(("127.0.0.1", srv.port), {"type": "x", "i": i})["i"]

        ths = [threading.Thread(target=client, args=(i,)) for i in range(24)]
        for t in ths:
            t.start()
        for t in ths:
            t.join(timeout=30)
    finally:
        srv.shutdown()
    assert out == {i: i for i in range(24)} and 1 <= len(seen) <= 2


def test_idle_replies_carry_the_backoff_and_batches_are_capped():
    c, e = _coord(idle_backoff=0.7)
    paths = list(e.topology.paths())
    held = [_req(c, f"w{i}") for i in range(len(paths))]  # every path leased
    idle = _req(c, "late")
    assert idle["type"] == "idle" and idle["retry_in"] == 0.7
    c._handle({"type": "nack", "path": list(held[0]["path"]), "lease": held[0]["lease"]}, 0)
    small = _req(c, "small", capabilities={"max_batch": 2})
    assert small["type"] == "task" and small["batch_size"] == 2
    plain, _ = _coord()
    for i in range(len(paths)):
        _req(plain, f"w{i}")
    assert _req(plain, "late") == {"type": "idle"}  # no backoff configured: the worker's own poll
