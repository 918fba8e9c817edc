"""Scheduler-less (decentralized) coordination on the owners (CPU): the path's
coordinating owner fences generations, checks the HRW assignee with takeover, rate
limits, guards the loss and the base-version lag, and mints a grant its co-owners
verify against the epoch; co-owner replicas are audited by digest and a divergent one
loses reputation until it drops out of the derived epoch.

Behaviours of the reference's ``tests/test_decentralized.py`` and the owner-audit part
of ``tests/test_decentralized_worker.py`` (``src/opendipaco/schedule/sharded.py``
decentralized coordination).
"""

import time

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import ParameterServer, PeerIdentity, RateLimiter, Reputation, make_peer_record
from opendipaco_b200.schedule.assignment import coordinator_key, rank_workers
from opendipaco_b200.schedule.ownership import derive_epoch, owners_for
from opendipaco_b200.schedule.sharded import grant_signed_by, make_grant

from helpers import tiny_config

DL = DiLoCoConfig(inner_steps=2, inner_lr=1e-3)
KEY = "cluster-secret"


def _cluster(n=3, k=3, embedding="private", **kw):
    """``n`` dynamic decentralized owners on loopback under one derived epoch."""
    cfg = tiny_config(embedding=embedding, head=embedding)
    ids = [PeerIdentity.generate() for _ in range(n)]
    owners = [ParameterServer(cfg, [], DL, host="127.0.0.1", identity=i, schedule_mode="decentralized", k=k,
                              replicate_interval=3600, auth_key=KEY, **kw) for i in ids]
    for ps in owners:
        ps.start()
    recs = [make_peer_record(ps.identity, reachability="public", addr=("127.0.0.1", ps.port), roles=["owner"])
            for ps in owners]
    epoch = derive_epoch(recs, k=k)
    for ps in owners:
        ps.apply_epoch(epoch, bootstrap=True)
    return cfg, owners, epoch


def _coord(owners, epoch, path):
    keys = owners[0]._topology.path_module_keys(path)
    pid = owners_for(coordinator_key(keys), epoch)[0]["peer_id"]
    return next(ps for ps in owners if ps.peer_id == pid)


def _base(ps, path):
    return {k: list(ps._versions[k]) for k in ps._topology.path_module_keys(path) if k in ps._active}


def _commit(ps, path, gen, member="w", loss=1.0, base=None):
    return ps._commit({"path": list(path), "gen_id": gen, "loss": loss, "worker_id": member,
                       "base_versions": _base(ps, path) if base is None else base}, member)


@pytest.fixture
def cluster():
    made = []

    def make(**kw):
        c = _cluster(**kw)
        made.extend(c[1])
        return c

    yield make
    for ps in made:
        ps.shutdown()


def test_coordinator_mints_a_signed_grant_and_fences_the_generation(cluster):
    cfg, owners, epoch = cluster()
    path = (0, 0)
    c = _coord(owners, epoch, path)
    g = c._generation({"path": [0, 0]})
    assert g["ok"] and g["generation"] == 0 and g["age"] >= 0
    out = _commit(c, path, 0)
    assert out["accepted"] and out["generation"] == 1 and grant_signed_by(out["grant"], c.peer_id)
    again = _commit(c, path, 0, member="w2")
    assert not again["accepted"] and again["reason"] == "stale_generation" and again["generation"] == 1
    assert _commit(c, path, 1, member="w2")["accepted"] and c.generation_of(path) == 2


def test_only_the_coordinator_and_only_in_decentralized_mode(cluster):
    cfg, owners, epoch = cluster()
    path = (1, 0)
    c = _coord(owners, epoch, path)
    other = next(ps for ps in owners if ps is not c)
    assert _commit(other, path, 0)["reason"] == "not_coordinator"
    assert not other._generation({"path": [1, 0]})["ok"]
    assert c._commit({"path": [9, 9], "gen_id": 0, "loss": 1.0}, "w")["reason"] == "bad_path"
    central = ParameterServer(cfg, cfg.build_topology().module_keys(), DL, host="127.0.0.1",
                              identity=PeerIdentity.generate())
    assert _commit(central, path, 0, base={})["reason"] == "not_decentralized"
    with pytest.raises(ValueError):
        ParameterServer(cfg, [], DL, identity=PeerIdentity.generate(), schedule_mode="decentralized",
                        compress="int8")
    with pytest.raises(ValueError):
        ParameterServer(cfg, [], DL, identity=PeerIdentity.generate(), schedule_mode="gossip")


def test_loss_guard_debits_and_acceptance_credits(cluster):
    rep = Reputation(floor=0.5, credit=0.1, debit=0.3, decay_halflife=0)
    cfg, owners, epoch = cluster(reputation=rep)
    path = (0, 1)
    c = _coord(owners, epoch, path)
    bad = c._commit({"path": [0, 1], "gen_id": 0, "loss": float("nan"), "base_versions": {}}, "liar")
    assert bad["reason"] == "bad_loss" and rep.get("liar") < 0.5 and c.generation_of(path) == 0
    assert _commit(c, path, 0, member="honest")["accepted"] and rep.get("honest") > 0.5


def test_throttled_committer_gets_no_grant(cluster):
    cfg, owners, epoch = cluster(rate_limiter=RateLimiter(capacity=1.0, refill_per_sec=0.0))
    path = (1, 1)
    c = _coord(owners, epoch, path)
    assert _commit(c, path, 0, member="busy")["accepted"]
    out = _commit(c, path, 1, member="busy")
    assert out["reason"] == "throttled" and "grant" not in out and c.generation_of(path) == 1


def test_stale_or_cross_epoch_base_is_rejected(cluster):
    cfg, owners, epoch = cluster(staleness_bound=1)
    path = (0, 0)
    c = _coord(owners, epoch, path)
    key = next(k for k in _base(c, path))
    base = _base(c, path)
    e, n = c._versions[key]
    c._versions[key] = (e, n + 3)  # three updates landed since the worker's fetch
    assert _commit(c, path, 0, base=base)["reason"] == "stale"
    cross = dict(base, **{key: [e + 7, n + 3]})
    assert _commit(c, path, 0, base=cross)["reason"] == "stale"
    assert _commit(c, path, 0, base=dict(base, **{key: [e, n + 2]}))["accepted"]  # lag 1: within the bound
    assert c.metrics.summary()["stale_rejected"] == 2


def test_only_the_hrw_assignee_commits_until_its_slot_times_out(cluster):
    workers = ["wa", "wb", "wc"]
    cfg, owners, epoch = cluster(worker_set=lambda: workers, lease_ttl=0.2)
    path = (1, 0)
    c = _coord(owners, epoch, path)
    ranked = rank_workers(path, 0, workers)
    assert _commit(c, path, 0, member=ranked[1])["reason"] == "not_assignee"
    c._generation({"path": list(path)})
    c._gen_counters[path][1] -= 0.25  # the slot has been open past one lease: the successor may take it
    assert _commit(c, path, 0, member=ranked[1])["accepted"]
    assert _commit(c, path, 1, member=rank_workers(path, 1, workers)[0])["accepted"]


def test_co_owner_accepts_only_the_coordinators_grant(cluster):
    cfg, owners, epoch = cluster()
    path = (0, 1)
    c = _coord(owners, epoch, path)
    co = next(ps for ps in owners if ps is not c)
    key = next(k for k in cfg.build_topology().path_module_keys(path) if not k.startswith(("embed", "head")))
    grad = [torch.full(tuple(p.shape), 1e-3) for p in co.bank[key].parameters()]
    ack = _commit(c, path, 0)
    assert co._push({"grant": ack["grant"], "updates": {key: {"grad": grad}}, "private": {}})["applied"]
    assert co._versions[key][1] == 1
    assert not co._push({"grant": ack["grant"], "updates": {key: {"grad": grad}}, "private": {}})["applied"]
    forged = make_grant(path, cfg.build_topology().path_module_keys(path), 1.0, "tok", identity=co.identity)
    assert not co._push({"grant": forged, "updates": {key: {"grad": grad}}, "private": {}})["applied"]
    assert co._versions[key][1] == 1


def test_replica_audit_blames_only_a_diverged_replica(cluster):
    cfg, owners, epoch = cluster()
    a, b, z = owners
    key = sorted(a._active & b._active & z._active)[0]
    with z._lock:  # z silently corrupts its copy without changing the version
        next(iter(z.bank[key].parameters())).data.add_(1.0)
    flagged = a.audit_replicas_once()
    assert flagged.get(key) == {z.peer_id}
    assert a.reputation.get(z.peer_id) < a.reputation.floor <= a.reputation.get(b.peer_id)
    # a replica that is only behind is not blamed
    reports = {key: {"p": ((0, 4), "aa"), "q": ((0, 4), "aa"), "r": ((0, 3), "old")}}
    assert a.apply_replica_audit(reports) == {}


def test_repeatedly_divergent_owner_drops_out_of_the_derived_epoch(cluster):
    cfg, owners, epoch = cluster(min_owner_reputation=0.3)
    a, b, z = owners
    key = sorted(a._active & z._active)[0]
    with z._lock:
        next(iter(z.bank[key].parameters())).data.add_(1.0)
    for _ in range(3):
        a.audit_replicas_once()
    recs = [make_peer_record(ps.identity, reachability="public", addr=("127.0.0.1", ps.port), roles=["owner"])
            for ps in owners]
    nxt = derive_epoch(recs, k=3, prev=epoch,
                       is_eligible=lambda pid: a.reputation.get(pid) >= a.min_owner_reputation)
    assert {o["peer_id"] for o in nxt["owners"]} == {a.peer_id, b.peer_id} and nxt["epoch"] == epoch["epoch"] + 1


def test_decentralized_workers_train_every_path_over_tcp(cluster):
    """Two self-assigning workers commit each path's generations to its coordinator and
    push to every owner; the co-owners of every shared key end bit-identical."""
    import threading

    from opendipaco_b200.schedule import run_decentralized_worker

    from helpers import rr_corpus

    cfg, owners, epoch = cluster(embedding="shared")
    corpus = rr_corpus(cfg)
    ids = [PeerIdentity.generate() for _ in range(2)]
    stop = threading.Event()
    ths = [threading.Thread(target=run_decentralized_worker, args=(cfg, DL, lambda: epoch, corpus),
                            kwargs=dict(identity=i, auth_key=KEY, batch_size=2, total_rounds=2, stop_event=stop,
                                        workers_fn=lambda: [x.peer_id for x in ids], lease_ttl=5.0),
                            daemon=True) for i in ids]
    for t in ths:
        t.start()
    topo = cfg.build_topology()
    deadline = time.monotonic() + 120
    while time.monotonic() < deadline and not all(
            _coord(owners, epoch, p).generation_of(p) >= 2 for p in topo.paths()):
        time.sleep(0.1)
    stop.set()
    for t in ths:
        t.join(timeout=30)
    assert all(_coord(owners, epoch, p).generation_of(p) >= 2 for p in topo.paths())
    time.sleep(0.2)
    for key in topo.module_keys():
        reps = [ps for ps in owners if key in ps._active]
        states = [ps.bank[key].state_dict() for ps in reps]
        assert all(torch.equal(states[0][n], s[n]) for s in states[1:] for n in states[0]), key
        assert len({ps._versions[key] for ps in reps}) == 1


def test_owners_keep_converging_by_gossip_after_the_tracker_is_gone():
    """Decentralized owners fed by a tracker: once it is gone they exchange their
    directories, and an owner that crashes ages out of every survivor's derived epoch."""
    from opendipaco_b200.schedule import Tracker

    cfg = tiny_config()
    tracker = Tracker(host="127.0.0.1", open_enrollment=True, ttl=30.0)
    tracker.start()
    ids = [PeerIdentity.generate() for _ in range(3)]
    owners = [ParameterServer(cfg, [], DL, host="127.0.0.1", identity=i, schedule_mode="decentralized", k=2,
                              replicate_interval=0.2, auth_key=KEY, directory_ttl=3.0) for i in ids]
    try:
        for ps in owners:
            ps.start()
            ps.start_tracker_heartbeat(("127.0.0.1", tracker.port), "127.0.0.1", interval=0.3)

        def converged(pss, n):
            eps = [ps._epoch for ps in pss]
            return all(e is not None and len(e["owners"]) == n for e in eps) and len({e["epoch"] for e in eps}) == 1

        deadline = time.monotonic() + 15
        while time.monotonic() < deadline and not converged(owners, 3):
            time.sleep(0.1)
        assert converged(owners, 3)
        tracker.shutdown()
        owners[2].simulate_crash()
        deadline = time.monotonic() + 20
        while time.monotonic() < deadline and not converged(owners[:2], 2):
            time.sleep(0.1)
        assert converged(owners[:2], 2)
        assert {o["peer_id"] for o in owners[0]._epoch["owners"]} == {ids[0].peer_id, ids[1].peer_id}
        assert owners[0].directory()[0]["peer_id"] == ids[0].peer_id  # its own record first
    finally:
        for ps in owners:
            ps.shutdown()
        tracker.shutdown()


def test_workers_read_the_owners_directories_when_every_seed_is_gone():
    from opendipaco_b200.schedule.sharded import _owner_directories

    a, b, c = (PeerIdentity.generate() for _ in range(3))
    old = make_peer_record(c, reachability="public", addr=("10.0.0.3", 1), roles=["owner"])
    time.sleep(0.01)
    new = make_peer_record(c, reachability="public", addr=("10.0.0.3", 2), roles=["owner"])
    dirs = {"x": [make_peer_record(a, roles=["worker"]), old], "y": [new, dict(old, roles=["scheduler"])]}

    class _Link:
        def ps_rpc(self, addr, msg):
            if addr == "dead":
                raise ConnectionError("gone")
            assert msg == {"type": "directory"}
            return {"records": dirs[addr]}

    epoch = {"owners": [{"addr": "x"}, {"addr": "dead"}, {"addr": "y"}]}
    got = {r["peer_id"]: r for r in _owner_directories(_Link(), epoch)}
    assert set(got) == {a.peer_id, c.peer_id} and got[c.peer_id]["addr"] == ["10.0.0.3", 2]  # newest, tamper dropped
    assert b.peer_id not in got
