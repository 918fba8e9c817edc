"""Sharded scheduler / parameter servers / tracker / epochs, all on loopback TCP (CPU).

Mirrors the reference's ``tests/test_sharded*.py``, ``tests/test_tracker*.py`` and
``tests/test_ownership*.py`` coverage: grant signing and replay, shape screening,
end-to-end generations, checkpoint + resume, epochs and primary-only writes,
replication, directory admission and multi-seed union.
"""

import os
import threading
import time

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import (EpochManager, ParameterServer, PeerIdentity, Scheduler, Tracker,
                                      assign_shards, derive_epoch, deregister_peer, fetch_directory,
                                      fetch_directory_multi, get_epoch, grant_signed_by, make_epoch_record,
                                      make_grant, make_peer_record, owners_for, put_epoch, register_peer,
                                      run_sharded_worker, verify_epoch_record, verify_grant)
from opendipaco_b200.schedule.rpc import one_shot

from helpers import rr_corpus, tiny_config

KEY = "k3y"


def _diloco():
    return DiLoCoConfig(inner_steps=2, inner_lr=1e-3)


def _servers(cfg, n, **kw):
    keys = cfg.build_topology().module_keys()
    place = assign_shards(keys, n)
    out = []
    for i in range(n):
        ps = ParameterServer(cfg, [k for k, j in place.items() if j == i], _diloco(), host="127.0.0.1",
                             auth_key=KEY, grant_key="g", **kw)
        ps.start()
        out.append(ps)
    return out


def _state(servers):
    out = {}
    for ps in servers:
        for k, m in ps.bank.items():
            out[k] = {n: p.detach().clone() for n, p in m.state_dict().items()}
    return out


# ------------------------------------------------------------------------ grants
def test_grant_hmac_and_ed25519():
    g = make_grant((0, 1), ["b", "a"], 0.25, "tok", "secret")
    assert g["keys"] == ["a", "b"] and verify_grant(g, "secret")
    assert not verify_grant(g, "other")
    assert not verify_grant(dict(g, weight=0.5), "secret")
    ident = PeerIdentity.generate()
    sg = make_grant((0, 1), ["a"], 1.0, "t2", identity=ident)
    assert verify_grant(sg, None, scheduler_pub=ident.public_key_hex)
    assert not verify_grant(sg, None, scheduler_pub=PeerIdentity.generate().public_key_hex)
    assert grant_signed_by(sg, ident.peer_id) and not grant_signed_by(sg, "x" * 64)


def test_assign_shards_round_robin():
    assert assign_shards(["c", "a", "b", "d"], 2) == {"a": 0, "b": 1, "c": 0, "d": 1}


# ------------------------------------------------------------------------ push screening
def test_push_replay_and_shape_checks():
    cfg = tiny_config()
    (ps,) = _servers(cfg, 1)
    try:
        key = "L0E0"
        shapes = [tuple(p.shape) for p in ps.bank[key].parameters()]
        grad = [torch.full(s, 1e-3) for s in shapes]
        g = make_grant((0, 0), [key], 1.0, "t1", "g")
        send = lambda m: one_shot(("127.0.0.1", ps.port), m, auth_key=KEY)  # noqa: E731
        assert send({"type": "push", "grant": g, "updates": {key: {"grad": grad}}, "private": {}})["applied"]
        assert ps._versions[key] == (0, 1)
        assert not send({"type": "push", "grant": g, "updates": {key: {"grad": grad}}, "private": {}})["applied"]
        bad = [torch.zeros(3)] + grad[1:]
        g2 = make_grant((0, 0), [key], 1.0, "t2", "g")
        assert not send({"type": "push", "grant": g2, "updates": {key: {"grad": bad}}, "private": {}})["applied"]
        nan = [torch.full(s, float("nan")) for s in shapes]
        g3 = make_grant((0, 0), [key], 1.0, "t3", "g")
        assert not send({"type": "push", "grant": g3, "updates": {key: {"grad": nan}}, "private": {}})["applied"]
        forged = dict(make_grant((0, 0), [key], 1.0, "t4", "g"), weight=100.0)
        assert not send({"type": "push", "grant": forged, "updates": {key: {"grad": grad}}, "private": {}})["applied"]
        assert ps._versions[key] == (0, 1)
        assert ps.metrics.invalid_rejected >= 2
    finally:
        ps.shutdown()


def test_robust_buffer_applies_aggregate_at_quorum():
    cfg = tiny_config()
    (ps,) = _servers(cfg, 1, robustness="quorum", quorum_target=3, aggregate="median")
    try:
        key = "embed"
        shapes = [tuple(p.shape) for p in ps.bank[key].parameters()]
        before = [p.detach().clone() for p in ps.bank[key].parameters()]
        vals = [1e-3, 2e-3, 1e3]   # the outlier must not move the median
        for i, v in enumerate(vals):
            g = make_grant((0, 0), [key], 1.0, f"t{i}", "g")
            one_shot(("127.0.0.1", ps.port), {"type": "push", "grant": g,
                                               "updates": {key: {"grad": [torch.full(s, v) for s in shapes]}},
                                               "private": {}}, auth_key=KEY)
            assert ps._versions[key] == ((0, 1) if i == 2 else (0, 0))
        after = list(ps.bank[key].parameters())
        # SGD(lr, nesterov) first step on the summed weight (3.0) times the median (2e-3)
        lr, mom = ps.diloco.outer_lr, ps.diloco.outer_momentum
        exp = before[0] - lr * (1 + mom) * 3.0 * 2e-3
        torch.testing.assert_close(after[0].detach(), exp, rtol=1e-5, atol=1e-6)
    finally:
        ps.shutdown()


# ------------------------------------------------------------------------ end to end
def _run_cluster(cfg, corpus, servers, *, generations=1, workers=2, ckpt=None, **skw):
    sch = Scheduler(cfg, corpus, [("127.0.0.1", ps.port) for ps in servers], _diloco(), 4, host="127.0.0.1",
                    auth_key=KEY, grant_key="g", heartbeat_timeout=10.0, **skw)
    sch.start()
    out = {}
    th = threading.Thread(target=lambda: out.setdefault("c", sch.fit(generations, checkpoint_dir=ckpt,
                                                                    checkpoint_every=1000 if ckpt else 0)))
    th.start()
    stop = threading.Event()
    ws = [threading.Thread(target=run_sharded_worker, args=(cfg, _diloco(), ("127.0.0.1", sch.port)),
                           kwargs=dict(auth_key=KEY, stop_event=stop)) for _ in range(workers)]
    for w in ws:
        w.start()
    th.join(timeout=180)
    stop.set()
    sch.shutdown()
    for w in ws:
        w.join(timeout=30)
    assert not th.is_alive()
    return sch, out["c"]


@pytest.mark.parametrize("compress", ["none", "int8"])
def test_sharded_generation_end_to_end(compress):
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    servers = _servers(cfg, 2, compress=compress)
    try:
        before = _state(servers)
        sch, done = _run_cluster(cfg, corpus, servers)
        assert min(done.values()) >= 1
        # a worker may re-lease a finished path while the last one is in flight (async policy)
        assert sch.metrics.accepted_updates >= cfg.num_paths
        after = _state(servers)
        topo = cfg.build_topology()
        for k in topo.module_keys():
            changed = any(not torch.equal(before[k][n], after[k][n]) for n in before[k])
            assert changed, k
            v = next(ps._versions[k] for ps in servers if k in ps.bank)
            assert v[1] >= topo.sharing_count(k)   # >= one outer step per path through the key
            assert all(torch.isfinite(t).all() for t in after[k].values())
    finally:
        for ps in servers:
            ps.shutdown()


def test_checkpoint_and_resume(tmp_path):
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    servers = _servers(cfg, 2)
    try:
        sch, _ = _run_cluster(cfg, corpus, servers, ckpt=str(tmp_path))
        assert os.path.exists(tmp_path / "scheduler.pt")
        assert not os.path.exists(tmp_path / "manifest.json")  # static owners, no identity: no recovery floor
        sch._checkpoint_cluster(str(tmp_path))   # again, now that no push is in flight
        saved = _state(servers)
        versions = {k: v for ps in servers for k, v in ps._versions.items()}
    finally:
        for ps in servers:
            ps.shutdown()
    resumed = _servers(cfg, 2, resume_dir=str(tmp_path))
    try:
        for k, sd in _state(resumed).items():
            for n, t in sd.items():
                assert torch.equal(t, saved[k][n])
        assert {k: v for ps in resumed for k, v in ps._versions.items()} == versions
    finally:
        for ps in resumed:
            ps.shutdown()


# ------------------------------------------------------------------------ epochs
def _owner_rec(ident, port):
    return make_peer_record(ident, reachability="public", addr=("127.0.0.1", port), roles=["owner"])


def test_epoch_primary_only_writes_and_replication():
    cfg = tiny_config()
    sched_id = PeerIdentity.generate()
    ids = [PeerIdentity.generate() for _ in range(3)]
    keys = cfg.build_topology().module_keys()
    servers = [ParameterServer(cfg, keys, _diloco(), host="127.0.0.1", auth_key=KEY, identity=i,
                               scheduler_pub=sched_id.public_key_hex, replicate_interval=3600)
               for i in ids]
    for ps in servers:
        ps.start()
    try:
        recs = [_owner_rec(i, ps.port) for i, ps in zip(ids, servers)]
        epoch = make_epoch_record(sched_id, epoch=0, owner_records=recs, k=2, bootstrap=True)
        assert verify_epoch_record(epoch, signer_pub=sched_id.public_key_hex)
        for ps in servers:
            ps.apply_epoch(epoch)
        key = keys[0]
        owners = owners_for(key, epoch)
        by_id = {ps.peer_id: ps for ps in servers}
        primary, backup = by_id[owners[0]["peer_id"]], by_id[owners[1]["peer_id"]]
        grad = [torch.full(tuple(p.shape), 1e-3) for p in primary.bank[key].parameters()]
        g = make_grant((0, 0), [key], 1.0, "tok", identity=sched_id)
        ack = one_shot(("127.0.0.1", backup.port), {"type": "push", "grant": g, "updates": {key: {"grad": grad}},
                                                     "private": {}}, auth_key=KEY)
        assert ack["reason"] == "not_primary" and ack["skipped"] == [key]
        g = make_grant((0, 0), [key], 1.0, "tok2", identity=sched_id)
        ack = one_shot(("127.0.0.1", primary.port), {"type": "push", "grant": g, "updates": {key: {"grad": grad}},
                                                      "private": {}}, auth_key=KEY)
        assert ack["applied"] and primary._versions[key] == (0, 1)
        pulled = backup._replicate_once()
        assert pulled[key] == (0, 1)
        for a, b in zip(primary.bank[key].parameters(), backup.bank[key].parameters()):
            assert torch.equal(a, b)
        # momentum travelled too: one more identical step keeps them identical
        g = make_grant((0, 0), [key], 1.0, "tok3", identity=sched_id)
        one_shot(("127.0.0.1", primary.port), {"type": "push", "grant": g, "updates": {key: {"grad": grad}},
                                                "private": {}}, auth_key=KEY)
        backup._outer_opts[key].zero_grad()
        from opendipaco_b200.optim.diloco import apply_outer_grads
        apply_outer_grads(backup.bank[key], grad)
        backup._outer_opts[key].step()
        for a, b in zip(primary.bank[key].parameters(), backup.bank[key].parameters()):
            torch.testing.assert_close(a, b)
    finally:
        for ps in servers:
            ps.shutdown()


def test_derive_epoch_and_manager_hysteresis():
    ids = [PeerIdentity.generate() for _ in range(3)]
    recs = [_owner_rec(i, 9000 + n) for n, i in enumerate(ids)]
    e0 = derive_epoch(recs, k=2)
    assert e0["epoch"] == 0 and verify_epoch_record(e0, allow_deterministic=True)
    assert derive_epoch(recs, k=2, prev=e0) is e0
    e1 = derive_epoch(recs[:2], k=2, prev=e0)
    assert e1["epoch"] == 1
    placed = {k: owners_for(k, e0)[0]["peer_id"] for k in ("a", "b", "c", "d")}
    assert placed == {k: owners_for(k, dict(e0))[0]["peer_id"] for k in placed}

    m = EpochManager(owner_grace=10.0, min_epoch_interval=5.0)
    assert len(m.observe(recs, now=0.0)) == 3
    assert m.observe(recs, now=1.0) is None
    assert m.observe(recs[:2], now=8.0) is None          # still within grace
    assert m.observe(recs[:2], now=11.5) is not None     # unseen since t=1 + grace -> new epoch
    # a fresh tombstone evicts at once, a stale one does not
    m2 = EpochManager(owner_grace=100.0, min_epoch_interval=0.0)
    m2.observe(recs, now=0.0)
    stale = {recs[0]["peer_id"]: recs[0]["issued_at"] - 1}
    assert m2.observe(recs[1:], tombstoned=stale, now=1.0) is None
    fresh = {recs[0]["peer_id"]: recs[0]["issued_at"] + 1}
    out = m2.observe(recs[1:], tombstoned=fresh, now=2.0)
    assert [r["peer_id"] for r in out] == sorted(r["peer_id"] for r in recs[1:])


# ------------------------------------------------------------------------ tracker
def test_tracker_admission_directory_and_epoch_cache():
    a, b, intruder = PeerIdentity.generate(), PeerIdentity.generate(), PeerIdentity.generate()
    t = Tracker(host="127.0.0.1", enroll_peers=[a.public_key_hex, b.public_key_hex], ttl=60.0)
    t.start()
    addr = ("127.0.0.1", t.port)
    try:
        assert register_peer(addr, a, reachability="public", peer_addr=("127.0.0.1", 1), roles=["owner"])["type"] \
            == "registered"
        assert register_peer(addr, b, roles=["worker"])["type"] == "registered"
        assert register_peer(addr, intruder, roles=["worker"])["reason"] == "not enrolled"
        old = make_peer_record(a, reachability="public", addr=("127.0.0.1", 1), roles=["owner"])
        old["issued_at"] -= 100
        from opendipaco_b200.schedule.identity import sign_record
        old = sign_record(a, {k: v for k, v in old.items() if k not in ("pub", "sig", "peer_id")})
        assert one_shot(addr, {"type": "register", "record": old})["reason"] == "stale record"
        owners = fetch_directory(addr, roles=["owner"])
        assert [r["peer_id"] for r in owners] == [a.peer_id]
        assert deregister_peer(addr, b)["type"] == "deregistered"
        assert {r["peer_id"] for r in fetch_directory(addr)} == {a.peer_id}
        assert t.tombstones() == [b.peer_id]
        recs, n = fetch_directory_multi([addr, addr, ("127.0.0.1", t.port)])
        assert n == 1 and [r["peer_id"] for r in recs] == [a.peer_id]
        s1, s2 = PeerIdentity.generate(), PeerIdentity.generate()
        rec = make_peer_record(a, reachability="public", addr=("127.0.0.1", 1), roles=["owner"])
        e = make_epoch_record(s1, epoch=0, owner_records=[rec])
        assert put_epoch(addr, e)["type"] == "epoch_cached"
        assert put_epoch(addr, make_epoch_record(s2, epoch=5, owner_records=[rec]))["reason"] == "wrong signer"
        assert put_epoch(addr, e)["reason"] == "stale epoch"
        assert get_epoch(addr, signer_pub=s1.public_key_hex)["epoch"] == 0
        assert get_epoch(addr, signer_pub=s2.public_key_hex) is None
    finally:
        t.shutdown()


def test_grant_required_for_push_without_key_material():
    cfg = tiny_config()
    (ps,) = _servers(cfg, 1)
    try:
        key = "embed"
        grad = [torch.zeros(tuple(p.shape)) for p in ps.bank[key].parameters()]
        ack = one_shot(("127.0.0.1", ps.port), {"type": "push", "grant": {"token": "x", "path": [0, 0],
                                                                             "weight": 1.0, "keys": [key]},
                                                 "updates": {key: {"grad": grad}}, "private": {}}, auth_key=KEY)
        assert not ack["applied"]
        time.sleep(0)
    finally:
        ps.shutdown()
