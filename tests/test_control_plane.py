"""Sharded-scheduler policies driven message by message (no sockets for the scheduler):
task sizing to a time window (W5), parking of too-slow workers, redundant-execution
audits resolved by digest majority or deadline, and a gracefully leaving primary owner
draining its keys to the backup (loopback TCP).

Reference behaviour: ``src/opendipaco/schedule/sharded.py`` (task sizing, audits,
drain) and its ``tests/test_task_sizing*.py``, ``tests/test_audit*.py``,
``tests/test_drain.py``, ``tests/test_graceful_leave.py``.
"""

import time

import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import (ParameterServer, PeerIdentity, Reputation, Scheduler, make_epoch_record,
                                      make_grant, make_peer_record, owners_for)
from opendipaco_b200.schedule.rpc import one_shot

from helpers import rr_corpus, tiny_config


def _sched(levels=(2, 2), **kw):
    cfg = tiny_config(levels=levels)
    s = Scheduler(cfg, rr_corpus(cfg), ["127.0.0.1:1"], DiLoCoConfig(inner_steps=10, inner_lr=1e-3), 8,
                  host="127.0.0.1", **kw)
    with s._lock:  # what fit() sets up, without its serving loop
        s._completed = {p: 0 for p in s.topology.paths()}
        s._target = 10 ** 6
        s._serving = True
    return s


def _req(s, wid, peer=None, **caps):
    return s._handle({"type": "request", "worker_id": wid, **({"capabilities": caps} if caps else {})}, 0, peer)


def _commit(s, task, wid, peer=None, **extra):
    msg = {"type": "commit", "path": list(task["path"]), "lease": task["lease"], "gen_id": task["gen_id"],
           "worker_id": wid, "loss": 1.0, **extra}
    return s._handle(msg, 0, peer)


# ------------------------------------------------------------------ task sizing (W5)
def test_task_is_sized_to_the_time_window():
    s = _sched(task_seconds=1.0)
    seq = s.config.sequence_length
    t = _req(s, "w")  # no rate yet: the full batch and the configured inner steps
    assert t["batch_size"] == 8 and t["inner_steps"] == 10
    s._record_rate("w", 20 * seq, 1.0)  # 20 sequences a second -> 2 per step over 10 steps
    t = _req(s, "w")
    assert (t["batch_size"], t["inner_steps"]) == (2, 10)
    s._worker_rate["w"] = 5 * seq  # 5 sequences a second: one per step, 5 steps
    t = _req(s, "w")
    assert (t["batch_size"], t["inner_steps"]) == (1, 5)
    s._worker_rate["w"] = 1000 * seq  # fast: capped by the worker's own max_batch
    t = _req(s, "w", max_batch=3)
    assert t["batch_size"] == 3 and t["inner_steps"] == 10


def test_rate_is_an_exponential_moving_average_of_committed_work():
    s = _sched()
    t = _req(s, "w")
    s._lease_at[tuple(t["path"])] -= 2.0  # the task took about two seconds
    assert _commit(s, t, "w")["accepted"]
    r1 = s.worker_rate("w")
    work = 8 * 10 * s.config.sequence_length
    assert abs(r1 - work / 2.0) / (work / 2.0) < 0.05
    s._record_rate("w", work, 1.0)
    assert abs(s.worker_rate("w") - (0.7 * r1 + 0.3 * work)) < 1e-6


def test_too_slow_worker_is_parked_between_tasks():
    s = _sched(min_task_rate=100.0, park_factor=3.0)
    s._worker_rate["slow"] = 10.0
    assert _req(s, "slow")["type"] == "task"  # one task, then parked
    assert _req(s, "slow")["type"] == "idle"
    s._parked["slow"] -= 10 ** 6  # the parking window has passed
    assert _req(s, "slow")["type"] == "task"
    s._worker_rate["fast"] = 1e9
    assert _req(s, "fast")["type"] == "task" and _req(s, "fast")["type"] == "task"


# ------------------------------------------------------------------ audits
def _audited_round(s, digests):
    """A primary and len(digests) checkers on the audit of path p0, generation 0."""
    a = _req(s, "A", "A")
    assert a.get("audit")
    others = [_req(s, w, w) for w in ("B", "C", "D")]  # every other path is now in flight
    assert all(o["type"] == "task" for o in others)
    assert _commit(s, a, "A", "A", digest="good", base=[1, 2])["accepted"]
    again = _req(s, "E", "E")  # path p0 is eligible again: a normal task (its own audit)
    assert again["type"] == "task" and tuple(again["path"]) == tuple(a["path"])
    checks = []
    for i, d in enumerate(digests):
        w = f"X{i}"
        t = _req(s, w, w)
        assert t.get("check_only") and t["base"] == [1, 2] and tuple(t["path"]) == tuple(a["path"])
        checks.append((w, t, d))
    for w, t, d in checks:
        assert s._handle({"type": "commit", "check_only": True, "path": list(t["path"]), "gen_id": t["gen_id"],
                          "lease": t["lease"], "worker_id": w, "digest": d}, 0, w)["check"]
    return s, (tuple(a["path"]), a["gen_id"])


def test_audit_majority_credits_agreeing_peers_and_debits_the_odd_one():
    rep = Reputation(decay_halflife=0)
    s, key = _audited_round(_sched(redundancy=3, redundancy_rate=1.0, reputation=rep), ["good", "bad"])
    f = rep.floor
    assert rep.get("X0") > f and rep.get("X1") < f
    assert rep.get("A") > f + rep.credit_step  # credited for its commit and for the audit
    assert s.metrics.invalid_rejected == 1
    assert key not in s._audits  # settled once both checks arrived


def test_unresolved_audit_is_settled_at_its_deadline():
    rep = Reputation(decay_halflife=0)
    s = _sched(redundancy=3, redundancy_rate=1.0, reputation=rep, audit_timeout=0.2)
    s, key = _audited_round(s, ["good"])  # one of the two checks never arrives
    assert s._audits[key]["checks"] == [("X0", "good")]
    time.sleep(0.3)
    with s._lock:
        s._reclaim_locked()
    assert key not in s._audits
    assert rep.get("X0") > rep.floor


# ------------------------------------------------------------------ graceful leave / drain
def test_graceful_primary_drains_to_the_backup():
    cfg = tiny_config()
    sched_id = PeerIdentity.generate()
    ids = [PeerIdentity.generate() for _ in range(2)]
    keys = cfg.build_topology().module_keys()
    servers = [ParameterServer(cfg, keys, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), host="127.0.0.1",
                               auth_key="k", identity=i, scheduler_pub=sched_id.public_key_hex,
                               replicate_interval=3600) for i in ids]
    for ps in servers:
        ps.start()
    try:
        recs = [make_peer_record(i, reachability="public", addr=("127.0.0.1", ps.port), roles=["owner"])
                for i, ps in zip(ids, servers)]
        epoch = make_epoch_record(sched_id, epoch=0, owner_records=recs, k=2, bootstrap=True)
        for ps in servers:
            ps.apply_epoch(epoch)
        by_id = {ps.peer_id: ps for ps in servers}
        key = keys[0]
        owners = owners_for(key, epoch)
        primary, backup = by_id[owners[0]["peer_id"]], by_id[owners[1]["peer_id"]]
        grad = [torch.full(tuple(p.shape), 1e-3) for p in primary.bank[key].parameters()]
        g = make_grant((0, 0), [key], 1.0, "t1", identity=sched_id)
        ack = one_shot(("127.0.0.1", primary.port), {"type": "push", "grant": g, "updates": {key: {"grad": grad}},
                                                      "private": {}}, auth_key="k")
        assert ack["applied"] and primary._versions[key] == (0, 1) and backup._versions[key] == (0, 0)
        primary.shutdown(graceful=True)  # leaves: pushes its newest state to each key's backup
        assert backup._versions[key] == (0, 1)
        for a, b in zip(primary.bank[key].parameters(), backup.bank[key].parameters()):
            assert torch.equal(a, b)
        # momentum travelled too: the backup's next step equals the primary's would-be step
        ps0 = backup._outer_opts[key].state_dict()["state"]
        assert ps0 and all("momentum_buffer" in v for v in ps0.values())
        assert primary._draining and not primary._primary(key)
    finally:
        for ps in servers:
            ps.shutdown()


def test_drain_ignores_older_versions():
    cfg = tiny_config()
    keys = cfg.build_topology().module_keys()
    ps = ParameterServer(cfg, keys, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), host="127.0.0.1", auth_key="k")
    key = keys[0]
    sd = {n: t.clone() + 1 for n, t in ps.bank[key].state_dict().items()}
    ps._versions[key] = (0, 3)
    reply = ps._drain_recv({"states": {key: {"version": [0, 2], "weights": sd, "state": None}}})
    assert reply["adopted"] == []
    reply = ps._drain_recv({"states": {key: {"version": [0, 4], "weights": sd, "state": None}}})
    assert reply["adopted"] == [key] and ps._versions[key] == (0, 4)
    assert all(torch.equal(a, sd[n]) for n, a in ps.bank[key].state_dict().items())


def test_rate_guards_empty_commits_and_reclaimed_leases():
    s = _sched()
    for bad in ((None, 100, 1.0), ("w", 0, 1.0), ("w", 100, 0.0), ("w", -5, 1.0)):
        s._record_rate(*bad)
    assert s.worker_rate("w") is None
    t = _req(s, "w")
    s._lease_at[tuple(t["path"])] -= 1.0
    assert _commit(s, t, "w", empty=True, loss=None)["accepted"]  # an empty shard trains nothing
    assert s.worker_rate("w") is None
    s2 = _sched(heartbeat_timeout=0.01)
    t = _req(s2, "z")
    time.sleep(0.05)
    with s2._lock:
        s2._reclaim_locked()              # the lease ran out: the late commit is refused, no rate
    assert not _commit(s2, t, "z")["accepted"] and s2.worker_rate("z") is None
