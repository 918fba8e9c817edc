"""Failure detection and recovery on the host (CPU, loopback TCP, gloo ranks):

* a coordinator that crashes (every socket dropped, as a killed process) is restarted
  in place from its cluster checkpoint; the worker reconnects and the run completes;
* a restarted sharded scheduler with a signed recovery manifest serves no task until a
  live owner holds the manifest's version of every key; a planted manifest is ignored;
* an owner whose tracker heartbeat is paused (a suspended machine) drops out of the
  directory after the TTL and reappears when it resumes;
* a rank that leaves between synchronous rounds makes the other rank's next collective
  fail within the process-group timeout instead of hanging.
"""

import os
import subprocess
import sys
import threading
import time

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig, DiPaCoEngine, LocalBackend
from opendipaco_b200.schedule import (AsyncScheduler, CoordinatorServer, ParameterServer, PeerIdentity, Scheduler,
                                      Tracker, fetch_directory, make_peer_record, run_worker, sign_record)
from opendipaco_b200.schedule.rpc import one_shot

from helpers import rr_corpus, tiny_config

HERE = os.path.dirname(os.path.abspath(__file__))
KEY = "k"


def _coordinator(cfg, corpus, port=0):
    eng = DiPaCoEngine(cfg, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), LocalBackend(cfg.build_topology()),
                       materialize="serial", seed=0)
    srv = CoordinatorServer(AsyncScheduler(eng), corpus, 2, host="127.0.0.1", port=port, auth_key=KEY,
                            heartbeat_timeout=5.0)
    srv.start()
    return srv


def test_coordinator_crash_restart_in_place_and_worker_reconnect(tmp_path):
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    first = _coordinator(cfg, corpus)
    port, ckpt = first.port, str(tmp_path / "ck")
    out = {}
    fit1 = threading.Thread(target=lambda: out.setdefault(
        "a", first.fit(6, checkpoint_dir=ckpt, checkpoint_every=2)))
    fit1.start()
    worker = threading.Thread(target=run_worker, args=(cfg, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), "127.0.0.1",
                                                       port),
                              kwargs=dict(auth_key=KEY, reconnect=True, reconnect_timeout=60.0,
                                          poll_interval=0.01))
    worker.start()
    deadline = time.time() + 120
    while first._T < 4 and time.time() < deadline:
        time.sleep(0.02)
    assert first._T >= 4
    first.simulate_crash()
    fit1.join(timeout=30)
    assert not fit1.is_alive()
    second = _coordinator(cfg, corpus, port=port)  # restarted in place
    try:
        done = second.fit(6, checkpoint_dir=ckpt, checkpoint_every=2, resume=True)
        assert second._T >= 4 + 6 * cfg.num_paths - cfg.num_paths  # resumed from the checkpoint, then served
        assert min(done.values()) >= 1
        assert second.metrics.accepted_updates > 0
    finally:
        second.shutdown()
        worker.join(timeout=60)
    assert not worker.is_alive()


def _owner(cfg, keys, ident, sched_pub):
    ps = ParameterServer(cfg, keys, DiLoCoConfig(inner_steps=2), host="127.0.0.1", auth_key=KEY, identity=ident,
                         scheduler_pub=sched_pub, replicate_interval=3600)
    ps.start()
    return ps


def test_recovery_manifest_gates_serving_until_owners_catch_up(tmp_path):
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    keys = cfg.build_topology().module_keys()
    sid = PeerIdentity.generate()
    ids = [PeerIdentity.generate() for _ in range(2)]
    owners = [_owner(cfg, keys, i, sid.public_key_hex) for i in ids]
    recs = [make_peer_record(i, reachability="public", addr=("127.0.0.1", ps.port), roles=["owner"])
            for i, ps in zip(ids, owners)]
    try:
        before = Scheduler(cfg, corpus, [], DiLoCoConfig(inner_steps=2), 2, host="127.0.0.1", auth_key=KEY,
                           identity=sid)
        before.publish_epoch(recs, k=2)
        for ps in owners:  # the owners have reached version (0, 5) of every key when the checkpoint is taken
            ps._versions = {k: (0, 5) for k in ps._versions}
        before._checkpoint_cluster(str(tmp_path))
        before.shutdown()
        assert (tmp_path / "manifest.json").exists()
        for ps in owners:  # ... and come back older after the restart
            ps._versions = {k: (0, 2) for k in ps._versions}
        after = Scheduler(cfg, corpus, [], DiLoCoConfig(inner_steps=2), 2, host="127.0.0.1", auth_key=KEY,
                          identity=sid)
        after.start()
        t = threading.Thread(target=lambda: after.fit(1, checkpoint_dir=str(tmp_path), resume=True,
                                                      recovery_poll=0.05), daemon=True)
        t.start()
        time.sleep(0.3)
        assert not after._serving and after._recovery is not None  # no owner set known yet
        after.publish_epoch(recs, k=2)
        assert after._epoch_record["epoch"] >= 1  # numbered after the checkpoint's epoch
        time.sleep(0.3)
        assert not after._serving  # the owners are below the recovery floor
        reply = one_shot(("127.0.0.1", after.port), {"type": "request", "worker_id": "w"}, auth_key=KEY)
        assert reply["type"] in ("idle", "stop")  # nothing served below the recovery floor
        owners[1]._versions = {k: (0, 5) for k in owners[1]._versions}  # one owner catches up
        deadline = time.time() + 10
        while not after._serving and time.time() < deadline:
            time.sleep(0.02)
        assert after._serving
        after.shutdown()
        t.join(timeout=10)
        # a manifest signed by someone else does not set a floor
        planted = sign_record(PeerIdentity.generate(), {"kind": "manifest", "epoch": 0, "keys": {keys[0]: [9, 9]},
                                                       "issued_at": 0.0})
        import json

        (tmp_path / "manifest.json").write_text(json.dumps(planted))
        third = Scheduler(cfg, corpus, [], DiLoCoConfig(inner_steps=2), 2, host="127.0.0.1", auth_key=KEY,
                          identity=sid)
        third._load_state(str(tmp_path))
        assert third._recovery is None
        third.shutdown()
    finally:
        for ps in owners:
            ps.shutdown()


def test_paused_heartbeat_lapses_from_the_tracker_and_resumes():
    cfg = tiny_config()
    keys = cfg.build_topology().module_keys()
    tracker = Tracker(host="127.0.0.1", ttl=0.6, open_enrollment=True)
    tracker.start()
    ident = PeerIdentity.generate()
    ps = _owner(cfg, keys, ident, PeerIdentity.generate().public_key_hex)
    try:
        ps.start_tracker_heartbeat(("127.0.0.1", tracker.port), "127.0.0.1", interval=0.1)

        def listed():
            return any(r["peer_id"] == ident.peer_id for r in fetch_directory(("127.0.0.1", tracker.port),
                                                                               roles=["owner"]))

        deadline = time.time() + 10
        while not listed() and time.time() < deadline:
            time.sleep(0.05)
        assert listed()
        ps.pause_heartbeat()
        time.sleep(1.5)  # > TTL: the record lapses, the server itself is still up
        assert not listed()
        assert one_shot(("127.0.0.1", ps.port), {"type": "status"}, auth_key=KEY)["type"] == "status"
        ps.resume_heartbeat()
        deadline = time.time() + 10
        while not listed() and time.time() < deadline:
            time.sleep(0.05)
        assert listed()
    finally:
        ps.shutdown()
        tracker.shutdown()


def test_rank_leaving_between_rounds_is_detected(tmp_path):
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29641", os.path.join(HERE, "mp_leave.py"),
           str(tmp_path)]
    subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ, OMP_NUM_THREADS="1"))
    outcome = torch.load(tmp_path / "leave_rank0.pt", weights_only=False)
    assert outcome["detected"], outcome
    assert outcome["seconds"] < 60, outcome
