"""Launcher lifecycle (CPU): the shipped launch defaults keep the anti-thrash and
anti-false-eviction invariants while the library constructors keep their conservative
values; the bounded graceful shutdown hands off and cancels its deadline; only the
worker loops that can stop between tasks take over SIGINT / SIGTERM.

Behaviours of the reference's ``tests/test_w4d_launch.py``.
"""

import threading

from opendipaco_b200.launch import roles
from opendipaco_b200.launch.config import LaunchConfig, OwnershipCfg, ScheduleCfg, TrackerCfg, TransportCfg
from opendipaco_b200.schedule import EpochManager, Tracker

_TINY = {"model": {"vocab_size": 64, "hidden_size": 32, "num_attention_heads": 4, "intermediate_size": 64,
                   "max_position_embeddings": 64, "layers_per_level": [1, 1], "level_sizes": [2, 2],
                   "sequence_length": 16},
         "data": {"source": "synthetic", "num_documents": 16},
         "transport": {"host": "127.0.0.1", "port": 0},
         "sharded": {"num_shards": 2}}


def test_launch_defaults_keep_their_invariants():
    t, o, sch, tr = TrackerCfg(), OwnershipCfg(), ScheduleCfg(), TransportCfg()
    assert o.owner_grace >= 2 * t.ttl            # one missed heartbeat never evicts
    assert o.heartbeat_interval < t.ttl
    assert o.min_epoch_interval < o.owner_grace  # a flapping owner cannot thrash ownership
    assert t.ttl < 120.0 and o.owner_grace < 240.0 and tr.heartbeat_timeout < 30.0 and sch.lease_ttl < 30.0


def test_library_defaults_stay_conservative():
    tracker = Tracker(host="127.0.0.1")
    try:
        assert tracker.ttl == 120.0
    finally:
        tracker.shutdown()
    m = EpochManager()
    assert m.owner_grace == 240.0 and m.min_epoch_interval == 60.0


def test_bounded_graceful_shutdown_hands_off_and_cancels_its_deadline():
    seen = {}

    class _Server:
        def shutdown(self, *, graceful=False):
            seen["graceful"] = graceful

    roles._graceful_shutdown(_Server(), deadline=300.0)  # an uncancelled deadline would end this process
    assert seen == {"graceful": True}
    timers = [t for t in threading.enumerate() if isinstance(t, threading.Timer)]
    for t in timers:
        t.join(timeout=2.0)  # a cancelled timer's thread exits at once
    assert not any(t.is_alive() for t in timers)


def test_only_stoppable_worker_loops_take_over_the_signals(monkeypatch):
    installed, got = [], {}
    monkeypatch.setattr(roles, "_signal_event", lambda: installed.append(1) or threading.Event())
    monkeypatch.setattr(roles, "run_worker", lambda *a, **k: got.setdefault("coordinator", k.get("stop_event")))
    monkeypatch.setattr(roles, "run_sharded_worker", lambda *a, **k: got.setdefault("sharded", k.get("stop_event")))
    roles.run_worker_role(LaunchConfig.from_dict({**_TINY, "mode": "coordinator"}))
    assert installed == []
    roles.run_worker_role(LaunchConfig.from_dict({**_TINY, "mode": "sharded"}))
    assert installed == [1] and isinstance(got["sharded"], threading.Event)
    mine = threading.Event()
    roles.run_worker_role(LaunchConfig.from_dict({**_TINY, "mode": "sharded"}), stop_event=mine)
    assert installed == [1]  # a caller's own stop event is used as is
