"""Eclipse resistance of the peer directory (CPU, loopback trackers): a client reads
the union of several seed trackers, keeps each peer's freshest signed record, honours
signed tombstones, can demand that a record be served by a quorum of seeds, and an
owner heartbeats to every seed so one bad seed cannot hide it.

Behaviours of the reference's ``tests/test_eclipse.py``
(``src/opendipaco/schedule/tracker.py`` multi-seed reads).
"""

import time

import pytest

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import ParameterServer, PeerIdentity, Tracker, make_peer_record
from opendipaco_b200.schedule.tracker import (dedup_seeds, deregister_peer, fetch_directory, fetch_directory_multi,
                                              import_records, register_peer)

from helpers import tiny_config


@pytest.fixture
def seeds():
    ts = [Tracker(host="127.0.0.1", port=0, open_enrollment=True, ttl=30.0) for _ in range(3)]
    for t in ts:
        t.start()
    yield ts
    for t in ts:
        t.shutdown()


def _a(t):
    return ("127.0.0.1", t.port)


def _ids(recs):
    return {r["peer_id"] for r in recs}


def test_union_recovers_peers_a_seed_omits(seeds):
    a, b, c = (PeerIdentity.generate() for _ in range(3))
    register_peer(_a(seeds[0]), a)
    register_peer(_a(seeds[1]), b)          # an eclipsing seed 0 never shows b
    register_peer(_a(seeds[2]), c)
    union, answered = fetch_directory_multi([_a(t) for t in seeds])
    assert answered == 3 and _ids(union) == {a.peer_id, b.peer_id, c.peer_id}


def test_union_keeps_the_freshest_record_per_peer(seeds):
    p = PeerIdentity.generate()
    old = make_peer_record(p, reachability="public", addr=("10.0.0.1", 1), roles=["owner"])
    time.sleep(0.01)
    new = make_peer_record(p, reachability="public", addr=("10.0.0.2", 2), roles=["owner"])
    import_records(_a(seeds[0]), [old])     # a seed replaying a stale record
    import_records(_a(seeds[1]), [new])
    (rec,), _ = fetch_directory_multi([_a(seeds[0]), _a(seeds[1])])
    assert rec["addr"] == ["10.0.0.2", 2]


def test_tombstone_suppresses_a_replayed_record(seeds):
    p = PeerIdentity.generate()
    stale = make_peer_record(p, roles=["worker"])
    import_records(_a(seeds[0]), [stale])   # seed 0 still serves the old record
    time.sleep(0.01)
    register_peer(_a(seeds[1]), p, roles=["worker"])
    deregister_peer(_a(seeds[1]), p)        # the peer left: seed 1 holds its signed tombstone
    union, _ = fetch_directory_multi([_a(seeds[0]), _a(seeds[1])])
    assert p.peer_id not in _ids(union)
    # a record issued after the tombstone (the peer came back) is served again
    time.sleep(0.01)
    register_peer(_a(seeds[0]), p, roles=["worker"])
    union, _ = fetch_directory_multi([_a(seeds[0]), _a(seeds[1])])
    assert p.peer_id in _ids(union)


def test_unreachable_seeds_and_a_single_seed():
    dead = [("127.0.0.1", 1), ("127.0.0.1", 2)]
    assert fetch_directory_multi(dead, timeout=0.5) == ([], 0)
    t = Tracker(host="127.0.0.1", port=0, open_enrollment=True)
    t.start()
    try:
        for _ in range(3):
            register_peer(_a(t), PeerIdentity.generate(), roles=["worker"])
        union, n = fetch_directory_multi([_a(t)] + dead, timeout=0.5)
        assert n == 1 and _ids(union) == _ids(fetch_directory(_a(t)))
    finally:
        t.shutdown()


def test_seed_quorum_drops_records_too_few_seeds_serve(seeds):
    known, planted = PeerIdentity.generate(), PeerIdentity.generate()
    for t in seeds:
        register_peer(_a(t), known)
    register_peer(_a(seeds[0]), planted)    # only one (possibly malicious) seed knows this one
    addrs = [_a(t) for t in seeds]
    assert _ids(fetch_directory_multi(addrs, seed_quorum=2)[0]) == {known.peer_id}
    # the trade-off: an honest newcomer that has reached one seed so far is dropped too
    newcomer = PeerIdentity.generate()
    register_peer(_a(seeds[2]), newcomer)
    assert newcomer.peer_id not in _ids(fetch_directory_multi(addrs, seed_quorum=2)[0])
    assert newcomer.peer_id in _ids(fetch_directory_multi(addrs, seed_quorum=1)[0])


def test_dedup_seeds_and_aliases_count_once(seeds):
    primary = ("127.0.0.1", str(seeds[0].port))
    out = dedup_seeds(primary, [("127.0.0.1", seeds[0].port), ("127.0.0.1", seeds[1].port), _a(seeds[1])])
    assert out == [_a(seeds[0]), _a(seeds[1])]
    p = PeerIdentity.generate()
    register_peer(_a(seeds[0]), p)
    # the same seed listed twice (once with a string port) cannot make up a quorum of two
    union, n = fetch_directory_multi([_a(seeds[0]), ("127.0.0.1", str(seeds[0].port))], seed_quorum=2)
    assert n == 1 and union == []


def test_owner_heartbeats_to_every_seed_despite_a_bad_one(seeds):
    cfg = tiny_config()
    ident = PeerIdentity.generate()
    ps = ParameterServer(cfg, [], DiLoCoConfig(inner_steps=2), host="127.0.0.1", identity=ident)
    ps.start()
    try:
        ps.start_tracker_heartbeat(_a(seeds[0]), "127.0.0.1", interval=0.2,
                                   seeds=[("127.0.0.1", 1), _a(seeds[1]), _a(seeds[2])])
        deadline = time.monotonic() + 10
        while time.monotonic() < deadline and not all(ident.peer_id in _ids(t.records()) for t in seeds):
            time.sleep(0.05)
        assert all(ident.peer_id in _ids(t.records()) for t in seeds)
    finally:
        ps.shutdown()
