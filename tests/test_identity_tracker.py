"""Peer identities and the tracker directory (CPU, loopback TCP): key files, challenge
signatures, self-certifying records, reachability rules, registration and filtering,
TTL expiry and signed deregistration, enrollment, tampered records, bootstrap import,
the directory cap, several trackers at once and the epoch cache.

Behaviours of the reference's ``tests/test_identity_tracker.py`` and
``src/opendipaco/schedule/tracker.py``.
"""

import os
import stat
import time

import pytest

from opendipaco_b200.schedule import PeerIdentity, Tracker, make_epoch_record, make_peer_record, sign_record
from opendipaco_b200.schedule.identity import peer_id_of, verify_auth, verify_record
from opendipaco_b200.schedule.tracker import (deregister_peer, fetch_directory, fetch_directory_and_tombstones,
                                              fetch_directory_multi, get_epoch, import_records, put_epoch,
                                              register_peer, tracker_rpc)


@pytest.fixture
def tracker():
    t = Tracker(host="127.0.0.1", port=0, open_enrollment=True, ttl=30.0)
    t.start()
    yield t
    t.shutdown()


def _addr(t):
    return ("127.0.0.1", t.port)


# ------------------------------------------------------------------ identities and records
def test_identity_key_file_round_trip_is_owner_only(tmp_path):
    ident = PeerIdentity.generate()
    path = tmp_path / "keys" / "peer.pem"
    path.parent.mkdir()
    path.write_text("old")
    os.chmod(path, 0o644)
    ident.save(path)  # an existing file is narrowed to the owner too
    assert stat.S_IMODE(os.stat(path).st_mode) == 0o600
    again = PeerIdentity.load(path)
    assert again.peer_id == ident.peer_id == peer_id_of(ident.public_key_hex)
    assert again.public_key_hex == ident.public_key_hex


def test_challenge_signature_binds_key_and_nonce():
    a, b = PeerIdentity.generate(), PeerIdentity.generate()
    nonce = os.urandom(32)
    r = a.auth_response(nonce)
    assert verify_auth(r["pub"], r["sig"], nonce)
    assert not verify_auth(b.public_key_hex, r["sig"], nonce)  # someone else's key
    assert not verify_auth(r["pub"], r["sig"], os.urandom(32))  # a replay on a fresh nonce
    assert not verify_auth(r["pub"], "zz", nonce) and not verify_auth(None, r["sig"], nonce)


def test_records_are_self_certifying():
    a, b = PeerIdentity.generate(), PeerIdentity.generate()
    rec = make_peer_record(a, reachability="public", addr=("10.0.0.1", 9000), roles=["owner", "worker"])
    assert verify_record(rec) and rec["roles"] == ["owner", "worker"]
    assert not verify_record(dict(rec, addr=["10.0.0.2", 9000]))       # moved without re-signing
    assert not verify_record(dict(rec, peer_id=b.peer_id))             # claims another id
    assert not verify_record(dict(rec, pub=b.public_key_hex))          # someone else's key
    assert not verify_record(sign_record(a, {"kind": "peer"}) | {"pub": "not hex"})
    assert not verify_record("record") and not verify_record({})


def test_reachability_rules():
    ident = PeerIdentity.generate()
    with pytest.raises(ValueError):
        make_peer_record(ident, reachability="public")                 # public needs an address
    with pytest.raises(ValueError):
        make_peer_record(ident, reachability="nat", addr=("h", 1))      # nat dials out only
    with pytest.raises(ValueError):
        make_peer_record(ident, reachability="relay")
    rec = make_peer_record(ident, reachability="nat", circuit_addrs=["/ip4/1.2.3.4/tcp/1/p2p-circuit"])
    assert verify_record(rec) and rec["addr"] is None and rec["circuit_addrs"]


# ------------------------------------------------------------------ tracker directory
def test_register_filter_and_refresh(tracker):
    owner, worker, natp = (PeerIdentity.generate() for _ in range(3))
    assert register_peer(_addr(tracker), owner, reachability="public", peer_addr=("127.0.0.1", 1),
                         roles=["owner"])["type"] == "registered"
    register_peer(_addr(tracker), worker, reachability="public", peer_addr=("127.0.0.1", 2), roles=["worker"])
    register_peer(_addr(tracker), natp, roles=["worker"])
    ids = lambda recs: {r["peer_id"] for r in recs}  # noqa: E731
    assert ids(fetch_directory(_addr(tracker))) == {owner.peer_id, worker.peer_id, natp.peer_id}
    assert ids(fetch_directory(_addr(tracker), roles=["owner"])) == {owner.peer_id}
    assert ids(fetch_directory(_addr(tracker), roles=["worker"], reachability="nat")) == {natp.peer_id}
    # a heartbeat replaces the record (newer issued_at); a replayed older one is refused
    old = make_peer_record(owner, reachability="public", addr=("127.0.0.1", 1), roles=["owner"])
    time.sleep(0.01)
    register_peer(_addr(tracker), owner, reachability="public", peer_addr=("127.0.0.1", 3), roles=["owner"])
    assert tracker_rpc(_addr(tracker), {"type": "register", "record": old})["reason"] == "stale record"
    (rec,) = fetch_directory(_addr(tracker), roles=["owner"])
    assert rec["addr"] == ["127.0.0.1", 3]


def test_ttl_expiry_and_signed_deregistration():
    t = Tracker(host="127.0.0.1", port=0, open_enrollment=True, ttl=0.3)
    t.start()
    try:
        a, b = PeerIdentity.generate(), PeerIdentity.generate()
        register_peer(_addr(t), a, roles=["worker"])
        register_peer(_addr(t), b, roles=["worker"])
        assert deregister_peer(_addr(t), b)["type"] == "deregistered"
        recs, tombs = fetch_directory_and_tombstones(_addr(t))
        assert [r["peer_id"] for r in recs] == [a.peer_id] and b.peer_id in tombs
        # only the key owner can deregister: a forged deregistration is refused
        forged = dict(sign_record(PeerIdentity.generate(), {"kind": "deregister", "issued_at": time.time()}),
                      peer_id=a.peer_id)
        assert tracker_rpc(_addr(t), {"type": "deregister", "record": forged})["type"] == "refused"
        time.sleep(0.45)  # nothing re-registered: the record and the tombstone lapse
        assert fetch_directory(_addr(t)) == [] and t.tombstones() == []
    finally:
        t.shutdown()


def test_enrollment_gate_and_expulsion():
    member, stranger = PeerIdentity.generate(), PeerIdentity.generate()
    t = Tracker(host="127.0.0.1", port=0, enroll_peers=[member])
    t.start()
    try:
        assert register_peer(_addr(t), member, roles=["worker"])["type"] == "registered"
        assert register_peer(_addr(t), stranger, roles=["worker"])["reason"] == "not enrolled"
        t.enroll(stranger.public_key_hex)
        assert register_peer(_addr(t), stranger, roles=["worker"])["type"] == "registered"
        t.expel(stranger)
        assert {r["peer_id"] for r in t.records()} == {member.peer_id}
        assert register_peer(_addr(t), stranger, roles=["worker"])["reason"] == "not enrolled"
    finally:
        t.shutdown()


def test_unsigned_tampered_and_malformed_records_are_refused(tracker):
    ident = PeerIdentity.generate()
    rec = make_peer_record(ident, reachability="public", addr=("127.0.0.1", 5), roles=["owner"])
    bad = [dict(rec, roles=["owner", "scheduler"]), {k: v for k, v in rec.items() if k != "sig"},
           sign_record(ident, {"kind": "epoch"}), sign_record(ident, {"kind": "peer", "reachability": "public",
                                                                      "addr": None, "issued_at": 1.0}),
           sign_record(ident, {"kind": "peer", "reachability": "nat", "addr": None})]
    for r in bad:
        assert tracker_rpc(_addr(tracker), {"type": "register", "record": r})["type"] == "refused"
    assert tracker.records() == []


def test_bootstrap_import_and_union_over_trackers(tracker):
    """A new tracker imports a peer's cached directory (records still verified), and a
    client reads the union of several trackers, newest record per peer."""
    peers = [PeerIdentity.generate() for _ in range(3)]
    recs = [make_peer_record(p, roles=["worker"]) for p in peers]
    tampered = dict(make_peer_record(PeerIdentity.generate(), roles=["worker"]), roles=["owner"])
    second = Tracker(host="127.0.0.1", port=0, open_enrollment=True)
    second.start()
    try:
        assert import_records(_addr(second), recs + [tampered])["accepted"] == 3
        register_peer(_addr(tracker), peers[0], roles=["worker", "owner"])  # newer on the first tracker
        union, answered = fetch_directory_multi([_addr(tracker), _addr(second), ("127.0.0.1", 1)])
        assert answered == 2 and {r["peer_id"] for r in union} == {p.peer_id for p in peers}
        newest = next(r for r in union if r["peer_id"] == peers[0].peer_id)
        assert newest["roles"] == ["owner", "worker"]
        # a quorum of 2 trackers keeps only the peer both of them serve
        both, _ = fetch_directory_multi([_addr(tracker), _addr(second)], seed_quorum=2)
        assert [r["peer_id"] for r in both] == [peers[0].peer_id]
    finally:
        second.shutdown()


def test_directory_cap_refuses_newcomers_but_not_heartbeats():
    t = Tracker(host="127.0.0.1", port=0, open_enrollment=True, max_peers=2)
    t.start()
    try:
        a, b, c = (PeerIdentity.generate() for _ in range(3))
        register_peer(_addr(t), a)
        register_peer(_addr(t), b)
        assert register_peer(_addr(t), c)["reason"] == "directory full"
        time.sleep(0.01)
        assert register_peer(_addr(t), a)["type"] == "registered"  # a heartbeat of a held peer
    finally:
        t.shutdown()


def test_tracker_behind_a_shared_secret():
    t = Tracker(host="127.0.0.1", port=0, open_enrollment=True, auth_key="enroll-token")
    t.start()
    try:
        ident = PeerIdentity.generate()
        assert register_peer(_addr(t), ident, auth_key="enroll-token")["type"] == "registered"
        with pytest.raises((PermissionError, ConnectionError, OSError)):
            fetch_directory(_addr(t), auth_key="wrong", timeout=2.0)
        assert len(fetch_directory(_addr(t), auth_key="enroll-token")) == 1
    finally:
        t.shutdown()


def test_epoch_cache_pins_its_signer_and_only_moves_forward(tracker):
    sched, rogue = PeerIdentity.generate(), PeerIdentity.generate()
    owners = [make_peer_record(PeerIdentity.generate(), reachability="public", addr=("127.0.0.1", 10 + i),
                               roles=["owner"]) for i in range(3)]
    e1 = make_epoch_record(sched, epoch=1, owner_records=owners, k=2)
    assert put_epoch(_addr(tracker), e1)["type"] == "epoch_cached"
    e2 = make_epoch_record(sched, epoch=2, owner_records=owners[:2], k=2)
    assert put_epoch(_addr(tracker), e2)["type"] == "epoch_cached"
    assert put_epoch(_addr(tracker), e1)["reason"] == "stale epoch"      # an older epoch never returns
    time.sleep(0.01)
    again = make_epoch_record(sched, epoch=2, owner_records=owners, k=2)  # a re-issue of the same epoch
    assert put_epoch(_addr(tracker), again)["type"] == "epoch_cached"
    assert put_epoch(_addr(tracker), make_epoch_record(rogue, epoch=5, owner_records=owners, k=2))["reason"] \
        == "wrong signer"
    got = get_epoch(_addr(tracker), signer_pub=sched.public_key_hex)
    assert got["epoch"] == 2 and len(got["owners"]) == 3
    assert get_epoch(_addr(tracker), signer_pub=rogue.public_key_hex) is None
