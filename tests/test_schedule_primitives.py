import socket
import threading
import time

import pytest
import torch

from opendipaco_b200.schedule import aggregate, assignment, guard, quorum, ratelimit, reputation, throttle, wire
from opendipaco_b200.schedule.identity import PeerIdentity, sign_record, verify_auth, verify_record


def test_robust_delta_modes():
    g = [(1.0, [torch.tensor([1.0, 10.0])]), (1.0, [torch.tensor([2.0, 20.0])]), (2.0, [torch.tensor([100.0, 30.0])])]
    d, w = aggregate.robust_delta(g, aggregate="trimmed_mean")
    assert w == 4.0 and torch.equal(d[0], torch.tensor([2.0, 20.0]))
    d, _ = aggregate.robust_delta(g, aggregate="median")
    assert torch.equal(d[0], torch.tensor([2.0, 20.0]))
    one, w1 = aggregate.robust_delta(g[:1])
    assert one[0] is g[0][1][0] and w1 == 1.0
    with pytest.raises(ValueError):
        aggregate.robust_delta(g, aggregate="max")


def test_guard():
    assert guard.contribution_ok(1.0, False, {"a": [torch.ones(2)]})
    assert not guard.contribution_ok(float("nan"), False)
    assert guard.contribution_ok(float("nan"), True)
    assert not guard.all_finite({"a": {"w": torch.tensor([1.0, float("inf")])}})
    t = [torch.tensor([3.0, 4.0])]
    assert guard.clip_norm_(t, 1.0) == pytest.approx(5.0) and float(t[0].norm()) == pytest.approx(1.0, rel=1e-5)


def test_reputation_and_rate_limit():
    r = reputation.Reputation()
    assert r.get("a") == 0.5
    r.debit("a")
    assert r.get("a") == pytest.approx(0.3) and not r.eligible("a", 0.4)
    r2 = reputation.Reputation()
    r2.restore(r.snapshot())
    assert r2.get("a") == pytest.approx(0.3, abs=1e-3)
    lim = ratelimit.RateLimiter(capacity=2, refill_per_sec=0.0)
    assert lim.allow("p", reputation=0.5) and lim.allow("p", reputation=0.5) and not lim.allow("p", reputation=0.5)


def test_assignment_and_quorum(reference_pkg):
    from opendipaco.schedule import assignment as RA

    workers = [f"w{i}" for i in range(5)]
    assert assignment.rank_workers((1, 2), 3, workers) == RA.rank_workers((1, 2), 3, workers)
    assert assignment.assignee((0,), 0, workers, elapsed=25, lease_ttl=10) == RA.assignee(
        (0,), 0, workers, elapsed=25, lease_ttl=10)
    assert assignment.version_lag({"a": (0, 1)}, {"a": (0, 4)}) == 3
    assert assignment.version_lag({"a": (0, 1)}, {"a": (1, 4)}) is None
    reps = [((0, 2), "x"), ((0, 2), "x"), ((0, 3), "y")]
    assert quorum.confirm_version(reps, 2) == ((0, 2), "x")
    assert quorum.divergent_peers({"p": ((0, 2), "z"), "q": ((0, 2), "x")}, ((0, 2), "x")) == {"p"}
    assert quorum.valid_report([[0, True], "d"]) is None


def test_identity_records(reference_pkg):
    from opendipaco.schedule import identity as RI

    me = PeerIdentity.generate()
    rec = sign_record(me, {"addr": "1.2.3.4:5", "ttl": 3})
    assert verify_record(rec) and RI.verify_record(rec)
    bad = dict(rec, addr="evil")
    assert not verify_record(bad)
    nonce = b"n" * 32
    r = me.auth_response(nonce)
    assert verify_auth(r["pub"], r["sig"], nonce) and not verify_auth(r["pub"], r["sig"], b"x" * 32)


def test_throttle_encoding_and_bucket():
    assert throttle.tailor_encoding(None) == ("none", 1.0)
    assert throttle.tailor_encoding(10) == ("int8", 1.0)
    assert throttle.tailor_encoding(1, base_density=0.8) == ("int4", 0.5)
    b = throttle.TokenBucket(1e6)
    t0 = time.monotonic()
    b.take(1_500_000)
    assert time.monotonic() - t0 > 0.3


def test_handshake_hmac_over_socket():
    a, b = socket.socketpair()
    out = {}
    th = threading.Thread(target=lambda: out.setdefault("srv", wire.server_handshake(a, ["k1", "k2"])))
    th.start()
    ok = wire.client_handshake(b, "k2")
    th.join()
    assert ok and out["srv"]
    a2, b2 = socket.socketpair()

    def refuse():
        out["srv2"] = wire.server_handshake(a2, "k1")
        a2.close()  # a server drops a connection that failed authentication

    th = threading.Thread(target=refuse)
    th.start()
    assert not wire.client_handshake(b2, "wrong")
    th.join()
    assert not out["srv2"]
