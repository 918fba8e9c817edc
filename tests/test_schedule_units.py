"""Unit behaviour of the control-plane building blocks (CPU): rendezvous placement and
epochs, leaderless assignment, quorum reads, guards, probes, bandwidth tailoring, token
buckets and reputation-scaled rate limits.

Mirrors the reference's ``tests/test_ownership.py``, ``test_assignment.py``,
``test_quorum.py``, ``test_update_guard.py``, ``test_probe.py``, ``test_tailor.py``,
``test_throttle.py`` and ``test_reputation.py`` coverage.
"""

import math
import time

import pytest
import torch

from opendipaco_b200.schedule import (EpochManager, PeerIdentity, RateLimiter, Reputation, assignee,
                                      confirm_version, coordinator_key, derive_epoch, divergent_peers, is_assignee,
                                      make_epoch_record, make_peer_record, owner_eligible, owners_for,
                                      rank_owners, rank_workers, read_quorum_versions, responsible_rank,
                                      verify_epoch_record, version_lag)
from opendipaco_b200.schedule.guard import all_finite, clip_norm_, contribution_ok, loss_ok
from opendipaco_b200.schedule.probe import TrustedProbe, as_finite_float, is_harmful
from opendipaco_b200.schedule.throttle import TokenBucket, rate_from_mbps, tailor_encoding


def _owners(n, start=0):
    ids = [PeerIdentity.generate() for _ in range(n)]
    return ids, [make_peer_record(i, reachability="public", addr=("10.0.0.%d" % (start + j), 9000 + j),
                                  roles=["owner"]) for j, i in enumerate(ids)]


# ------------------------------------------------------------------ placement and epochs
def test_hrw_moves_only_the_departed_owners_keys():
    _, recs = _owners(6)
    keys = [f"L{i}E{j}" for i in range(4) for j in range(8)]
    before = {k: rank_owners(k, recs)[0]["peer_id"] for k in keys}
    gone = recs[2]["peer_id"]
    after = {k: rank_owners(k, [r for r in recs if r["peer_id"] != gone])[0]["peer_id"] for k in keys}
    for k in keys:
        if before[k] != gone:
            assert after[k] == before[k]
        else:
            assert after[k] != gone
    # a different salt is a different (but again deterministic) placement
    salted = {k: rank_owners(k, recs, salt="s")[0]["peer_id"] for k in keys}
    assert salted != before and salted == {k: rank_owners(k, recs, salt="s")[0]["peer_id"] for k in keys}


def test_epoch_record_signature_pins_the_signer_and_the_content():
    sched, other = PeerIdentity.generate(), PeerIdentity.generate()
    _, recs = _owners(4)
    rec = make_epoch_record(sched, epoch=3, owner_records=recs, k=2)
    assert verify_epoch_record(rec, signer_pub=sched.public_key_hex)
    assert not verify_epoch_record(rec, signer_pub=other.public_key_hex)
    tampered = dict(rec, k=3)
    assert not verify_epoch_record(tampered)
    assert [o["peer_id"] for o in owners_for("embed", rec)] == \
        [o["peer_id"] for o in rank_owners("embed", rec["owners"])[:2]]
    with pytest.raises(ValueError):
        make_epoch_record(sched, epoch=0, owner_records=[dict(recs[0], roles=["worker"])])


def test_owner_eligibility_needs_an_owner_role_and_a_dialable_address():
    ident = PeerIdentity.generate()
    assert owner_eligible(make_peer_record(ident, reachability="public", addr=("h", 1), roles=["owner"]))
    assert not owner_eligible(make_peer_record(ident, reachability="public", addr=("h", 1), roles=["worker"]))
    assert not owner_eligible({"kind": "peer", "peer_id": "x", "roles": ["owner"], "reachability": "nat"})


def test_derived_epoch_bumps_only_on_membership_change():
    _, recs = _owners(3)
    e0 = derive_epoch(recs, k=2)
    assert e0["epoch"] == 0 and e0["deterministic"] and not e0["bootstrap"]
    assert derive_epoch(list(reversed(recs)), k=2, prev=e0) is e0
    e1 = derive_epoch(recs[:2], k=2, prev=e0)
    assert e1["epoch"] == 1
    assert verify_epoch_record(e1, allow_deterministic=True) and not verify_epoch_record(e1)


def test_epoch_manager_grace_tombstones_and_rate_limit():
    _, recs = _owners(3)
    m = EpochManager(owner_grace=10.0, min_epoch_interval=5.0)
    assert [r["peer_id"] for r in m.observe(recs, now=0.0)] == sorted(r["peer_id"] for r in recs)
    assert m.observe(recs, now=1.0) is None                # unchanged
    assert m.observe(recs[:2], now=2.0) is None            # unseen for less than the grace
    assert m.observe(recs[:2], now=11.0) is not None       # now gone (and past the rate limit)
    # a fresh signed tombstone evicts at once, but the rate limit still applies
    gone = recs[0]["peer_id"]
    tomb = {gone: recs[0]["issued_at"] + 1}
    assert m.observe(recs[:2], tombstoned=tomb, now=12.0) is None
    nxt = m.observe(recs[:2], tombstoned=tomb, now=17.0)
    assert nxt is not None and gone not in [r["peer_id"] for r in nxt]
    # a replayed old tombstone does not evict a peer that registered again
    m2 = EpochManager(owner_grace=10.0, min_epoch_interval=0.0)
    m2.observe(recs, now=0.0)
    assert m2.observe(recs, tombstoned={gone: recs[0]["issued_at"] - 1}, now=1.0) is None


# ------------------------------------------------------------------ leaderless assignment
def test_assignment_is_deterministic_and_fails_over_by_lease():
    workers = [f"w{i}" for i in range(5)]
    path = (1, 2)
    ranked = rank_workers(path, 7, workers)
    assert sorted(ranked) == sorted(workers) and ranked == rank_workers(path, 7, list(reversed(workers)))
    assert rank_workers(path, 8, workers) != ranked or rank_workers((2, 1), 7, workers) != ranked
    assert assignee(path, 7, workers) == ranked[0]
    assert assignee(path, 7, workers, elapsed=25.0, lease_ttl=10.0) == ranked[2]
    assert responsible_rank(1e9, 10.0, 5) == 4 and responsible_rank(5.0, 0.0, 5) == 0
    assert is_assignee(ranked[0], path, 7, workers) and not is_assignee(None, path, 7, workers)


def test_version_lag_and_coordinator_key():
    assert version_lag({}, {"a": (0, 5)}) == 0
    assert version_lag({"a": (1, 3), "b": (1, 1)}, {"a": (1, 5), "b": (1, 4)}) == 3
    assert version_lag({"a": (1, 3)}, {"a": (2, 5)}) is None      # different epoch
    assert version_lag({"a": (1, 6)}, {"a": (1, 5)}) is None      # from the future
    assert version_lag({"z": (1, 1)}, {"a": (1, 1)}) is None      # unknown key
    assert coordinator_key(["L1E0", "embed", "head.p3", "L0E1"]) == "head.p3"
    assert coordinator_key(["L1E0", "embed", "L0E1"]) == "L0E1"


# ------------------------------------------------------------------ quorum reads
def test_quorum_confirms_the_newest_version_with_enough_agreeing_digests():
    reps = [((1, 4), "aa"), ((1, 4), "aa"), ((1, 5), "bb"), ((1, 4), "xx")]
    assert confirm_version(reps, 2) == ((1, 4), "aa")
    assert confirm_version(reps, 1) == ((1, 5), "bb")
    assert confirm_version(reps, 3) is None
    by_peer = {"p": ((1, 4), "aa"), "q": ((1, 4), "xx"), "r": ((1, 5), "bb"), "s": None}
    assert divergent_peers(by_peer, ((1, 4), "aa")) == {"q"}
    assert divergent_peers(by_peer, None) == set()


def test_quorum_read_skips_unreachable_and_malformed_replies():
    replies = {
        "a": {"digests": {"k": [[1, 2], "d1"], "j": [[1, 1], "e"]}},
        "b": {"digests": {"k": [[1, 2], "d1"], "j": ["bad"]}},
        "c": OSError("down"),
        "d": {"digests": {"k": [[1, True], "d1"]}},  # bool is not a counter
    }

    def rpc(addr, msg):
        r = replies[addr]
        if isinstance(r, Exception):
            raise r
        return r

    out = read_quorum_versions(["a", "b", "c", "d"], ["k", "j"], 2, rpc)
    assert out == {"k": ((1, 2), "d1")}


# ------------------------------------------------------------------ guards and probes
def test_guards_reject_non_finite_contributions_and_clip_norms():
    assert loss_ok(1.5) and loss_ok(None) and loss_ok(float("nan"), empty=True)
    assert not loss_ok(float("inf")) and not loss_ok("x")
    good = {"a": [torch.ones(3)], "b": torch.zeros(2)}
    bad = {"a": [torch.tensor([1.0, float("nan")])]}
    assert all_finite(good) and not all_finite(bad)
    assert contribution_ok(0.5, False, good) and not contribution_ok(0.5, False, bad)
    ts = [torch.full((4,), 3.0), torch.full((4,), 4.0)]
    n = clip_norm_(ts, 1.0)
    assert math.isclose(n, 10.0, rel_tol=1e-6)
    assert math.isclose(math.sqrt(sum(float((t * t).sum()) for t in ts)), 1.0, rel_tol=1e-5)
    small = [torch.full((4,), 0.1)]
    assert clip_norm_(small, 1.0) < 1.0 and torch.equal(small[0], torch.full((4,), 0.1))


def test_probe_margins_and_parsing():
    assert is_harmful(2.0, 2.2) and not is_harmful(2.0, 2.03)
    assert is_harmful(10.0, 10.3) and not is_harmful(10.0, 10.1)
    # untrusted wire values: numbers only (no strings, no booleans), finite
    assert as_finite_float(1.5) == 1.5 and as_finite_float(3) == 3.0
    assert as_finite_float("1.5") is None and as_finite_float(True) is None
    assert as_finite_float(float("nan")) is None and as_finite_float(None) is None
    assert not is_harmful(float("nan"), 5.0)
    assert TrustedProbe(None).empty and not TrustedProbe(torch.zeros(2, 8, dtype=torch.long)).empty


# ------------------------------------------------------------------ bandwidth
def test_encoding_tailored_to_the_declared_bandwidth():
    assert tailor_encoding(None) == ("none", 1.0) and tailor_encoding(100.0) == ("none", 1.0)
    assert tailor_encoding(10.0) == ("int8", 1.0)
    assert tailor_encoding(1.0, base_density=0.8) == ("int4", 0.5)
    assert tailor_encoding(10.0, base_compress="int4") == ("int4", 1.0)  # never weaker than the base
    assert rate_from_mbps(8.0) == 1e6 and rate_from_mbps(0) is None and rate_from_mbps(float("inf")) is None


def test_token_bucket_paces_sends_to_the_rate():
    b = TokenBucket(200_000.0, capacity=10_000.0)
    t0 = time.monotonic()
    for _ in range(6):
        b.take(10_000)  # 60 KB at 200 KB/s, 10 KB of burst: about 0.25 s
    dt = time.monotonic() - t0
    assert 0.2 <= dt < 1.5, dt
    TokenBucket(0.0).take(10 ** 9)  # rate 0 = unlimited


# ------------------------------------------------------------------ reputation and rate limits
def test_reputation_credit_debit_bounds_and_decay():
    r = Reputation(floor=0.5, credit=0.1, debit=0.3, decay_halflife=0)
    assert r.get("p") == 0.5 and r.get(None) == 0.5
    for _ in range(20):
        r.credit("p")
    assert r.get("p") == 1.0
    for _ in range(10):
        r.debit("q")
    assert r.get("q") == 0.0
    d = Reputation(floor=0.5, credit=0.4, decay_halflife=0.05)
    d.credit("p")
    high = d.get("p")
    time.sleep(0.2)
    assert 0.5 <= d.get("p") < high  # decays back toward the floor


def test_rate_limit_scales_with_reputation():
    rl = RateLimiter(capacity=4.0, refill_per_sec=0.0)
    trusted = sum(rl.allow("t", reputation=1.0) for _ in range(20))
    fresh = sum(rl.allow("f", reputation=0.0) for _ in range(20))
    assert trusted == 6 and fresh == 2
    assert all(rl.allow(None) for _ in range(50))  # local callers are not limited
