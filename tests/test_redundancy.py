"""Redundant execution, audits and private-state proposals (CPU, no sockets: the
scheduler's and the owner's handlers are driven message by message).

Behaviours of the reference's ``tests/test_redundancy.py`` (audits, check tasks, the
trusted-probe screen, private proposals), restated against this framework's API.
"""

import time

import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import ParameterServer, PeerIdentity, Reputation, Scheduler, make_grant
from opendipaco_b200.schedule.probe import TrustedProbe

from helpers import rr_corpus, tiny_config


def _sched(**kw):
    cfg = tiny_config()
    s = Scheduler(cfg, rr_corpus(cfg), ["127.0.0.1:1"], DiLoCoConfig(inner_steps=4, inner_lr=1e-3), 8,
                  host="127.0.0.1", **kw)
    with s._lock:
        s._completed = {p: 0 for p in s.topology.paths()}
        s._target = 10 ** 6
        s._serving = True
    return s


def _req(s, w):
    return s._handle({"type": "request", "worker_id": w}, 0, w)


def _commit(s, t, w, **extra):
    return s._handle({"type": "commit", "path": list(t["path"]), "lease": t["lease"], "gen_id": t["gen_id"],
                      "worker_id": w, "loss": 1.0, **extra}, 0, w)


def _check(s, t, w, digest, **extra):
    return s._handle({"type": "commit", "check_only": True, "path": list(t["path"]), "gen_id": t["gen_id"],
                      "lease": t["lease"], "worker_id": w, "digest": digest, **extra}, 0, w)


def _audit_with_checks(s, n_checks, primary_digest="good", base=(1, 2)):
    """Primary A on an audited path; the three other paths busy; A commits; then
    ``n_checks`` checkers receive the check tasks."""
    a = _req(s, "A")
    assert a.get("audit")
    for w in ("B", "C", "D"):
        assert _req(s, w)["type"] == "task"
    assert _commit(s, a, "A", digest=primary_digest, base=list(base))["accepted"]
    assert _req(s, "E")["type"] == "task"  # the audited path itself is free again
    checks = [(f"X{i}", _req(s, f"X{i}")) for i in range(n_checks)]
    assert all(t.get("check_only") and t["base"] == list(base) for _, t in checks)
    return a, checks


def test_all_agreeing_audit_credits_everyone():
    rep = Reputation(decay_halflife=0)
    s = _sched(redundancy=3, redundancy_rate=1.0, reputation=rep)
    a, checks = _audit_with_checks(s, 2)
    for w, t in checks:
        assert _check(s, t, w, "good")["check"]
    assert (tuple(a["path"]), a["gen_id"]) not in s._audits and s.metrics.invalid_rejected == 0
    assert all(rep.get(w) > rep.floor for w in ("A", "X0", "X1"))


def test_two_way_split_is_inconclusive():
    """Primary and one checker disagree, nobody else reports: no majority, nobody is
    punished or rewarded by the audit."""
    rep = Reputation(decay_halflife=0)
    s = _sched(redundancy=2, redundancy_rate=1.0, reputation=rep)
    a, checks = _audit_with_checks(s, 1)
    before = rep.get("X0")
    (w, t), = checks
    _check(s, t, w, "other")
    assert (tuple(a["path"]), a["gen_id"]) not in s._audits
    assert rep.get("X0") == before and s.metrics.invalid_rejected == 0


def test_timeout_resolves_without_punishing():
    rep = Reputation(decay_halflife=0)
    s = _sched(redundancy=3, redundancy_rate=1.0, reputation=rep, audit_timeout=0.1)
    _audit_with_checks(s, 2)  # check tasks handed out, no check ever commits
    a_rep = rep.get("A")
    time.sleep(0.2)
    with s._lock:
        s._reclaim_locked()
    assert not s._audits and rep.get("A") == a_rep and rep.get("X0") == rep.floor


def test_uncommitted_audit_is_reaped():
    """The primary never commits: the audit is dropped at its deadline and no check task
    is ever offered (there is no base to check)."""
    s = _sched(redundancy=3, redundancy_rate=1.0, audit_timeout=0.1)
    a = _req(s, "A")
    assert a.get("audit") and len(s._audits) == 1
    for w in ("B", "C", "D"):
        _req(s, w)
    assert _req(s, "X")["type"] == "idle"  # busy paths and an audit without a base
    time.sleep(0.2)
    with s._lock:
        s._reclaim_locked()
    assert not s._audits


def test_unassigned_or_repeated_check_commits_are_ignored():
    rep = Reputation(decay_halflife=0)
    s = _sched(redundancy=3, redundancy_rate=1.0, reputation=rep)
    _, checks = _audit_with_checks(s, 2)
    (w0, t0), (w1, t1) = checks
    _check(s, t0, "intruder", "bad")           # no check lease for this member
    _check(s, dict(t0, lease="forged"), w0, "bad")
    key = (tuple(t0["path"]), t0["gen_id"])
    assert s._audits[key]["checks"] == []
    _check(s, t0, w0, "good")
    _check(s, t0, w0, "good")                  # a second report from the same checker
    assert s._audits[key]["checks"] == [(w0, "good")]


def test_check_offered_only_to_distinct_workers_and_only_up_to_the_target():
    s = _sched(redundancy=3, redundancy_rate=1.0)
    _audit_with_checks(s, 2)
    assert _req(s, "X0")["type"] == "idle"     # already a checker of this audit
    assert _req(s, "A")["type"] == "idle"      # the primary never checks itself
    assert _req(s, "Y")["type"] == "idle"      # both check slots taken


def test_no_audits_when_rate_zero():
    s = _sched(redundancy=3, redundancy_rate=0.0)
    for w in "ABCD":
        t = _req(s, w)
        assert t["type"] == "task" and not t.get("audit")
    assert not s._audits


def test_check_task_carries_the_probe_and_the_screen_flags_harm():
    probe = torch.randint(0, 48, (4, 16))
    rep = Reputation(decay_halflife=0)
    s = _sched(redundancy=3, redundancy_rate=1.0, reputation=rep, probe=TrustedProbe(probe, batch_size=2),
               probe_quorum=2, probe_debit=True)
    _, checks = _audit_with_checks(s, 2)
    for _, t in checks:
        assert torch.equal(t["probe"], probe) and t["probe_batch"] == 2
    # both checkers measured the probe loss rising well past the margins: flagged, debited
    for w, t in checks:
        _check(s, t, w, "good", probe_before=2.0, probe_after=2.5)
    assert s.metrics.poison_flagged == 1 and rep.get("A") < rep.floor + 2 * rep.credit_step


def test_probe_screen_needs_a_quorum_and_ignores_malformed_reports():
    s = _sched(redundancy=3, redundancy_rate=1.0, probe=torch.randint(0, 48, (4, 16)), probe_quorum=2)
    _, checks = _audit_with_checks(s, 2)
    (w0, t0), (w1, t1) = checks
    _check(s, t0, w0, "good", probe_before=2.0, probe_after=2.5)    # one harmful report
    _check(s, t1, w1, "good", probe_before="2.0", probe_after=True)  # not numbers: dropped
    assert s.metrics.poison_flagged == 0


def test_honest_contribution_passes_the_screen_and_the_screen_is_off_by_default():
    s = _sched(redundancy=3, redundancy_rate=1.0, probe=torch.randint(0, 48, (4, 16)), probe_quorum=2)
    _, checks = _audit_with_checks(s, 2)
    for w, t in checks:
        _check(s, t, w, "good", probe_before=2.0, probe_after=1.98)
    assert s.metrics.poison_flagged == 0
    off = _sched(redundancy=3, redundancy_rate=1.0)
    _, checks = _audit_with_checks(off, 2)
    assert all("probe" not in t for _, t in checks)
    for w, t in checks:
        _check(off, t, w, "good", probe_before=2.0, probe_after=9.0)
    assert off.metrics.poison_flagged == 0


# ------------------------------------------------------------------ private proposals
def _owner(policy, quorum=2):
    cfg = tiny_config(embedding="private", head="private")
    sched = PeerIdentity.generate()
    keys = cfg.build_topology().module_keys()
    ps = ParameterServer(cfg, keys, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), host="127.0.0.1",
                         scheduler_pub=sched.public_key_hex, private_policy=policy, private_quorum=quorum)
    return ps, sched


def _propose(ps, sched, key, sd, token, peer=None):
    g = make_grant((0, 0), [key], 1.0, token, identity=sched)
    return ps._push({"grant": g, "updates": {}, "private": {key: sd}}, peer)


def _shifted(ps, key, by):
    return {n: t + by for n, t in ps.bank[key].state_dict().items()}


def test_proposal_applies_only_on_quorum_agreement():
    ps, sched = _owner("proposal")
    key = "embed.p0"
    old, new = ps.bank[key].state_dict()["embed_tokens.weight"].clone(), _shifted(ps, key, 0.5)
    _propose(ps, sched, key, new, "t1", "peer-a")
    assert torch.equal(ps.bank[key].state_dict()["embed_tokens.weight"], old)
    _propose(ps, sched, key, new, "t2", "peer-b")
    assert torch.equal(ps.bank[key].state_dict()["embed_tokens.weight"], new["embed_tokens.weight"])
    assert ps._versions[key][1] == 1 and key not in ps._proposals


def test_lone_repeated_or_forged_proposals_never_apply():
    ps, sched = _owner("proposal")
    key = "head.p1"
    old = {n: t.clone() for n, t in ps.bank[key].state_dict().items()}
    new = _shifted(ps, key, 1.0)
    _propose(ps, sched, key, new, "t1", "peer-a")
    _propose(ps, sched, key, new, "t2", "peer-a")       # the same proposer again
    rogue = PeerIdentity.generate()                      # a grant the scheduler did not sign
    g = make_grant((0, 0), [key], 1.0, "t3", identity=rogue)
    assert not ps._push({"grant": g, "updates": {}, "private": {key: new}}, "peer-b")["applied"]
    _propose(ps, sched, key, new, "t1", "peer-c")        # a replayed grant token
    assert all(torch.equal(ps.bank[key].state_dict()[n], old[n]) for n in old)


def test_disagreeing_proposals_do_not_corroborate():
    ps, sched = _owner("proposal")
    key = "embed.p1"
    old = ps.bank[key].state_dict()["embed_tokens.weight"].clone()
    for i, peer in enumerate(("a", "b", "c")):
        _propose(ps, sched, key, _shifted(ps, key, 0.1 * (i + 1)), f"t{i}", peer)
    assert torch.equal(ps.bank[key].state_dict()["embed_tokens.weight"], old)


def test_private_proposal_bucket_is_bounded():
    ps, sched = _owner("proposal", quorum=3)
    key = "embed.p2"
    for i in range(3 * ps._PROPOSALS_MAX):
        _propose(ps, sched, key, _shifted(ps, key, 0.01 * (i + 1)), f"t{i}", f"peer{i}")
    assert len(ps._proposals[key]) == ps._PROPOSALS_MAX


def test_overwrite_policy_applies_verbatim():
    ps, sched = _owner("overwrite")
    key = "head.p3"
    new = _shifted(ps, key, -0.25)
    assert _propose(ps, sched, key, new, "t1", "peer-a")["applied"]
    assert all(torch.equal(ps.bank[key].state_dict()[n], new[n]) for n in new)
