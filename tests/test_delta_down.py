"""Delta-down (CPU): an owner with ``down="delta"`` ships a worker int8 deltas against
the version the worker holds while that version is in its ring (8 deep by default),
full weights after it ages out; ``down="full"`` never ships a delta; the worker keeps
one keyframe per key and recovers with a full fetch when it lacks the base; whole
sharded runs train with delta-down, with audits and across path switches; a fetch falls back
to the next replica when the primary lacks a key or does not answer.

Behaviours of the reference's ``tests/test_w2_delta.py``.
"""

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import ParameterServer, PeerIdentity, make_grant
from opendipaco_b200.schedule.compress import apply_state_delta
from opendipaco_b200.schedule.sharded import _fetch_keys

from helpers import tiny_config

SCHED = PeerIdentity.generate()


def _owner(**kw):
    cfg = tiny_config()
    keys = sorted(cfg.build_topology().module_keys())
    ps = ParameterServer(cfg, keys, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), host="127.0.0.1",
                         scheduler_pub=SCHED.public_key_hex, **kw)
    return ps, "L0E0"


def _push(ps, key, tok, scale=0.01):
    grad = [scale * torch.ones_like(p) for p in ps.bank[key].parameters()]
    assert ps._push({"grant": make_grant((0, 0), [key], 1.0, tok, identity=SCHED), "updates": {key: {"grad": grad}},
                     "private": {}})["applied"]


def _maxdiff(a, b):
    return max((a[n].float() - b[n].float()).abs().max().item() for n in a)


def test_owner_ships_deltas_then_full_weights_once_the_base_ages_out():
    ps, key = _owner(down="delta")
    assert ps.version_history == 8
    full = ps._fetch({"keys": [key], "have": {}})
    keyframe = full["weights"][key]
    assert "delta" not in keyframe and tuple(full["versions"][key]) == (0, 0)
    _push(ps, key, "t1")
    payload = ps._fetch({"keys": [key], "have": {key: [0, 0]}})["weights"][key]
    assert "delta" in payload and tuple(payload["base"]) == (0, 0)
    cur = ps.bank[key].state_dict()
    recon = apply_state_delta(keyframe, payload["delta"])
    assert _maxdiff(recon, cur) < _maxdiff(keyframe, cur) / 20
    for i in range(9):  # nine more versions: (0, 0) leaves the ring
        _push(ps, key, f"a{i}")
    assert "delta" not in ps._fetch({"keys": [key], "have": {key: [0, 0]}})["weights"][key]
    assert ps._fetch({"keys": [key], "have": {key: list(ps._versions[key])}})["weights"] == {}  # up to date


def test_down_full_never_ships_a_delta():
    ps, key = _owner(version_history=8)
    _push(ps, key, "t1")
    assert "delta" not in ps._fetch({"keys": [key], "have": {key: [0, 0]}})["weights"][key]


class _Loop:
    """A worker link that calls the owner's handler in process."""

    def __init__(self, ps):
        self.ps = ps

    def ps_rpc(self, addr, msg):
        return self.ps._fetch(msg)


def test_worker_keeps_one_keyframe_per_key_and_recovers_without_one():
    ps, key = _owner(down="delta")
    link, routing = _Loop(ps), {key: [("127.0.0.1", 1)]}
    versions, keyframes = {}, {}
    _fetch_keys(link, routing, [key], versions, set(), keyframes)
    for i in range(3):
        _push(ps, key, f"t{i}")
        got = _fetch_keys(link, routing, [key], versions, set(), keyframes)
        assert versions[key] == ps._versions[key] and list(keyframes) == [key]
        assert _maxdiff(got[key], ps.bank[key].state_dict()) < 1e-3
    # a worker that lost its keyframe (another path's keys evicted it) gets a full copy next
    keyframes.clear()
    _push(ps, key, "t9")
    with pytest.raises(ValueError):
        _fetch_keys(link, routing, [key], versions, set(), keyframes)
    assert key not in versions
    got = _fetch_keys(link, routing, [key], versions, set(), keyframes)
    assert all(torch.equal(got[key][n], ps.bank[key].state_dict()[n]) for n in got[key])


@pytest.mark.parametrize("audits", [False, True])
def test_sharded_runs_train_with_delta_down(audits):
    from opendipaco_b200.launch import LaunchConfig, run_local

    d = {"mode": "sharded",
         "model": {"vocab_size": 64, "hidden_size": 32, "num_attention_heads": 4, "intermediate_size": 64,
                   "max_position_embeddings": 64, "layers_per_level": [1, 1], "level_sizes": [2, 2],
                   "sequence_length": 16},
         "diloco": {"inner_steps": 2},
         "data": {"source": "synthetic", "num_documents": 32, "synthetic_doc_len": 40},
         "transport": {"host": "127.0.0.1", "port": 0, "auth_key": "s3cret", "down": "delta",
                       "heartbeat_timeout": 10.0},
         "sharded": {"num_shards": 2},
         "run": {"generations": 3, "batch_size": 4, "local_workers": 2}}
    if audits:
        d["robustness"] = {"redundancy": 2, "redundancy_rate": 0.5}
    sched, completed = run_local(LaunchConfig.from_dict(d))
    assert len(completed) == 4 and min(completed.values()) >= 3
    assert sched.metrics.accepted_updates >= 12


def test_fetch_falls_back_to_the_next_replica():
    """A key its primary reports missing (syncing, not active there yet) or a primary
    that does not answer is fetched from the key's next replica."""
    a, key = _owner()
    b, _ = _owner()
    _push(b, key, "t1")
    a._active.discard(key)                       # the primary still syncs this key

    class _Owners:
        def ps_rpc(self, addr, msg):
            if addr == "down":
                raise ConnectionError("gone")
            return {"a": a, "b": b}[addr]._fetch(msg)

    versions, keyframes = {}, {}
    got = _fetch_keys(_Owners(), {key: ["a", "b"]}, [key], versions, set(), keyframes)
    assert versions[key] == b._versions[key] and torch.equal(got[key]["layers.0.mlp.up_proj.weight"],
                                                             b.bank[key].state_dict()["layers.0.mlp.up_proj.weight"])
    versions.clear()
    assert key in _fetch_keys(_Owners(), {key: ["down", "b"]}, [key], versions, set(), keyframes)
    with pytest.raises(ConnectionError):
        _fetch_keys(_Owners(), {key: ["down", "a"]}, [key], {}, set(), {})
