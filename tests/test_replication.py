"""Owner-to-owner replication under epochs (CPU, loopback): exact state (weights and
outer momentum) only for sessions authenticated as owners of the key, drains only from
them, a new owner syncs its gained keys before serving them (presenting the epoch that
gives it the key), a key with no reachable previous replica is served after the sync
timeout, and decentralized backups adopt only quorum-confirmed states.

Behaviours of the reference's ``tests/test_replication.py`` and
``tests/test_persistence.py`` (``src/opendipaco/schedule/sharded.py`` replication).
"""

import time

import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import ParameterServer, PeerIdentity, make_epoch_record, make_peer_record
from opendipaco_b200.schedule.ownership import derive_epoch, owners_for

from helpers import tiny_config

DL = DiLoCoConfig(inner_steps=2, inner_lr=1e-3)
KEY = "owners-secret"


def _servers(n, cfg, sched=None, **kw):
    ids = [PeerIdentity.generate() for _ in range(n)]
    pss = [ParameterServer(cfg, [], DL, host="127.0.0.1", auth_key=KEY, identity=i, replicate_interval=3600,
                           scheduler_pub=sched.public_key_hex if sched else None, **kw) for i in ids]
    for ps in pss:
        ps.start()
    return pss


def _recs(pss):
    return [make_peer_record(ps.identity, reachability="public", addr=("127.0.0.1", ps.port), roles=["owner"])
            for ps in pss]


def _shutdown(pss):
    for ps in pss:
        ps.shutdown()


def _fetch_state(key, **extra):
    return {"type": "fetch", "keys": [key], "have": {}, "include_state": True, **extra}


def test_exact_state_only_for_owner_sessions():
    cfg, sched = tiny_config(), PeerIdentity.generate()
    pss = _servers(3, cfg, sched)
    try:
        epoch = make_epoch_record(sched, epoch=0, owner_records=_recs(pss), k=2, bootstrap=True)
        for ps in pss:
            ps.apply_epoch(epoch)
        key = "L0E0"
        prim, back = (next(p for p in pss if p.peer_id == o["peer_id"]) for o in owners_for(key, epoch))
        third = next(p for p in pss if p not in (prim, back))
        assert key in prim._fetch(_fetch_state(key), None)["missing"]                    # shared-key session
        assert key in prim._fetch(_fetch_state(key), PeerIdentity.generate().peer_id)["missing"]
        assert key in prim._fetch(_fetch_state(key), third.peer_id)["missing"]            # an owner, not of this key
        reply = prim._fetch(_fetch_state(key), back.peer_id)
        assert key in reply["weights"] and key in reply["state"]
        plain = prim._fetch({"type": "fetch", "keys": [key], "have": {}})               # a worker's fetch
        assert key in plain["weights"] and "state" not in plain
        # over TCP the backup dials by identity (its epoch admitted it) and pulls
        prim._versions[key] = (0, 3)
        assert back._replicate_once().get(key) == (0, 3)
    finally:
        _shutdown(pss)


def test_a_newer_signed_epoch_lets_a_new_owner_sync_first():
    """The new owner presents the epoch that gives it the key before the serving owner
    has seen that epoch; a forged or older claim does not work."""
    cfg, sched = tiny_config(), PeerIdentity.generate()
    pss = _servers(2, cfg, sched)
    try:
        old = make_epoch_record(sched, epoch=0, owner_records=_recs(pss[:1]), k=1, bootstrap=True)
        pss[0].apply_epoch(old)
        new = make_epoch_record(sched, epoch=1, owner_records=_recs(pss), k=2)
        key = "L1E1"
        joiner = pss[1].peer_id
        assert key in pss[0]._fetch(_fetch_state(key), joiner)["missing"]
        assert key in pss[0]._fetch(_fetch_state(key, epoch=new), joiner)["weights"]
        forged = make_epoch_record(PeerIdentity.generate(), epoch=1, owner_records=_recs(pss), k=2)
        assert key in pss[0]._fetch(_fetch_state(key, epoch=forged), joiner)["missing"]
    finally:
        _shutdown(pss)


def test_drains_only_from_owners_and_never_in_decentralized_mode():
    cfg = tiny_config()
    sched = PeerIdentity.generate()
    pss = _servers(2, cfg, sched)
    dec = ParameterServer(cfg, [], DL, identity=PeerIdentity.generate(), schedule_mode="decentralized",
                          auth_key=KEY)
    try:
        epoch = make_epoch_record(sched, epoch=0, owner_records=_recs(pss), k=2, bootstrap=True)
        for ps in pss:
            ps.apply_epoch(epoch)
        a, b = pss
        key = "L0E1"
        sd = {n: t + 1 for n, t in b.bank[key].state_dict().items()}
        msg = {"states": {key: {"version": [0, 5], "weights": sd, "state": None}}}
        assert b._drain_recv(msg, None)["adopted"] == []                          # a worker with the shared key
        assert b._drain_recv(msg, PeerIdentity.generate().peer_id)["adopted"] == []
        assert b._drain_recv(msg, a.peer_id)["adopted"] == [key] and b._versions[key] == (0, 5)
        assert dec._drain_recv(msg, a.peer_id)["adopted"] == []
    finally:
        _shutdown(pss)


def test_gained_keys_wait_for_a_previous_replica():
    """A joining owner serves its gained keys only after a previous replica answered;
    with none reachable it serves them after the sync timeout."""
    cfg, sched = tiny_config(), PeerIdentity.generate()
    pss = _servers(2, cfg, sched, sync_timeout=0.3)
    try:
        first, joiner = pss
        old = make_epoch_record(sched, epoch=0, owner_records=_recs([first]), k=1, bootstrap=True)
        first.apply_epoch(old)
        key = "L0E0"
        first._versions[key] = (0, 7)
        with torch.no_grad():
            next(iter(first.bank[key].parameters())).add_(0.5)
        joiner.apply_epoch(old, bootstrap=False)   # a non-member of the old epoch holds nothing active
        new = make_epoch_record(sched, epoch=1, owner_records=_recs(pss), k=2)
        first.admit_peer(joiner.identity)          # the operator admitted the newcomer; first is still on epoch 0
        joiner.apply_epoch(new)
        assert key in joiner._active and joiner._versions[key] == (0, 7)
        assert torch.equal(next(iter(joiner.bank[key].parameters())), next(iter(first.bank[key].parameters())))
        # the only previous replica is gone: the gained keys wait, then are served locally
        first.simulate_crash()
        lone = ParameterServer(cfg, [], DL, host="127.0.0.1", auth_key=KEY, identity=PeerIdentity.generate(),
                               scheduler_pub=sched.public_key_hex, sync_timeout=0.3)
        lone.start()
        try:
            lone.apply_epoch(old, bootstrap=False)  # its previous epoch: only the crashed owner
            gained = make_epoch_record(sched, epoch=3, owner_records=_recs([lone]), k=1)
            lone.apply_epoch(gained)
            assert lone._syncing and not lone._active & set(lone._syncing)
            time.sleep(0.35)
            lone._retry_sync()
            assert not lone._syncing and key in lone._active
        finally:
            lone.shutdown()
    finally:
        _shutdown(pss)


def test_decentralized_backup_adopts_only_quorum_confirmed_state():
    cfg = tiny_config()
    pss = _servers(3, cfg, schedule_mode="decentralized", read_quorum=2)
    try:
        epoch = derive_epoch(_recs(pss), k=3)
        for ps in pss:
            ps.apply_epoch(epoch, bootstrap=True)
        key = "L1E0"
        owners = [next(p for p in pss if p.peer_id == o["peer_id"]) for o in owners_for(key, epoch)]
        prim, b1, b2 = owners
        with torch.no_grad():  # a Byzantine primary claims a newer version of a state nobody else has
            next(iter(prim.bank[key].parameters())).add_(3.0)
        prim._versions[key] = (epoch["epoch"], 9)
        assert key not in b1._replicate_once()
        # once a second replica holds the same (version, state) the pull is confirmed
        b2.bank[key].load_state_dict(prim.bank[key].state_dict())
        b2._versions[key] = prim._versions[key]
        assert b1._replicate_once().get(key) == prim._versions[key]
    finally:
        _shutdown(pss)


def test_restarted_owner_adopts_the_newest_replica_before_serving(tmp_path):
    """A primary restarts from a checkpoint older than its backup's state: it pulls the
    backup's newer version (weights and momentum) before it serves the key, and a lone
    owner (no other replica) serves its checkpoint at once."""
    cfg, sched = tiny_config(), PeerIdentity.generate()
    pss = _servers(2, cfg, sched)
    try:
        epoch = make_epoch_record(sched, epoch=0, owner_records=_recs(pss), k=2, bootstrap=True)
        for ps in pss:
            ps.apply_epoch(epoch)
        key = "L1E1"
        prim_id = owners_for(key, epoch)[0]["peer_id"]
        prim = next(p for p in pss if p.peer_id == prim_id)
        back = next(p for p in pss if p is not prim)
        prim.save_modules(str(tmp_path))                    # checkpoint at (0, 0)
        with torch.no_grad():
            next(iter(back.bank[key].parameters())).add_(0.25)
        back._versions[key] = (0, 4)                        # the backup trained on
        ident = prim.identity
        prim.shutdown()
        again = ParameterServer(cfg, [], DL, host="127.0.0.1", auth_key=KEY, identity=ident,
                                replicate_interval=3600, scheduler_pub=sched.public_key_hex,
                                resume_dir=str(tmp_path))
        again.start()
        try:
            moved = make_epoch_record(sched, epoch=1, owner_records=_recs([again, back]), k=2)
            back.apply_epoch(moved)
            again.apply_epoch(moved)
            assert key in again._active and again._versions[key] == (0, 4)
            assert torch.equal(next(iter(again.bank[key].parameters())), next(iter(back.bank[key].parameters())))
        finally:
            again.shutdown()
        lone = ParameterServer(cfg, [], DL, host="127.0.0.1", auth_key=KEY, identity=ident, replicate_interval=3600,
                               scheduler_pub=sched.public_key_hex, resume_dir=str(tmp_path))
        lone.start()
        try:
            lone.apply_epoch(make_epoch_record(sched, epoch=2, owner_records=_recs([lone]), k=1))
            assert key in lone._active and not lone._syncing
        finally:
            lone.shutdown()
    finally:
        _shutdown(pss)
