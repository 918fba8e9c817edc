"""Churn harness: a real in-process sharded cluster (tracker, signed-epoch scheduler,
parameter servers as key owners, sharded workers over loopback TCP) trained for a few
generations while owners crash, leave, sleep or join, reporting whether the run
survived and how membership moved.

    python -m opendipaco_b200.launch.churn --arm abrupt --rounds 4

Arms (the owner-churn patterns of the reference's ``examples/validate_churn.py``):

* ``none``     -- control: no membership change;
* ``abrupt``   -- an owner drops every connection and stops heartbeating; after the
  tracker TTL and the scheduler's ``owner_grace`` a new epoch moves its keys;
* ``graceful`` -- an owner leaves with ``shutdown(graceful=True)``: it drains its keys to
  the backups and tombstones itself, so failover does not wait out the grace;
* ``flap``     -- an owner is silent for less than the grace and comes back: absorbed,
  no new epoch;
* ``suspend``  -- an owner sleeps past the grace (removed) and wakes (added back);
* ``join``     -- a new owner appears mid-run and cold-syncs the keys it is assigned.

Metrics: ``survived`` (every generation completed), ``epochs`` (the final epoch number),
``remaps`` (keys whose owner set changed between the first and the final epoch),
``reclaims`` (leases the scheduler took back), ``failover_s`` (departure until the
survivors serve every key; ``abrupt`` / ``graceful``) and ``settle_s`` (arrival until the
returning or new owner is in the epoch and every key is served; ``suspend`` / ``join``). The detection timings are
deliberately short so a run takes seconds.
"""

from __future__ import annotations

import argparse
import json
import threading
import time

import torch

from .. import BackboneConfig, DiLoCoConfig, DiPaCoConfig
from ..data import ShardedCorpus
from ..schedule import ParameterServer, PeerIdentity, Scheduler, Tracker, owners_for, run_sharded_worker

ARMS = ("none", "abrupt", "graceful", "flap", "suspend", "join")
AUTH = "churn"


def _wait_until(pred, timeout: float, step: float = 0.05) -> bool:
    end = time.monotonic() + timeout
    while time.monotonic() < end:
        if pred():
            return True
        time.sleep(step)
    return False


def small_config() -> DiPaCoConfig:
    bb = BackboneConfig(vocab_size=48, hidden_size=32, num_attention_heads=4, intermediate_size=64,
                        layers_per_level=[1, 1], max_position_embeddings=64)
    return DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=16)


def _corpus(cfg: DiPaCoConfig) -> ShardedCorpus:
    g = torch.Generator().manual_seed(0)
    docs = [torch.randint(0, cfg.backbone.vocab_size, (48,), generator=g) for _ in range(32)]
    assign = torch.arange(len(docs)) % cfg.num_paths
    return ShardedCorpus.from_assignments(docs, assign, cfg.num_paths, cfg.sequence_length)


class ChurnCluster:
    """Tracker + scheduler + ``n_owners`` owners + ``n_workers`` workers on loopback."""

    def __init__(self, *, n_owners: int = 4, n_workers: int = 2, k: int = 3, ttl: float = 1.0,
                 owner_grace: float = 2.0, min_epoch_interval: float = 0.5):
        self.cfg, self.dl = small_config(), DiLoCoConfig(inner_steps=4, inner_lr=1e-3)
        self.keys = self.cfg.build_topology().module_keys()
        self.k, self.ttl, self.grace, self.min_interval = k, ttl, owner_grace, min_epoch_interval
        self.n_owners, self.n_workers = n_owners, n_workers
        self.sched_id = PeerIdentity.generate()
        self.owner_ids = [PeerIdentity.generate() for _ in range(n_owners)]
        self.tracker = self.sched = None
        self.owners: list[ParameterServer] = []
        self.workers: list[threading.Thread] = []
        self._stop_workers = threading.Event()

    # -- lifecycle ------------------------------------------------------------------
    def _owner(self, ident: PeerIdentity, admitted) -> ParameterServer:
        ps = ParameterServer(self.cfg, [], self.dl, host="127.0.0.1", port=0, identity=ident, auth_key=AUTH,
                             scheduler_pub=self.sched_id.public_key_hex,
                             scheduler_addr=("127.0.0.1", self.sched.port), replicate_interval=0.2,
                             admitted_peers=admitted)
        ps.start()
        ps.start_tracker_heartbeat(("127.0.0.1", self.tracker.port), "127.0.0.1", interval=max(0.1, self.ttl / 3))
        return ps

    def __enter__(self) -> "ChurnCluster":
        self.tracker = Tracker(host="127.0.0.1", port=0, open_enrollment=True, ttl=self.ttl)
        self.tracker.start()
        self.sched = Scheduler(self.cfg, _corpus(self.cfg), [], self.dl, 4, host="127.0.0.1", port=0,
                               identity=self.sched_id, auth_key=AUTH, admitted_peers=self.owner_ids,
                               heartbeat_timeout=2.0)
        self.sched.start()
        for ident in self.owner_ids:
            self.owners.append(self._owner(ident, [p for p in self.owner_ids if p is not ident]))
        if not _wait_until(lambda: len(self.tracker.records()) >= self.n_owners, 10):
            raise RuntimeError("owners did not register with the tracker")
        self.sched.watch_tracker(("127.0.0.1", self.tracker.port), k=self.k, owner_grace=self.grace,
                                 min_epoch_interval=self.min_interval, poll_interval=0.2)
        if not _wait_until(lambda: all(ps._epoch is not None for ps in self.owners), 10):
            raise RuntimeError("owners did not receive the first epoch")
        for seed in range(self.n_workers):
            t = threading.Thread(target=run_sharded_worker, args=(self.cfg, self.dl, ("127.0.0.1", self.sched.port)),
                                 kwargs=dict(seed=seed, auth_key=AUTH, heartbeat_interval=0.5, reconnect=True,
                                             reconnect_timeout=10.0, stop_event=self._stop_workers),
                                 daemon=True)
            t.start()
            self.workers.append(t)
        return self

    def __exit__(self, *exc) -> None:
        self._stop_workers.set()
        if self.sched is not None:
            self.sched.shutdown()
        for ps in self.owners:
            ps.shutdown()
        if self.tracker is not None:
            self.tracker.shutdown()
        for t in self.workers:
            t.join(timeout=15)

    # -- membership views -----------------------------------------------------------
    def epoch_ids(self) -> set:
        rec = self.sched._epoch_record
        return {o["peer_id"] for o in rec["owners"]} if rec else set()

    def placement(self) -> dict:
        rec = self.sched._epoch_record
        return {key: frozenset(o["peer_id"] for o in owners_for(key, rec)) for key in self.keys} if rec else {}

    def served_by(self, live: list[ParameterServer]) -> bool:
        """Every key's owners are live and at least one of them serves it active."""
        rec = self.sched._epoch_record
        if rec is None:
            return False
        ids = {ps.peer_id for ps in live}
        for key in self.keys:
            own = {o["peer_id"] for o in owners_for(key, rec)}
            if not own <= ids or not any(key in ps._active for ps in live if ps.peer_id in own):
                return False
        return True

    def join_new_owner(self) -> ParameterServer:
        """A new owner mid-run: the incumbents and the scheduler admit it at runtime."""
        ident = PeerIdentity.generate()
        for ps in self.owners:
            ps.admit_peer(ident)
        self.sched.admit_peer(ident)
        joiner = self._owner(ident, list(self.owner_ids))
        self.owners.append(joiner)
        return joiner


def _inject(arm: str, cl: ChurnCluster, metrics: dict) -> None:
    if arm == "none":
        return
    _wait_until(lambda: cl.sched._T >= max(1, cl.sched._target // 3), 30)
    victim = cl.owners[0]
    if arm in ("abrupt", "graceful"):
        t0 = time.monotonic()
        if arm == "abrupt":
            victim.simulate_crash()
        else:
            victim.shutdown(graceful=True)
        live = cl.owners[1:]
        if _wait_until(lambda: victim.peer_id not in cl.epoch_ids() and cl.served_by(live), 30):
            metrics["failover_s"] = round(time.monotonic() - t0, 2)
    elif arm == "flap":
        victim.pause_heartbeat()
        time.sleep(cl.grace * 0.3)
        victim.resume_heartbeat()
    elif arm == "suspend":
        victim.pause_heartbeat()
        _wait_until(lambda: victim.peer_id not in cl.epoch_ids(), 30)
        t0 = time.monotonic()
        victim.resume_heartbeat()
        if _wait_until(lambda: victim.peer_id in cl.epoch_ids() and cl.served_by(cl.owners), 30):
            metrics["settle_s"] = round(time.monotonic() - t0, 2)
    elif arm == "join":
        t0 = time.monotonic()
        joiner = cl.join_new_owner()
        if _wait_until(lambda: joiner.peer_id in cl.epoch_ids() and bool(joiner._active)
                       and cl.served_by(cl.owners), 30):
            metrics["settle_s"] = round(time.monotonic() - t0, 2)
    else:
        raise ValueError(f"unknown churn arm {arm!r} (one of {ARMS})")


def run_arm(arm: str, *, rounds: int = 4, **cluster_kw) -> dict:
    """Train ``rounds`` generations under churn pattern ``arm``; returns the metrics."""
    if arm not in ARMS:
        raise ValueError(f"unknown churn arm {arm!r} (one of {ARMS})")
    metrics = {"arm": arm, "survived": False, "epochs": 0, "remaps": 0, "reclaims": 0, "failover_s": None,
               "settle_s": None}
    with ChurnCluster(**cluster_kw) as cl:
        first = cl.placement()
        injector = threading.Thread(target=_inject, args=(arm, cl, metrics), daemon=True)
        injector.start()
        completed = cl.sched.fit(num_generations=rounds, total_generations=rounds)
        injector.join(timeout=40)
        metrics["survived"] = sum(completed.values()) >= cl.sched._target
        rec = cl.sched._epoch_record
        metrics["epochs"] = int(rec["epoch"]) if rec else 0
        last = cl.placement()
        metrics["remaps"] = sum(1 for key in cl.keys if first.get(key) != last.get(key))
        metrics["reclaims"] = cl.sched.metrics.reclaims
    return metrics


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--arm", choices=ARMS, default="abrupt")
    ap.add_argument("--rounds", type=int, default=4)
    ap.add_argument("--owners", type=int, default=4)
    ap.add_argument("--grace", type=float, default=2.0)
    args = ap.parse_args(argv)
    print(json.dumps(run_arm(args.arm, rounds=args.rounds, n_owners=args.owners, owner_grace=args.grace)))


if __name__ == "__main__":
    main()
