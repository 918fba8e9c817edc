"""In-process, fault-tolerant task-queue scheduler (reference ``schedule/scheduler.py``).

Worker threads lease path-tasks of a *generation* from a queue, train them and hand
back a :class:`Contribution` (shared pseudo-gradients, private weights, the path's
inner-optimizer state). A worker that raises :class:`TransientFault` nacks (the path
is re-queued at once); one that raises :class:`Preempt` dies silently and the
monitor re-queues its lease when it expires. A path that exhausts ``max_attempts``
is dropped for the generation. Every task trains with its own generator seeded from
``(seed, path, generation)`` (same mixing constants as the reference, so a run is
reproducible across the two frameworks), and the reduce folds contributions in path
order, so results do not depend on worker count or on the pattern of recovered
failures. The outer step reuses the engine's weighting and optimizer.
"""

from __future__ import annotations

import collections
import math
import threading
import time
from dataclasses import dataclass, field

import torch

from ..models.path import build_path_model
from ..optim.diloco import apply_outer_grads, make_inner_optimizer, module_delta
from ..topology import Path, is_private_key
from ..train.loop import DiPaCoEngine, RoundMetrics, _opt_state_cpu, _state_cpu, run_inner_steps
from .probe import safe_probe_loss


class TransientFault(Exception):
    """Raised by a fault hook: recoverable error -> immediate re-queue."""


class Preempt(Exception):
    """Raised by a fault hook: the worker vanishes -> re-queue after lease expiry."""


@dataclass
class Contribution:
    path: Path
    path_idx: int
    loss: float
    shared_delta: dict[str, list[torch.Tensor]]
    private_state: dict[str, dict]
    opt_state: dict
    empty: bool = False
    probe_before: float | None = None
    probe_after: float | None = None


@dataclass
class _OuterAccumulator:
    acc_sum: dict[str, list[torch.Tensor]]
    acc_w: dict[str, float]
    per_path_loss: dict


@dataclass
class _Generation:
    """Thread-safe lease / complete / nack / reclaim bookkeeping for one generation."""

    paths: list[Path]
    lease_timeout: float
    max_attempts: int
    min_success: int
    _cv: threading.Condition = field(default_factory=threading.Condition)
    _pending: collections.deque = field(default_factory=collections.deque)
    _leased: dict = field(default_factory=dict)
    _attempts: collections.Counter = field(default_factory=collections.Counter)
    results: dict = field(default_factory=dict)
    failed: set = field(default_factory=set)
    reclaimed: int = 0

    def __post_init__(self):
        self._pending.extend(self.paths)

    def _expire(self) -> None:
        now = time.monotonic()
        for path, deadline in list(self._leased.items()):
            if now < deadline:
                continue
            del self._leased[path]
            if path in self.results:
                continue
            if self._attempts[path] >= self.max_attempts:
                self.failed.add(path)
            else:
                self._pending.append(path)
                self.reclaimed += 1

    def _finished(self) -> bool:
        return not self._pending and not self._leased and \
            len(self.results) + len(self.failed) >= len(self.paths)

    def _take(self, path: Path):
        self._attempts[path] += 1
        self._leased[path] = time.monotonic() + self.lease_timeout
        return path, self._attempts[path]

    def lease(self, wait: float = 0.05):
        with self._cv:
            while True:
                self._expire()
                if self._finished():
                    return None
                if self._pending:
                    return self._take(self._pending.popleft())
                self._cv.wait(wait)

    def poll_lease(self, pick=None):
        """Non-blocking: ``(path, attempt)``, ``"done"`` or ``"idle"``; ``pick(pending)``
        may choose which pending path to hand out (data locality)."""
        with self._cv:
            self._expire()
            if self._finished():
                return "done"
            if not self._pending:
                return "idle"
            if pick is None:
                path = self._pending.popleft()
            else:
                path = pick(list(self._pending))
                if path is None:
                    return "idle"
                self._pending.remove(path)
            return self._take(path)

    def refresh_lease(self, path: Path) -> None:
        with self._cv:
            if path in self._leased:
                self._leased[path] = time.monotonic() + self.lease_timeout

    def complete(self, path: Path, contrib: Contribution) -> None:
        with self._cv:
            if path in self.results:
                return
            self._leased.pop(path, None)
            self.failed.discard(path)
            try:
                self._pending.remove(path)
            except ValueError:
                pass
            self.results[path] = contrib
            self._cv.notify_all()

    def nack(self, path: Path) -> None:
        with self._cv:
            self._leased.pop(path, None)
            if path in self.results:
                return
            if self._attempts[path] >= self.max_attempts:
                self.failed.add(path)
            else:
                self._pending.append(path)
            self._cv.notify_all()

    def reclaim(self) -> None:
        with self._cv:
            self._expire()
            self._cv.notify_all()

    def is_done(self) -> bool:
        with self._cv:
            return self._finished()

    def pending_paths(self) -> list:
        with self._cv:
            self._expire()
            return list(self._pending)


def task_seed(seed: int, path_idx: int, generation: int) -> int:
    return ((seed * 0x9E3779B1) ^ (path_idx * 0x85EBCA77) ^ (generation * 0xC2B2AE35)) & 0x7FFFFFFFFFFFFFFF


class AsyncScheduler:
    """Drives a :class:`DiPaCoEngine` (use ``materialize="serial"``) through the queue."""

    def __init__(self, engine: DiPaCoEngine, *, num_workers: int = 4, lease_timeout: float = 30.0,
                 max_attempts: int = 3, min_fraction: float = 1.0):
        self.engine = engine
        self.num_workers = num_workers
        self.lease_timeout = lease_timeout
        self.max_attempts = max_attempts
        self.min_fraction = min_fraction
        self.seed = getattr(engine, "_seed", 0)
        self.dropped: set[Path] = set()
        self.errors: dict[Path, str] = {}
        self._last_batch_size = 1

    # -- map ---------------------------------------------------------------
    def _train_path(self, path: Path, shard: torch.Tensor, batch_size: int, generation: int,
                    inner_steps: int | None = None, probe=None) -> Contribution:
        e = self.engine
        pidx = e.topology.path_index(path)
        shard = shard.to(e.device)
        if shard.size(0) == 0:
            return Contribution(path, pidx, float("nan"), {}, {}, {}, empty=True)
        pm = build_path_model(e.config, path, e.bank, deepcopy=True,
                              dedup_private=getattr(e.diloco, "dedup_private", False)).to(e.device)
        opt = make_inner_optimizer(pm, e.diloco)
        if e._opt_state.get(path) is not None:
            opt.load_state_dict(e._opt_state[path])
        gen = torch.Generator().manual_seed(task_seed(self.seed, pidx, generation))
        steps = inner_steps or e.diloco.inner_steps
        total = e.total_rounds * steps if e.total_rounds else None
        screening = probe is not None and not probe.empty
        before = safe_probe_loss(probe, pm) if screening else None
        loss = run_inner_steps(pm, opt, shard, batch_size, gen, inner_steps=steps, total_steps=total,
                               base_step=generation * steps, diloco=e.diloco, device=e.device)
        after = safe_probe_loss(probe, pm) if screening else None
        shared, private = {}, {}
        for key, mod in pm.modules_by_key().items():
            if is_private_key(key):
                private[key] = _state_cpu(mod.state_dict())
            else:
                shared[key] = [d.detach().cpu() for d in module_delta(e.bank[key], mod)]
        return Contribution(path, pidx, loss, shared, private, _opt_state_cpu(opt.state_dict()),
                            probe_before=before, probe_after=after)

    def _worker(self, gen: _Generation, corpus, batch_size, generation, fault_hook):
        while True:
            leased = gen.lease()
            if leased is None:
                return
            path, attempt = leased
            try:
                if fault_hook is not None:
                    fault_hook(path, attempt)
                shard = corpus.shard(self.engine.topology.path_index(path))
                gen.complete(path, self._train_path(path, shard, batch_size, generation))
            except Preempt:
                continue
            except Exception as exc:  # recorded for debugging, then re-queued
                self.errors[path] = repr(exc)
                gen.nack(path)

    def _monitor(self, gen: _Generation):
        while not gen.is_done():
            time.sleep(max(self.lease_timeout / 2, 0.005))
            gen.reclaim()

    # -- reduce --------------------------------------------------------------
    def _new_accumulator(self) -> _OuterAccumulator:
        e = self.engine
        keys = [k for k in e.topology.module_keys() if not is_private_key(k) and k in e.bank]
        return _OuterAccumulator({k: [torch.zeros_like(p) for p in e.bank[k].parameters()] for k in keys},
                                 dict.fromkeys(keys, 0.0), {})

    def _fold_contribution(self, acc: _OuterAccumulator, corpus, c: Contribution, *,
                           persist_opt: bool = True) -> None:
        if c.empty:
            return
        e = self.engine
        acc.per_path_loss[c.path] = c.loss
        for key, sd in c.private_state.items():
            e.bank[key].load_state_dict({k: v.to(e.device) for k, v in sd.items()})
        for key, delta in c.shared_delta.items():
            w = e._outer_weight(key, c.path_idx, corpus)
            for a, d in zip(acc.acc_sum[key], delta):
                a.add_(w * d.to(e.device))
            acc.acc_w[key] += w
        if persist_opt and c.opt_state:
            e._opt_state[c.path] = c.opt_state

    def _finalize_outer_step(self, acc: _OuterAccumulator, corpus, generation) -> RoundMetrics:
        e = self.engine
        norms = []
        for key, w in acc.acc_w.items():
            if w == 0.0:
                continue
            avg = ([s / max(w, 1e-12) for s in acc.acc_sum[key]] if e.diloco.normalize_outer_delta
                   else acc.acc_sum[key])
            if e.diloco.rescale_by_sqrt_sharing:
                sc = math.sqrt(e.topology.sharing_count(key))
                avg = [a * sc for a in avg]
            apply_outer_grads(e.bank[key], avg)
            norms.append(math.sqrt(sum(float(a.pow(2).sum()) for a in avg)) if avg else 0.0)
        e.outer_opt.step()
        e.outer_opt.zero_grad(set_to_none=True)
        val = e._track_best(corpus, batch_size=self._last_batch_size) if corpus.has_validation else None
        losses = acc.per_path_loss
        return RoundMetrics(round=generation,
                            inner_loss=sum(losses.values()) / len(losses) if losses else float("nan"),
                            per_path_loss=dict(losses),
                            delta_norm=sum(norms) / len(norms) if norms else 0.0, val_loss=val)

    def _apply_generation(self, corpus, contributions, generation) -> RoundMetrics:
        acc = self._new_accumulator()
        for c in sorted(contributions, key=lambda c: c.path_idx):
            self._fold_contribution(acc, corpus, c)
        return self._finalize_outer_step(acc, corpus, generation)

    # -- drive ---------------------------------------------------------------
    def run_generation(self, corpus, batch_size, generation, *, fault_hook=None) -> RoundMetrics:
        self._last_batch_size = batch_size
        paths = list(self.engine.topology.paths())
        gen = _Generation(paths, self.lease_timeout, self.max_attempts,
                          max(1, math.ceil(self.min_fraction * len(paths))))
        threads = [threading.Thread(target=self._worker, args=(gen, corpus, batch_size, generation, fault_hook),
                                    daemon=True) for _ in range(self.num_workers)]
        mon = threading.Thread(target=self._monitor, args=(gen,), daemon=True)
        for t in threads:
            t.start()
        mon.start()
        for t in threads:
            t.join()
        mon.join()
        self.dropped = set(gen.failed)
        return self._apply_generation(corpus, list(gen.results.values()), generation)

    def fit(self, corpus, num_generations: int, batch_size: int, *, total_generations: int | None = None,
            log_every: int = 1, fault_hook=None):
        e = self.engine
        if total_generations is not None:
            e.total_rounds = total_generations
        elif e.total_rounds is None:
            e.total_rounds = e._global_round + num_generations
        hist = []
        for i in range(num_generations):
            m = self.run_generation(corpus, batch_size, e._global_round, fault_hook=fault_hook)
            e._global_round += 1
            hist.append(m)
            if log_every and (m.round % log_every == 0 or i == num_generations - 1):
                drop = f" dropped={len(self.dropped)}" if self.dropped else ""
                print(f"[gen {m.round:4d}] inner_loss={m.inner_loss:.4f} delta_norm={m.delta_norm:.4f}{drop}")
        return hist
