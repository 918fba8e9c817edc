"""In-process, fault-tolerant generations of path tasks.

One *generation* trains every path once from the current global modules and then takes
one outer step from their pseudo-gradients. ``AsyncScheduler`` runs a generation on a
pool of worker threads that lease path tasks from a :class:`LeaseBoard`:

* a task whose worker raises :class:`TransientFault` is returned at once (re-queued);
* a worker that raises :class:`Preempt` vanishes with its lease; the lease expires after
  ``lease_timeout`` and the path is re-queued;
* a path that fails ``max_attempts`` times is dropped for the generation.

Each task samples its batches with its own generator seeded by :func:`task_seed`
(seed, path, generation) -- the reference's mixing constants, so a run reproduces
across the two frameworks -- and the :class:`DeltaReducer` folds the finished tasks in
path order, so the result depends on neither the worker count nor the pattern of
recovered failures. The outer step reuses the engine's weighting and outer optimizer.
Behaviour follows the reference's ``src/opendipaco/schedule/scheduler.py``.
"""

from __future__ import annotations

import enum
import math
import threading
import time
from collections import deque
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


def task_seed(seed: int, path_idx: int, generation: int) -> int:
    """Seed of a task's batch generator (the reference's hash, for cross-framework runs)."""
    return ((seed * 0x9E3779B1) ^ (path_idx * 0x85EBCA77) ^ (generation * 0xC2B2AE35)) & 0x7FFFFFFFFFFFFFFF


@dataclass
class Contribution:
    """What one finished path task hands back."""

    path: Path
    path_idx: int
    loss: float
    shared_delta: dict[str, list[torch.Tensor]]  # module key -> pseudo-gradient per parameter
    private_state: dict[str, dict]                # private module key -> its new state dict
    opt_state: dict                               # the path's inner-optimizer state
    empty: bool = False                           # the path had no data this generation
    probe_before: float | None = None
    probe_after: float | None = None


# ---------------------------------------------------------------------- leases
class _State(enum.Enum):
    PENDING = 0
    LEASED = 1
    DONE = 2
    FAILED = 3


@dataclass
class _Task:
    state: _State = _State.PENDING
    attempts: int = 0
    deadline: float = 0.0
    result: Contribution | None = None


class LeaseBoard:
    """Per-path task states of one generation behind one condition variable. Pending
    paths are handed out first-in first-out; a returned or expired task goes to the back
    of the queue unless it used up its attempts."""

    def __init__(self, paths, lease_timeout: float, max_attempts: int):
        self.lease_timeout, self.max_attempts = lease_timeout, max_attempts
        self.tasks = {p: _Task() for p in paths}
        self.queue: deque = deque(paths)
        self.reclaimed = 0
        self._cv = threading.Condition()

    # -- transitions (caller holds the lock)
    def _requeue(self, path: Path) -> None:
        t = self.tasks[path]
        if t.attempts >= self.max_attempts:
            t.state = _State.FAILED
        else:
            t.state = _State.PENDING
            self.queue.append(path)

    def _sweep(self) -> None:
        now = time.monotonic()
        for path, t in self.tasks.items():
            if t.state is _State.LEASED and now >= t.deadline:
                if t.attempts < self.max_attempts:
                    self.reclaimed += 1
                self._requeue(path)

    def _settled(self) -> bool:
        return all(t.state in (_State.DONE, _State.FAILED) for t in self.tasks.values())

    def _hand_out(self, path: Path) -> tuple[Path, int]:
        t = self.tasks[path]
        t.state, t.attempts = _State.LEASED, t.attempts + 1
        t.deadline = time.monotonic() + self.lease_timeout
        return path, t.attempts

    # -- API
    def lease(self, wait: float = 0.05):
        """Block until a task is available: ``(path, attempt)``; None once every task is
        settled (done or failed)."""
        with self._cv:
            while True:
                self._sweep()
                if self._settled():
                    return None
                if self.queue:
                    return self._hand_out(self.queue.popleft())
                self._cv.wait(wait)

    def poll_lease(self, pick=None):
        """Non-blocking lease: ``(path, attempt)``, ``"done"`` or ``"idle"``. ``pick`` may
        choose among the pending paths (e.g. one whose data the worker holds)."""
        with self._cv:
            self._sweep()
            if self._settled():
                return "done"
            if not self.queue:
                return "idle"
            path = self.queue[0] if pick is None else pick(list(self.queue))
            if path is None:
                return "idle"
            self.queue.remove(path)
            return self._hand_out(path)

    def refresh_lease(self, path: Path) -> None:
        with self._cv:
            t = self.tasks[path]
            if t.state is _State.LEASED:
                t.deadline = time.monotonic() + self.lease_timeout

    def complete(self, path: Path, contrib: Contribution) -> None:
        """Record a result (the first one wins, even from a lease that had expired)."""
        with self._cv:
            t = self.tasks[path]
            if t.state is _State.DONE:
                return
            if t.state is _State.PENDING and path in self.queue:
                self.queue.remove(path)
            t.state, t.result = _State.DONE, contrib
            self._cv.notify_all()

    def nack(self, path: Path) -> None:
        with self._cv:
            t = self.tasks[path]
            if t.state is _State.LEASED:
                self._requeue(path)
            self._cv.notify_all()

    def reclaim(self) -> None:
        with self._cv:
            self._sweep()
            self._cv.notify_all()

    def is_done(self) -> bool:
        with self._cv:
            return self._settled()

    def pending_paths(self) -> list:
        with self._cv:
            self._sweep()
            return list(self.queue)

    @property
    def results(self) -> dict:
        with self._cv:
            return {p: t.result for p, t in self.tasks.items() if t.state is _State.DONE}

    @property
    def failed(self) -> set:
        with self._cv:
            return {p for p, t in self.tasks.items() if t.state is _State.FAILED}


# ---------------------------------------------------------------------- reduce
class DeltaReducer:
    """Weighted sum of the pseudo-gradients of one generation per shared key, then one
    outer step (normalised by the weight sum, optionally times sqrt(sharing))."""

    def __init__(self, engine: DiPaCoEngine, corpus):
        self.e, self.corpus = engine, corpus
        keys = [k for k in engine.topology.module_keys() if not is_private_key(k) and k in engine.bank]
        self.sums = {k: [torch.zeros_like(p) for p in engine.bank[k].parameters()] for k in keys}
        self.weights = dict.fromkeys(keys, 0.0)
        self.losses: dict = {}

    def add(self, c: Contribution, *, persist_opt: bool = True) -> None:
        if c.empty:
            return
        e = self.e
        self.losses[c.path] = c.loss
        for key, sd in c.private_state.items():
            e.bank[key].load_state_dict({n: v.to(e.device) for n, v in sd.items()})
        for key, delta in c.shared_delta.items():
            w = e._outer_weight(key, c.path_idx, self.corpus)
            for acc, d in zip(self.sums[key], delta):
                acc.add_(w * d.to(e.device))
            self.weights[key] += w
        if persist_opt and c.opt_state:
            e._opt_state[c.path] = c.opt_state

    def step(self, generation: int, batch_size: int) -> RoundMetrics:
        e = self.e
        norms = []
        for key, w in self.weights.items():
            if w == 0.0:
                continue
            scale = 1.0 / max(w, 1e-12) if e.diloco.normalize_outer_delta else 1.0
            if e.diloco.rescale_by_sqrt_sharing:
                scale *= math.sqrt(e.topology.sharing_count(key))
            grads = [s * scale for s in self.sums[key]]
            apply_outer_grads(e.bank[key], grads)
            norms.append(math.sqrt(sum(float(g.pow(2).sum()) for g in grads)))
        e.outer_opt.step()
        e.outer_opt.zero_grad(set_to_none=True)
        val = e._track_best(self.corpus, batch_size=batch_size) if self.corpus.has_validation else None
        mean = sum(self.losses.values()) / len(self.losses) if self.losses else float("nan")
        return RoundMetrics(round=generation, inner_loss=mean, per_path_loss=dict(self.losses),
                            delta_norm=sum(norms) / len(norms) if norms else 0.0, val_loss=val)


# ---------------------------------------------------------------------- scheduler
class AsyncScheduler:
    """Drives a :class:`DiPaCoEngine` (use ``materialize="serial"``) through generations
    of leased path tasks; ``_train_path`` is also the task body of the TCP workers."""

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

    # -- one task
    def _train_path(self, path: Path, shard: torch.Tensor, batch_size: int, generation: int,
                    inner_steps: int | None = None, probe=None) -> Contribution:
        """Train one path task from the current global modules. On CUDA the task runs on
        the fused B200 kernels (``train/worker_trainer.py``: one CUDA graph per task, no
        host sync per step); otherwise, or when the shape is not supported, on PyTorch
        modules with the reference's arithmetic. Both draw the same batches."""
        e = self.engine
        pidx = e.topology.path_index(path)
        if shard.size(0) == 0:
            return Contribution(path, pidx, float("nan"), {}, {}, {}, empty=True)
        steps = inner_steps or e.diloco.inner_steps
        gen = torch.Generator().manual_seed(task_seed(self.seed, pidx, generation))
        from ..train.worker_trainer import path_trainer_for

        trainer = path_trainer_for(e) if e.device.type == "cuda" else None
        if trainer is not None:
            screening = probe is not None and not probe.empty
            before = (safe_probe_loss(probe, build_path_model(e.config, path, e.bank, deepcopy=True).to(e.device))
                      if screening else None)
            loss, shared, private, opt_state = trainer.train(path, shard, batch_size, gen, steps, generation * steps)
            after = safe_probe_loss(probe, trainer.model_view(path)) if screening else None
            return Contribution(path, pidx, loss, shared, private, opt_state, probe_before=before, probe_after=after)
        shard = shard.to(e.device)
        model = build_path_model(e.config, path, e.bank, deepcopy=True,
                                 dedup_private=getattr(e.diloco, "dedup_private", False)).to(e.device)
        opt = make_inner_optimizer(model, e.diloco)
        if e._opt_state.get(path) is not None:
            opt.load_state_dict(e._opt_state[path])
        screening = probe is not None and not probe.empty
        before = safe_probe_loss(probe, model) if screening else None
        loss = run_inner_steps(model, opt, shard, batch_size, gen, inner_steps=steps, total_steps=e.total_rounds * steps if e.total_rounds else None,
                               base_step=generation * steps, diloco=e.diloco, device=e.device)
        after = safe_probe_loss(probe, model) if screening else None
        shared, private = {}, {}
        for key, mod in model.modules_by_key().items():
            if is_private_key(key):
                private[key] = _state_cpu(mod.state_dict())
            else:
                shared[key] = [d.detach().cpu() for d in module_delta(e.bank[key], mod)]
        return Contribution(path, pidx, loss, shared, private, _opt_state_cpu(opt.state_dict()),
                            probe_before=before, probe_after=after)

    def _work(self, board: LeaseBoard, corpus, batch_size: int, generation: int, fault_hook) -> None:
        while (leased := board.lease()) is not None:
            path, attempt = leased
            try:
                if fault_hook is not None:
                    fault_hook(path, attempt)
                shard = corpus.shard(self.engine.topology.path_index(path))
                board.complete(path, self._train_path(path, shard, batch_size, generation))
            except Preempt:
                continue  # the lease lapses; another worker picks the path up later
            except Exception as exc:
                self.errors[path] = repr(exc)
                board.nack(path)

    # -- generations
    def run_generation(self, corpus, batch_size, generation, *, fault_hook=None) -> RoundMetrics:
        self._last_batch_size = batch_size
        board = LeaseBoard(list(self.engine.topology.paths()), self.lease_timeout, self.max_attempts)
        workers = [threading.Thread(target=self._work, args=(board, corpus, batch_size, generation, fault_hook),
                                    name=f"odp-task-{i}", daemon=True) for i in range(self.num_workers)]
        for w in workers:
            w.start()
        for w in workers:
            w.join()
        self.dropped = board.failed
        reducer = DeltaReducer(self.engine, corpus)
        for c in sorted(board.results.values(), key=lambda c: c.path_idx):
            reducer.add(c)
        return reducer.step(generation, batch_size)

    def fit(self, corpus, num_generations: int, batch_size: int, *, total_generations: int | None = None,
            log_every: int = 1, fault_hook=None):
        e = self.engine
        if total_generations is not None:
            e.total_rounds = total_generations
        elif e.total_rounds is None:
            e.total_rounds = e._global_round + num_generations
        history = []
        for i in range(num_generations):
            m = self.run_generation(corpus, batch_size, e._global_round, fault_hook=fault_hook)
            e._global_round += 1
            history.append(m)
            if log_every and (m.round % log_every == 0 or i == num_generations - 1):
                dropped = f" dropped={len(self.dropped)}" if self.dropped else ""
                print(f"[gen {m.round:4d}] inner_loss={m.inner_loss:.4f} delta_norm={m.delta_norm:.4f}{dropped}")
        return history
