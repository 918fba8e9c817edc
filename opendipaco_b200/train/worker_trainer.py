"""One path task on the B200 kernels: the training body of asynchronous, sharded and
volunteer workers when their device is CUDA.

A task trains one path from the current global modules and hands back its
pseudo-gradients (global - local per shared module), its private modules and its
inner-optimizer state. :class:`FusedPathTrainer` keeps a one-path ``FusedExecutor`` per
worker (flat fp32 master / bf16 copy / AdamW arenas, every inner step of the task in one
CUDA graph, the grouped tcgen05 kernels) and reuses it for every task of the same shape:
the task's modules are copied into its arena, the path's AdamW state loaded from the
worker's store, and the task's batches sampled on the host with the task's own generator
(the same draws as the PyTorch module path, ``run_inner_steps``). The engine's bank is only
read. The reference's worker loop is ``src/opendipaco/schedule/scheduler.py:270-337``.
"""

from __future__ import annotations

import threading

import torch

from ..topology import Path, is_private_key
from .loop import ExecOptions


class _Solo:
    """The engine-like view a one-path FusedExecutor is built from (never rebinds the bank)."""

    solo = True
    materialize = "serial"

    class _Backend:
        dp = 1

        def __init__(self, topology, path):
            self.topology, self._path = topology, path

        def owned_paths(self):
            return [self._path]

    def __init__(self, engine, path: Path):
        self.config, self.diloco, self.device = engine.config, engine.diloco, engine.device
        self.topology, self.bank = engine.topology, engine.bank
        self.backend = self._Backend(engine.topology, path)
        self.exec = ExecOptions(fused=True, cuda_graphs=True)
        self.total_rounds = engine.total_rounds
        self.path_models: dict = {}
        self._gen = torch.Generator()


class FusedPathTrainer:
    """Trains path tasks of one engine on its CUDA device with the fused executor."""

    tasks_trained = 0  # tasks run by any trainer of this process (observability / tests)

    def __init__(self, engine):
        self.e = engine
        self._ex = None
        self._lock = threading.Lock()  # one task at a time on the device

    @staticmethod
    def supported(engine) -> bool:
        """The fused executor's constraints (bf16 tcgen05 kernels, head_dim 64, hidden a
        multiple of 128, untied embeddings, AdamW inner optimizer)."""
        cfg, bb = engine.config, engine.config.backbone
        return (engine.device.type == "cuda" and not cfg.tie_word_embeddings and bb.head_dim == 64
                and bb.hidden_size % 128 == 0 and not getattr(engine.diloco, "optim_8bit", False)
                and cfg.sequence_length % 64 == 0)

    def _executor(self, path: Path):
        if self._ex is None:
            from .fused import FusedExecutor

            self._ex = FusedExecutor(_Solo(self.e, path))
        return self._ex

    @torch.no_grad()
    def _load_modules(self, ex, path: Path) -> dict:
        """Copy the path's global modules into the arena; returns key -> (start, rel entries)."""
        regions = {}
        for key in self.e.topology.path_module_keys(path):
            start = ex._region(key)[0]
            rel = {n: (shape, off, k) for n, shape, off, k in ex._rel_entries(key)}
            for name, p in self.e.bank[key].named_parameters():
                shape, off, k = rel[name]
                ex.W32[0, start + off:start + off + k].copy_(p.detach().reshape(-1))
            regions[key] = (start, rel)
        ex.W16.copy_(ex.W32)
        return regions

    @torch.no_grad()
    def _load_opt_state(self, ex, path: Path) -> None:
        ex.MOM1.zero_()
        ex.MOM2.zero_()
        ex.steps_taken[0] = 0
        sd = self.e._opt_state.get(path)
        if not sd:
            return
        opt = ex._inner_opt(ex.paths[0])
        opt.load_state_dict(sd)
        for name, p in ex.pms[ex.paths[0]].named_parameters():
            st = opt.state.get(p)
            if not st:
                continue
            shape, off, n = ex.layout.by_name[name]
            step = st["step"]
            ex.steps_taken[0] = int(step.item() if torch.is_tensor(step) else step)
            ex.MOM1[0, off:off + n].copy_(st["exp_avg"].reshape(-1))
            ex.MOM2[0, off:off + n].copy_(st["exp_avg_sq"].reshape(-1))
        opt.state.clear()

    def train(self, path: Path, shard: torch.Tensor, batch_size: int, gen: torch.Generator, steps: int,
              base_step: int) -> tuple[float, dict, dict, dict]:
        """(last loss, shared deltas key -> [global - local per parameter], private states,
        inner-optimizer state) of one task."""
        with self._lock:
            ex = self._executor(path)
            ex.e.total_rounds = self.e.total_rounds
            regions = self._load_modules(ex, path)
            self._load_opt_state(ex, path)
            seq = shard.size(1)
            active = ex._prepare_rows([shard.cpu()], seq, batch_size, [gen], [base_step], steps, ex._slot)
            ex._upload(ex._slot)
            ex._run_inner(steps)
            if active[0]:
                ex.steps_taken[0] += steps
            ex.loss_host.copy_(ex.LOSSES[steps - 1], non_blocking=True)
            torch.cuda.current_stream(ex.dev).synchronize()
            from ..ops._ext import check_errors

            check_errors(ex.dev)
            loss = float(ex.loss_host[0])
            shared, private = {}, {}
            for key, (start, rel) in regions.items():
                local = {name: ex.W32[0, start + off:start + off + k].view(shape) for name, (shape, off, k) in
                         rel.items()}
                if is_private_key(key):
                    private[key] = {n: t.detach().cpu().clone() for n, t in local.items()}
                else:
                    shared[key] = [(p.detach() - local[name]).cpu() for name, p in
                                   self.e.bank[key].named_parameters()]
            opt_state = ex.inner_state_dicts()[ex.paths[0]]
            FusedPathTrainer.tasks_trained += 1
            return loss, shared, private, opt_state

    def model_view(self, path: Path) -> torch.nn.Module:
        """A module holding the trainer's current weights (for probes between steps)."""
        ex = self._executor(path)
        return ex.pms[ex.paths[0]]


def path_trainer_for(engine) -> FusedPathTrainer | None:
    """The engine's cached fused task trainer, or None when the module path must be used
    (not CUDA, an unsupported shape, or ``ODP_WORKER_FUSED=0``)."""
    import os

    if os.environ.get("ODP_WORKER_FUSED", "1") == "0" or not FusedPathTrainer.supported(engine):
        return None
    if getattr(engine, "_path_trainer", None) is None:
        engine._path_trainer = FusedPathTrainer(engine)
    return engine._path_trainer


__all__ = ["FusedPathTrainer", "path_trainer_for"]
