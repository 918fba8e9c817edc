"""The DiPaCo training engine.

Public API of the reference engine (``src/opendipaco/train/loop.py:44-527``). One round
= one DiLoCo outer step:

1. every owned path takes ``inner_steps`` AdamW steps on its shard;
2. each shared module's pseudo-gradient ``global - local`` is weighted (alpha =
   shard token fraction, or 1, or 1/P) and summed over the sharing paths, locally
   and then across ranks through the backend;
3. optional normalisation and x sqrt(sharing count); outer SGD-Nesterov step;
4. new globals are copied back into every working copy.

Two executors implement a round behind one interface (``run_round``, ``path_model``,
``inner_state_dicts``, ``outer_state_dict``, ``load_states``, ``sync_bank_views``):

* :class:`ModuleExecutor` (CPU, or ``ExecOptions(fused=False)``) runs PyTorch
  modules + ``torch.optim`` with the reference's arithmetic, bit for bit on CPU; it is
  the numerical oracle;
* the *fused* executor (default on CUDA, ``opendipaco_b200/train/fused.py``) keeps
  every owned path's weights, grads and optimizer state in flat device buffers,
  runs all owned paths of a step in lock-step through the sm_100a kernels, captures
  a whole round's inner steps in one CUDA graph, and does the outer step in one
  fused kernel (or the NVLink kernel for multi-GPU groups).

Both draw batch indices on the CPU from the same engine generator in the same
order (path by path), so their RNG consumption, checkpoints and resume semantics
are identical.
"""

from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from ..config import DiLoCoConfig, DiPaCoConfig
from ..data.sharding import ShardedCorpus
from ..models.init import warm_start_modules
from ..models.path import build_module_bank, build_path_model
from ..optim.diloco import (
    apply_outer_grads, inner_lr_at, make_inner_optimizer, make_outer_optimizer, module_delta,
)
from ..parallel.backend.base import ReducedDelta, SyncBackend
from ..topology import Path, is_private_key


@dataclass
class RoundMetrics:
    round: int
    inner_loss: float
    per_path_loss: dict[Path, float] = field(default_factory=dict)
    delta_norm: float = 0.0
    val_loss: float | None = None


@dataclass
class ExecOptions:
    """B200 execution knobs (never part of the config fingerprint).

    ``fused``: None = fused executor on CUDA devices, module executor on CPU.
    ``cuda_graphs``: capture a round's inner steps in one CUDA graph.
    ``outer``: "auto" (fused device kernel; NVLink kernel across GPUs when the
    backend provides one), or "reduce" (generic ``backend.global_reduce`` path).
    """

    fused: bool | None = None
    cuda_graphs: bool = True
    outer: str = "auto"


def batch_indices(n: int, batch_size: int, steps: int, gen: torch.Generator) -> list[torch.Tensor]:
    """Row indices of ``steps`` batches: shuffled epochs without replacement, the
    tail of an epoch dropped, reshuffled at each epoch boundary (reference
    ``_iter_batches``, ``loop.py:52-69``; same generator calls in the same order)."""
    bs = min(batch_size, n)
    perm = torch.randperm(n, generator=gen)
    pos, out = 0, []
    for _ in range(steps):
        if pos + bs > n:
            perm = torch.randperm(n, generator=gen)
            pos = 0
        out.append(perm[pos:pos + bs])
        pos += bs
    return out


def _iter_batches(shard: torch.Tensor, batch_size: int, steps: int, gen: torch.Generator):
    for idx in batch_indices(shard.size(0), batch_size, steps, gen):
        yield shard[idx]


@torch.no_grad()
def _copy_into(dst: nn.Module, src: nn.Module) -> None:
    for d, s in zip(dst.parameters(), src.parameters()):
        d.data.copy_(s.data)


@torch.no_grad()
def token_loss_sum(model: nn.Module, sequences: torch.Tensor, *, batch_size: int, device,
                   ignore_index: int = -100) -> tuple[float, int]:
    """Summed next-token CE and scored-token count over ``sequences``."""
    total, tokens = 0.0, 0
    for i in range(0, sequences.size(0), batch_size):
        batch = sequences[i:i + batch_size].to(device)
        if batch.size(1) < 2:
            continue
        logits, _ = model(batch)
        pred, tgt = logits[:, :-1, :], batch[:, 1:]
        total += float(F.cross_entropy(pred.reshape(-1, pred.size(-1)).float(), tgt.reshape(-1),
                                       ignore_index=ignore_index, reduction="sum"))
        tokens += int((tgt != ignore_index).sum())
    return total, tokens


def _opt_state_cpu(state: dict) -> dict:
    return {"state": {i: {k: (v.detach().cpu() if torch.is_tensor(v) else v)
                          for k, v in e.items()} for i, e in state["state"].items()},
            "param_groups": state["param_groups"]}


def _state_cpu(sd: dict) -> dict:
    return {k: v.detach().cpu().clone() for k, v in sd.items()}


def config_fingerprint(config: DiPaCoConfig, diloco: DiLoCoConfig) -> str:
    return hashlib.sha256((repr(config) + "||" + repr(diloco)).encode()).hexdigest()[:16]


def run_inner_steps(pm, opt, shard, batch_size, gen, *, inner_steps, total_steps, base_step,
                    diloco, device):
    """One path's inner loop on the module executor; returns the last batch loss."""
    dtype = torch.device(device).type
    autocast_on = getattr(diloco, "inner_autocast", False)
    pm.train()
    pm.checkpoint = getattr(diloco, "activation_checkpoint", False)
    pm.loss_chunks = getattr(diloco, "loss_chunks", 1)
    last = 0.0
    for i, batch in enumerate(_iter_batches(shard, batch_size, inner_steps, gen)):
        for g in opt.param_groups:
            g["lr"] = inner_lr_at(base_step + i, total_steps, diloco)
        batch = batch.to(device)
        opt.zero_grad(set_to_none=True)
        with torch.autocast(device_type=dtype, dtype=torch.bfloat16, enabled=autocast_on):
            _, loss = pm(batch, labels=batch)
        loss = loss.float()
        loss.backward()
        if diloco.inner_grad_clip is not None:
            nn.utils.clip_grad_norm_(pm.parameters(), diloco.inner_grad_clip)
        opt.step()
        last = float(loss.detach())
    return last


class _WeightedDeltas:
    """Per shared key: sum over the paths of ``w * (global - local)`` and the weight sum,
    accumulated in path order."""

    def __init__(self, bank: dict, keys: list[str]):
        self.keys = keys
        self.sums = {k: [torch.zeros_like(p) for p in bank[k].parameters()] for k in keys}
        self.weights = dict.fromkeys(keys, 0.0)

    def add(self, key: str, w: float, deltas) -> None:
        for acc, d in zip(self.sums[key], deltas):
            acc.add_(w * d)
        self.weights[key] += w


class ModuleExecutor:
    """Rounds on PyTorch modules: the reference's training arithmetic (the oracle).

    ``materialize="eager"`` keeps one working model and inner optimizer per owned path;
    ``"serial"`` builds each path's model from the bank when it trains and keeps only its
    optimizer state between rounds (``engine._opt_state``), so memory holds one path.
    """

    def __init__(self, engine: "DiPaCoEngine"):
        self.e = engine
        self.models: dict[Path, nn.Module] = {}
        self.opts: dict[Path, torch.optim.Optimizer] = {}
        if engine.materialize == "eager":
            for path in engine.backend.owned_paths():
                self.models[path], self.opts[path] = self._fresh(path)

    def _fresh(self, path: Path):
        e = self.e
        model = build_path_model(e.config, path, e.bank, deepcopy=True).to(e.device)
        return model, make_inner_optimizer(model, e.diloco)

    def _checkout(self, path: Path):
        if path in self.models:
            return self.models[path], self.opts[path]
        model, opt = self._fresh(path)
        if path in self.e._opt_state:
            opt.load_state_dict(self.e._opt_state[path])
        return model, opt

    def _checkin(self, path: Path, opt) -> None:
        if path not in self.opts:  # serial: only the optimizer state outlives the round
            self.e._opt_state[path] = _opt_state_cpu(opt.state_dict())

    def path_model(self, path: Path) -> nn.Module:
        return self.models[path] if path in self.models else self._fresh(path)[0]

    def _train(self, path: Path, corpus, batch_size: int, round_idx: int, sums: _WeightedDeltas):
        """Inner steps of one path, then its contribution; returns its last loss (None
        for an empty shard)."""
        e = self.e
        pidx = e.topology.path_index(path)
        shard = corpus.shard(pidx).to(e.device)
        if shard.size(0) == 0:
            return None
        model, opt = self._checkout(path)
        steps = e.diloco.inner_steps
        loss = run_inner_steps(model, opt, shard, batch_size, e._gen, inner_steps=steps,
                               total_steps=e.total_rounds * steps if e.total_rounds else None,
                               base_step=round_idx * steps, diloco=e.diloco, device=e.device)
        for key, local in model.modules_by_key().items():
            if not e.backend.owns_module(key):
                continue
            if is_private_key(key):
                _copy_into(e.bank[key], local)
            else:
                sums.add(key, e._outer_weight(key, pidx, corpus), module_delta(e.bank[key], local))
        self._checkin(path, opt)
        return loss

    def _outer_step(self, sums: _WeightedDeltas) -> list[float]:
        e = self.e
        norms = []
        for key in sums.keys:
            red = e.backend.global_reduce(key, ReducedDelta(sums.sums[key], sums.weights[key]))
            grads = ([t / max(red.weight, 1e-12) for t in red.summed] if e.diloco.normalize_outer_delta
                     else list(red.summed))
            if e.diloco.rescale_by_sqrt_sharing:
                scale = math.sqrt(e.topology.sharing_count(key))
                grads = [g * scale for g in grads]
            apply_outer_grads(e.bank[key], grads)
            norms.append(math.sqrt(sum(float(g.pow(2).sum()) for g in grads)) if grads else 0.0)
        e.outer_opt.step()
        e.outer_opt.zero_grad(set_to_none=True)
        return norms

    def run_round(self, corpus, batch_size: int, round_idx: int, next_round=None):
        e = self.e
        shared = [k for k in e.topology.module_keys() if e.backend.owns_module(k) and not is_private_key(k)]
        sums = _WeightedDeltas(e.bank, shared)
        losses: dict[Path, float] = {}
        for path in e.backend.owned_paths():
            loss = self._train(path, corpus, batch_size, round_idx, sums)
            if loss is not None:
                losses[path] = loss
        norms = self._outer_step(sums)
        for model in self.models.values():  # eager working copies restart from the new globals
            for key, local in model.modules_by_key().items():
                if e.backend.owns_module(key) and not is_private_key(key):
                    _copy_into(local, e.bank[key])
        return losses, norms

    # -- checkpoint glue
    def sync_bank_views(self) -> None:
        pass

    def inner_state_dicts(self) -> dict:
        if self.opts:
            return {p: _opt_state_cpu(o.state_dict()) for p, o in self.opts.items()}
        return dict(self.e._opt_state)

    def outer_state_dict(self) -> dict:
        return _opt_state_cpu(self.e.outer_opt.state_dict())

    def load_states(self, outer_sd: dict, inner: dict) -> None:
        e = self.e
        e.outer_opt.load_state_dict(outer_sd)
        if e.materialize == "serial":
            e._opt_state = dict(inner)
            return
        for path in e.backend.owned_paths():
            model, opt = self._fresh(path)
            if path in inner:
                opt.load_state_dict(inner[path])
            self.models[path], self.opts[path] = model, opt


class DiPaCoEngine:
    """Backend-agnostic DiPaCo trainer (the reference engine's public API); the rounds
    run on a :class:`ModuleExecutor` or, on CUDA by default, a ``FusedExecutor``."""

    def __init__(self, config: DiPaCoConfig, diloco: DiLoCoConfig, backend: SyncBackend,
                 device: str | torch.device = "cpu", seed: int = 0,
                 init_from: str | nn.Module | None = None, materialize: str = "eager",
                 exec_options: ExecOptions | None = None):
        if materialize not in ("eager", "serial"):
            raise ValueError(f"materialize must be 'eager' or 'serial', got {materialize!r}")
        self.config, self.diloco, self.backend = config, diloco, backend
        self.device = torch.device(device)
        self.topology = backend.topology
        self.materialize = materialize
        self.exec = exec_options or ExecOptions()
        self._seed = seed
        self.total_rounds: int | None = None
        self._global_round = 0
        self._opt_state: dict[Path, dict] = {}  # serial materialization: inner states between rounds
        self.best_val_loss: dict[Path, float] = {}
        self.best_path_state: dict[Path, dict] = {}

        # module initialisation consumes the global RNG exactly as the reference does
        torch.manual_seed(seed)
        self.bank: dict[str, nn.Module] = {k: m.to(self.device) for k, m in build_module_bank(config).items()
                                           if backend.owns_module(k)}
        if init_from is not None:
            warm_start_modules(self.bank, self.topology, init_from)
        self.outer_opt = make_outer_optimizer({k: m for k, m in self.bank.items() if not is_private_key(k)}, diloco)

        use_fused = self.exec.fused if self.exec.fused is not None else self.device.type == "cuda"
        self._modules = None
        self._fused = None
        if use_fused:
            from .fused import FusedExecutor

            self._fused = FusedExecutor(self)
        else:
            self._modules = ModuleExecutor(self)
        self._gen = torch.Generator().manual_seed(seed + 1)

    @property
    def _executor(self):
        return self._fused if self._fused is not None else self._modules

    @property
    def fused(self) -> bool:
        return self._fused is not None

    @property
    def path_models(self) -> dict:
        """Persistent per-path working models (eager materialization)."""
        return self._modules.models if self._modules is not None else self._eager_views

    @property
    def _eager_views(self) -> dict:
        if not hasattr(self, "_fused_views"):
            self._fused_views = {}
        return self._fused_views

    @property
    def inner_opts(self) -> dict:
        return self._modules.opts if self._modules is not None else {}

    # -- outer weights -------------------------------------------------------------
    def _outer_weight(self, key: str, path_idx: int, corpus) -> float:
        """alpha of a path's pseudo-gradient for ``key``: its shard's token fraction, or
        1 (normalised later by the weight sum), or 1 / (paths sharing the key)."""
        if self.diloco.shard_size_weighting:
            return corpus.shard_weight(path_idx)
        return 1.0 if self.diloco.normalize_outer_delta else 1.0 / self.topology.sharing_count(key)

    def outer_scale(self, key: str) -> float:
        return math.sqrt(self.topology.sharing_count(key)) if self.diloco.rescale_by_sqrt_sharing else 1.0

    # -- rounds ------------------------------------------------------------------------
    def run_round(self, corpus: ShardedCorpus, batch_size: int, round_idx: int = 0,
                  _next_round: int | None = None) -> RoundMetrics:
        losses, norms = self._executor.run_round(corpus, batch_size, round_idx, _next_round)
        val = self._track_best(corpus, batch_size) if corpus.has_validation else None
        return RoundMetrics(round=round_idx, inner_loss=sum(losses.values()) / len(losses) if losses else float("nan"),
                            per_path_loss=losses, delta_norm=sum(norms) / len(norms) if norms else 0.0, val_loss=val)

    def fit(self, corpus: ShardedCorpus, num_rounds: int, batch_size: int, log_every: int = 1,
            total_rounds: int | None = None):
        if total_rounds is not None:
            self.total_rounds = total_rounds
        elif self.total_rounds is None:
            self.total_rounds = self._global_round + num_rounds
        history = []
        for i in range(num_rounds):
            # the fused executor samples the next round's batches while this one runs on
            # the GPU, when that round is certain to follow (no validation pass between)
            ahead = self._global_round + 1 if i + 1 < num_rounds and not corpus.has_validation else None
            m = self.run_round(corpus, batch_size, round_idx=self._global_round, _next_round=ahead)
            self._global_round += 1
            history.append(m)
            if log_every and (m.round % log_every == 0 or i == num_rounds - 1):
                print(f"[round {m.round:4d}] inner_loss={m.inner_loss:.4f} delta_norm={m.delta_norm:.4f}")
        return history

    # -- validation / best-path tracking -------------------------------------------
    def _val_loss(self, model: nn.Module, seqs: torch.Tensor, batch_size: int) -> float:
        model.eval()
        total, tokens = token_loss_sum(model, seqs, batch_size=batch_size, device=self.device)
        model.train()
        return total / max(tokens, 1)

    def _track_best(self, corpus, batch_size: int) -> float | None:
        """Validation loss of every owned path with a validation shard; a path's best
        state so far is kept for :meth:`compose_best`."""
        seen = []
        for path in self.backend.owned_paths():
            val = corpus.val_shard(self.topology.path_index(path))
            if val is None or val.size(0) == 0:
                continue
            model = self._executor.path_model(path)
            loss = self._val_loss(model, val, batch_size)
            seen.append(loss)
            if loss < self.best_val_loss.get(path, math.inf):
                self.best_val_loss[path] = loss
                self.best_path_state[path] = _state_cpu(model.state_dict())
        return sum(seen) / len(seen) if seen else None

    def compose_best(self, path: Path) -> nn.Module:
        model = build_path_model(self.config, path, self.bank, deepcopy=True).to(self.device)
        if path in self.best_path_state:
            model.load_state_dict(self.best_path_state[path])
        return model

    def global_modules(self) -> dict[str, nn.Module]:
        self._executor.sync_bank_views()
        return self.bank

    # -- checkpoint ------------------------------------------------------------------
    def _world_size(self) -> int:
        return len({self.backend.rank_of_path(p) for p in self.topology.paths()})

    def state_dict(self) -> dict:
        """The checkpoint payload (layout shared with the reference, so checkpoints load
        in either framework)."""
        ex = self._executor
        ex.sync_bank_views()
        return {
            "format": 1,
            "fingerprint": config_fingerprint(self.config, self.diloco),
            "world_size": self._world_size(),
            "materialize": self.materialize,
            "bank": {k: _state_cpu(m.state_dict()) for k, m in self.bank.items()},
            "outer_opt": ex.outer_state_dict(),
            "inner_opt_state": ex.inner_state_dicts(),
            "global_round": self._global_round,
            "total_rounds": self.total_rounds,
            "best_val_loss": dict(self.best_val_loss),
            "best_path_state": {p: _state_cpu(sd) for p, sd in self.best_path_state.items()},
            "gen_state": self._gen.get_state(),
            "torch_rng_state": torch.get_rng_state(),
        }

    def load_state_dict(self, state: dict, *, strict: bool = True) -> None:
        if strict:
            mine = config_fingerprint(self.config, self.diloco)
            if state.get("fingerprint") != mine:
                raise ValueError("checkpoint config fingerprint does not match this engine "
                                 f"({state.get('fingerprint')} != {mine}); pass strict=False to override")
            if state.get("world_size") != self._world_size():
                raise ValueError("checkpoint world_size does not match this engine "
                                 f"({state.get('world_size')} != {self._world_size()})")
        for key, sd in state["bank"].items():
            self.bank[key].load_state_dict({k: v.to(self.device) for k, v in sd.items()})
        self._global_round, self.total_rounds = state["global_round"], state["total_rounds"]
        self.best_val_loss = dict(state["best_val_loss"])
        self.best_path_state = {p: dict(sd) for p, sd in state["best_path_state"].items()}
        self._gen.set_state(state["gen_state"])
        torch.set_rng_state(state["torch_rng_state"])
        self._executor.load_states(state["outer_opt"], state["inner_opt_state"])
