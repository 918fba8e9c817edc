"""The DiPaCo training engine.

Reference: ``src/opendipaco/train/loop.py:44-527``. One round = one DiLoCo outer
step:

1. every owned path takes ``inner_steps`` AdamW steps on its shard;
2. each shared module's pseudo-gradient ``global - local`` is weighted (alpha =
   shard token fraction, or 1, or 1/P) and summed over the sharing paths, locally
   and then across ranks through the backend;
3. optional normalisation and x sqrt(sharing count); outer SGD-Nesterov step;
4. new globals are copied back into every working copy.

Two executors implement a round:

* the *module* executor (CPU, or ``ExecOptions(fused=False)``) runs PyTorch
  modules + ``torch.optim`` exactly like the reference; it is the oracle;
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


class DiPaCoEngine:
    """Backend-agnostic DiPaCo trainer (public API of the reference engine)."""

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

        torch.manual_seed(seed)
        full = build_module_bank(config)
        self.bank: dict[str, nn.Module] = {
            k: m.to(self.device) for k, m in full.items() if backend.owns_module(k)}
        if init_from is not None:
            warm_start_modules(self.bank, self.topology, init_from)
        shared = {k: m for k, m in self.bank.items() if not is_private_key(k)}
        self.outer_opt = make_outer_optimizer(shared, diloco)

        self.path_models: dict[Path, nn.Module] = {}
        self.inner_opts: dict[Path, torch.optim.Optimizer] = {}
        self._opt_state: dict[Path, dict] = {}
        self._fused = None
        use_fused = self.exec.fused if self.exec.fused is not None else self.device.type == "cuda"
        if use_fused:
            from .fused import FusedExecutor

            self._fused = FusedExecutor(self)
        elif materialize == "eager":
            for path in backend.owned_paths():
                pm = build_path_model(config, path, self.bank, deepcopy=True).to(self.device)
                self.path_models[path] = pm
                self.inner_opts[path] = make_inner_optimizer(pm, diloco)

        self._gen = torch.Generator().manual_seed(seed + 1)
        self.best_val_loss: dict[Path, float] = {}
        self.best_path_state: dict[Path, dict] = {}

    @property
    def fused(self) -> bool:
        return self._fused is not None

    # -- weights ------------------------------------------------------------
    def _outer_weight(self, key: str, path_idx: int, corpus) -> float:
        if self.diloco.shard_size_weighting:
            return corpus.shard_weight(path_idx)
        if self.diloco.normalize_outer_delta:
            return 1.0
        return 1.0 / self.topology.sharing_count(key)

    def outer_scale(self, key: str) -> float:
        return math.sqrt(self.topology.sharing_count(key)) if self.diloco.rescale_by_sqrt_sharing else 1.0

    # -- module-executor materialisation ----------------------------------------
    def _acquire(self, path: Path):
        if self.materialize == "eager":
            return self.path_models[path], self.inner_opts[path]
        pm = build_path_model(self.config, path, self.bank, deepcopy=True).to(self.device)
        opt = make_inner_optimizer(pm, self.diloco)
        if path in self._opt_state:
            opt.load_state_dict(self._opt_state[path])
        return pm, opt

    def _release(self, path: Path, opt) -> None:
        if self.materialize == "serial":
            self._opt_state[path] = _opt_state_cpu(opt.state_dict())

    def _path_model_for(self, path: Path) -> nn.Module:
        if self._fused is not None:
            return self._fused.path_model(path)
        if self.materialize == "eager":
            return self.path_models[path]
        return build_path_model(self.config, path, self.bank, deepcopy=True).to(self.device)

    def _inner_train(self, pm, opt, shard, batch_size, round_idx) -> float:
        steps = self.diloco.inner_steps
        total = self.total_rounds * steps if self.total_rounds else None
        return run_inner_steps(pm, opt, shard, batch_size, self._gen, inner_steps=steps,
                               total_steps=total, base_step=round_idx * steps,
                               diloco=self.diloco, device=self.device)

    # -- one round ------------------------------------------------------------
    def run_round(self, corpus: ShardedCorpus, batch_size: int, round_idx: int = 0,
                  _next_round: int | None = None) -> RoundMetrics:
        if self._fused is not None:
            per_path_loss, delta_norms = self._fused.run_round(corpus, batch_size, round_idx, _next_round)
        else:
            per_path_loss, delta_norms = self._module_round(corpus, batch_size, round_idx)
        val = self._track_best(corpus, batch_size) if corpus.has_validation else None
        mean = sum(per_path_loss.values()) / len(per_path_loss) if per_path_loss else float("nan")
        return RoundMetrics(round=round_idx, inner_loss=mean, per_path_loss=per_path_loss,
                            delta_norm=sum(delta_norms) / len(delta_norms) if delta_norms else 0.0,
                            val_loss=val)

    def _module_round(self, corpus, batch_size, round_idx):
        owned = [k for k in self.topology.module_keys() if self.backend.owns_module(k)]
        shared = [k for k in owned if not is_private_key(k)]
        acc = {k: [torch.zeros_like(p) for p in self.bank[k].parameters()] for k in shared}
        acc_w = dict.fromkeys(shared, 0.0)
        losses: dict[Path, float] = {}
        for path in self.backend.owned_paths():
            pidx = self.topology.path_index(path)
            shard = corpus.shard(pidx).to(self.device)
            if shard.size(0) == 0:
                continue
            pm, opt = self._acquire(path)
            losses[path] = self._inner_train(pm, opt, shard, batch_size, round_idx)
            for key, local in pm.modules_by_key().items():
                if not self.backend.owns_module(key):
                    continue
                if is_private_key(key):
                    _copy_into(self.bank[key], local)
                    continue
                w = self._outer_weight(key, pidx, corpus)
                for a, d in zip(acc[key], module_delta(self.bank[key], local)):
                    a.add_(w * d)
                acc_w[key] += w
            self._release(path, opt)
            if self.materialize == "serial":
                del pm, opt
        norms = []
        for key in shared:
            red = self.backend.global_reduce(key, ReducedDelta(acc[key], acc_w[key]))
            if self.diloco.normalize_outer_delta:
                den = max(red.weight, 1e-12)
                avg = [s / den for s in red.summed]
            else:
                avg = list(red.summed)
            if self.diloco.rescale_by_sqrt_sharing:
                sc = math.sqrt(self.topology.sharing_count(key))
                avg = [a * sc for a in avg]
            apply_outer_grads(self.bank[key], avg)
            norms.append(math.sqrt(sum(float(a.pow(2).sum()) for a in avg)) if avg else 0.0)
        self.outer_opt.step()
        self.outer_opt.zero_grad(set_to_none=True)
        if self.materialize == "eager":
            for pm in self.path_models.values():
                for key, local in pm.modules_by_key().items():
                    if self.backend.owns_module(key) and not is_private_key(key):
                        _copy_into(local, self.bank[key])
        return losses, norms

    # -- validation / early stopping -----------------------------------------------
    @torch.no_grad()
    def _eval_val(self, pm: nn.Module, seqs: torch.Tensor, batch_size: int) -> float:
        pm.eval()
        total, tokens = token_loss_sum(pm, seqs, batch_size=batch_size, device=self.device)
        pm.train()
        return total / max(tokens, 1)

    def _track_best(self, corpus, batch_size: int) -> float | None:
        losses = []
        for path in self.backend.owned_paths():
            val = corpus.val_shard(self.topology.path_index(path))
            if val is None or val.size(0) == 0:
                continue
            pm = self._path_model_for(path)
            loss = self._eval_val(pm, val, batch_size)
            losses.append(loss)
            if path not in self.best_val_loss or loss < self.best_val_loss[path]:
                self.best_val_loss[path] = loss
                self.best_path_state[path] = {k: v.detach().cpu().clone()
                                              for k, v in pm.state_dict().items()}
        return sum(losses) / len(losses) if losses else None

    def compose_best(self, path: Path) -> nn.Module:
        pm = build_path_model(self.config, path, self.bank, deepcopy=True).to(self.device)
        if path in self.best_path_state:
            pm.load_state_dict(self.best_path_state[path])
        return pm

    def fit(self, corpus: ShardedCorpus, num_rounds: int, batch_size: int, log_every: int = 1,
            total_rounds: int | None = None):
        if total_rounds is not None:
            self.total_rounds = total_rounds
        elif self.total_rounds is None:
            self.total_rounds = self._global_round + num_rounds
        hist = []
        for i in range(num_rounds):
            # the fused executor samples the next round's batches while this one runs on
            # the GPU, when that round is certain to follow (no validation pass in between)
            ahead = (self._global_round + 1 if i + 1 < num_rounds and not corpus.has_validation else None)
            m = self.run_round(corpus, batch_size, round_idx=self._global_round, _next_round=ahead)
            self._global_round += 1
            hist.append(m)
            if log_every and (m.round % log_every == 0 or i == num_rounds - 1):
                print(f"[round {m.round:4d}] inner_loss={m.inner_loss:.4f} "
                      f"delta_norm={m.delta_norm:.4f}")
        return hist

    def global_modules(self) -> dict[str, nn.Module]:
        if self._fused is not None:
            self._fused.sync_bank_views()
        return self.bank

    # -- checkpoint ----------------------------------------------------------
    def _gather_inner_state(self) -> dict[Path, dict]:
        if self._fused is not None:
            return self._fused.inner_state_dicts()
        if self.materialize == "eager":
            return {p: _opt_state_cpu(o.state_dict()) for p, o in self.inner_opts.items()}
        return dict(self._opt_state)

    def _world_size(self) -> int:
        return len({self.backend.rank_of_path(p) for p in self.topology.paths()})

    def state_dict(self) -> dict:
        if self._fused is not None:
            self._fused.sync_bank_views()
        return {
            "format": 1,
            "fingerprint": config_fingerprint(self.config, self.diloco),
            "world_size": self._world_size(),
            "materialize": self.materialize,
            "bank": {k: _state_cpu(m.state_dict()) for k, m in self.bank.items()},
            "outer_opt": (self._fused.outer_state_dict() if self._fused is not None
                          else _opt_state_cpu(self.outer_opt.state_dict())),
            "inner_opt_state": self._gather_inner_state(),
            "global_round": self._global_round,
            "total_rounds": self.total_rounds,
            "best_val_loss": dict(self.best_val_loss),
            "best_path_state": {p: _state_cpu(sd) for p, sd in self.best_path_state.items()},
            "gen_state": self._gen.get_state(),
            "torch_rng_state": torch.get_rng_state(),
        }

    def load_state_dict(self, state: dict, *, strict: bool = True) -> None:
        if strict:
            fp = config_fingerprint(self.config, self.diloco)
            if state.get("fingerprint") != fp:
                raise ValueError("checkpoint config fingerprint does not match this engine "
                                 f"({state.get('fingerprint')} != {fp}); pass strict=False to override")
            if state.get("world_size") != self._world_size():
                raise ValueError("checkpoint world_size does not match this engine "
                                 f"({state.get('world_size')} != {self._world_size()})")
        for key, sd in state["bank"].items():
            self.bank[key].load_state_dict({k: v.to(self.device) for k, v in sd.items()})
        self._global_round = state["global_round"]
        self.total_rounds = state["total_rounds"]
        self.best_val_loss = dict(state["best_val_loss"])
        self.best_path_state = {p: dict(sd) for p, sd in state["best_path_state"].items()}
        self._gen.set_state(state["gen_state"])
        torch.set_rng_state(state["torch_rng_state"])
        inner = state["inner_opt_state"]
        if self._fused is not None:
            self._fused.load_states(state["outer_opt"], inner)
            return
        self.outer_opt.load_state_dict(state["outer_opt"])
        if self.materialize == "serial":
            self._opt_state = dict(inner)
            return
        for path in self.backend.owned_paths():
            pm = build_path_model(self.config, path, self.bank, deepcopy=True).to(self.device)
            opt = make_inner_optimizer(pm, self.diloco)
            if path in inner:
                opt.load_state_dict(inner[path])
            self.path_models[path] = pm
            self.inner_opts[path] = opt
