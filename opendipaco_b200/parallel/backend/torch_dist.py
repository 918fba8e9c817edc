"""NCCL / gloo backend over ``torch.distributed`` subgroups (the baseline).

Reference ``src/opendipaco/backend/torch_dist.py:24-77``: one process group per
module key (built in the same order on every rank), ``all_reduce(SUM)`` of every
tensor of the key's summed delta plus a 1-element weight. Differences here:

* placement accepts any ``num_paths >= world`` (balanced contiguous blocks);
* the per-key tensors are flattened into ONE buffer before the all-reduce (one
  NCCL call per key instead of one per parameter), and the weight rides in the
  same buffer, so there is no extra scalar collective and no ``.item()`` per key
  beyond the final one;
* ``dp > 1`` (intra-path data parallelism, no counterpart in the reference): ranks
  form groups of ``dp`` consecutive ranks, paths are placed over groups, and every
  member of a group holds the group's paths. A path's ranks are all its group's
  members; only the first member of a group contributes to the outer reduction (the
  members hold identical pseudo-gradients).

The device outer step of the B200 engine does not go through this class; it is
the NCCL baseline the fused NVLink kernel is compared against.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ...topology import Path, PathTopology
from ..placement import path_ranks, rank_paths
from .base import ReducedDelta, SyncBackend


class TorchDistBackend(SyncBackend):
    def __init__(self, topology: PathTopology, device: torch.device | None = None, dp: int = 1):
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed is not initialized; call "
                               "dist.init_process_group first")
        self.topology = topology
        self.world_size = dist.get_world_size()
        self.rank = dist.get_rank()
        if dp < 1 or self.world_size % dp:
            raise ValueError(f"data-parallel degree {dp} must divide the world size {self.world_size}")
        self.dp = dp
        self.dp_index = self.rank % dp
        ngroups, grp = self.world_size // dp, self.rank // dp
        self.dp_ranks = list(range(grp * dp, grp * dp + dp))
        self._path_group = path_ranks(topology.num_paths, ngroups)
        self._ranks = [g * dp for g in self._path_group]  # first member of each path's group
        self._paths = [topology.path_from_index(i) for i in rank_paths(topology.num_paths, ngroups, grp)]
        # one subgroup per data-parallel group (built in the same order on every rank)
        self.dp_group = None
        if dp > 1:
            for g in range(ngroups):
                pg = dist.new_group(ranks=list(range(g * dp, g * dp + dp)))
                if g == grp:
                    self.dp_group = pg
        if device is None:
            device = (torch.device(f"cuda:{self.rank % torch.cuda.device_count()}")
                      if torch.cuda.is_available() else torch.device("cpu"))
        self.device = torch.device(device)
        self._groups: dict[str, object] = {}
        self._member: dict[str, bool] = {}
        for key in topology.module_keys():
            ranks = self.sharing_ranks(key)
            self._groups[key] = dist.new_group(ranks=ranks)
            self._member[key] = self.rank in ranks

    def rank_of_path(self, path: Path) -> int:
        return self._ranks[self.topology.path_index(path)]

    def sharing_ranks(self, key: str) -> list[int]:
        """Sorted ranks holding >= 1 path through ``key`` (every member of its groups)."""
        out = set()
        for p in self.topology.paths_through_module(key):
            g = self._path_group[self.topology.path_index(p)]
            out.update(range(g * self.dp, g * self.dp + self.dp))
        return sorted(out)

    def dp_allreduce(self, t: torch.Tensor) -> None:
        """Sum ``t`` over this rank's data-parallel group (host-side, off the hot path)."""
        if self.dp > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.dp_group)

    def owned_paths(self) -> list[Path]:
        return list(self._paths)

    def owns_module(self, key: str) -> bool:
        return self._member.get(key, False)

    def process_group(self, key: str):
        return self._groups[key]

    def global_reduce(self, key: str, local: ReducedDelta) -> ReducedDelta:
        ts = [t.to(self.device) for t in local.summed]
        flat = torch.cat([t.reshape(-1).float() for t in ts]
                         + [torch.tensor([local.weight], device=self.device, dtype=torch.float32)])
        if self.dp_index:
            flat.zero_()  # the group's first member speaks for its identical replicas
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self._groups[key])
        out, off = [], 0
        for t in ts:
            out.append(flat[off:off + t.numel()].view_as(t).to(t.dtype))
            off += t.numel()
        return ReducedDelta(summed=out, weight=float(flat[-1].item()))

    def barrier(self) -> None:
        dist.barrier()

    # -- fused-executor outer step over NCCL (the in-framework baseline) -------------
    def outer_launch_count(self, ex) -> int:
        """Kernels of one outer step (the NCCL all-reduces are not counted)."""
        return 1 if getattr(ex, "acc_fused", False) else 2

    def fused_outer_step(self, ex, plan, first: bool) -> None:
        """Local partial (kernel, unless the last inner step's optimizer kernel already
        wrote it) -> NCCL all-reduce per key group -> apply (kernel).

        Every sharer applies the full Nesterov update redundantly, as the reference
        does after its per-key all-reduce.
        """
        from ...ops.outer import MODE_ACC, MODE_APPLY, MODE_OUTER

        fused = getattr(ex, "acc_fused", False)
        cache = getattr(self, "_nccl_plans", None)
        if cache is None or cache[0] != id(plan):
            for s in plan.segments:
                if s.mode == MODE_OUTER and s.delta is None:
                    s.delta = torch.zeros_like(s.glob)
            cache = (id(plan), None if fused else plan.with_mode(MODE_ACC), plan.with_mode(MODE_APPLY),
                     [s for s in plan.segments if s.mode == MODE_OUTER])
            self._nccl_plans = cache
        _, acc, apply, outer = cache
        if acc is not None:
            acc.run(0.0, 0.0, False, False)
        for s in outer:
            if self.dp_index:
                s.delta.zero_()
            dist.all_reduce(s.delta, op=dist.ReduceOp.SUM, group=self._groups[s.key])
        dl = ex.e.diloco
        apply.run(dl.outer_lr, dl.outer_momentum, dl.outer_nesterov, first, status=getattr(ex, "OUTER_STATUS", None))

    def delta_norms(self) -> dict[str, float]:
        apply = self._nccl_plans[2]
        return {k: v for k, v in apply.delta_norms().items()}
