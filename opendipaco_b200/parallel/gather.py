"""Rebuild the complete module bank on every rank (for routed eval / EM).

Reference ``src/opendipaco/distributed.py:21-46``: for every key (in module-key
order, so the collective sequence is identical on all ranks) broadcast each
parameter from the rank owning the key's lowest-index path.
"""

from __future__ import annotations

import torch
from torch import nn

from ..config import DiPaCoConfig
from ..models.path import build_module_bank


@torch.no_grad()
def gather_full_bank(backend, owned_bank: dict[str, nn.Module], config: DiPaCoConfig):
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return owned_bank
    topo = backend.topology
    device = next(next(iter(owned_bank.values())).parameters()).device
    full = {k: m.to(device) for k, m in build_module_bank(config).items()}
    me = dist.get_rank()
    for key in topo.module_keys():
        src = backend.rank_of_path(min(topo.paths_through_module(key), key=topo.path_index))
        if me == src:
            for f, o in zip(full[key].parameters(), owned_bank[key].parameters()):
                f.data.copy_(o.data)
        for p in full[key].parameters():
            dist.broadcast(p.data, src=src)
    return full
