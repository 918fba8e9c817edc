"""Rebuild the complete module bank on every rank (for routed eval / EM).

Reference ``src/opendipaco/distributed.py:21-46``: for every key (in module-key order,
so the collective sequence is identical on all ranks) broadcast each parameter from the
rank owning the key's lowest-index path.

With the NVLink backend the bank already lives in symmetric (peer-addressable) arenas,
every key's region at the same offset on every rank. Then each rank PULLS what it lacks:
one launch of the peer-copy kernel reads every missing parameter straight from the
serving rank's arena over NVLink (plain loads, bracketed by two barriers), instead of
one NCCL broadcast per parameter. Inside a key's region the parameters sit in
``named_parameters`` order, each padded to a multiple of 256 elements (the fused
executor's layout).
"""

from __future__ import annotations

import torch
from torch import nn

from ..config import DiPaCoConfig
from ..models.path import build_module_bank

_PAD = 256


def _padded(n: int) -> int:
    return (n + _PAD - 1) // _PAD * _PAD


@torch.no_grad()
def gather_full_bank(backend, owned_bank: dict[str, nn.Module], config: DiPaCoConfig, method: str = "auto"):
    """Every module key on every rank (owned keys copied, the rest fetched). ``method``:
    "peer" (NVLink pull; needs the backend's arenas), "broadcast" (NCCL broadcast per
    parameter) or "auto" (peer when available)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return owned_bank
    if method not in ("auto", "peer", "broadcast"):
        raise ValueError(f"unknown gather method {method!r}")
    topo = backend.topology
    device = next(next(iter(owned_bank.values())).parameters()).device
    full = {k: m.to(device) for k, m in build_module_bank(config).items()}
    sources = backend.bank_sources() if method != "broadcast" and hasattr(backend, "bank_sources") else None
    if method == "peer" and sources is None:
        raise RuntimeError("peer gather needs a backend with peer-addressable bank arenas (NVLinkBackend after "
                           "its first round)")
    if sources is not None:
        return _pull(backend, owned_bank, full, sources)
    me = dist.get_rank()
    for key in topo.module_keys():
        src = backend.rank_of_path(min(topo.paths_through_module(key), key=topo.path_index))
        if me == src:
            for f, o in zip(full[key].parameters(), owned_bank[key].parameters()):
                f.data.copy_(o.data)
        for p in full[key].parameters():
            dist.broadcast(p.data, src=src)
    return full


def _pull(backend, owned_bank, full, sources):
    import torch.distributed as dist

    torch.cuda.synchronize(backend.dev)
    dist.barrier()  # every serving rank's arena holds its final weights
    segs = []
    for key, (addr, size) in sources.items():
        if key in owned_bank:
            for f, o in zip(full[key].parameters(), owned_bank[key].parameters()):
                f.data.copy_(o.data)
            continue
        rel = 0
        for p in full[key].parameters():
            segs.append((addr + 4 * rel, p.data_ptr(), p.numel()))
            rel += _padded(p.numel())
        if rel > _padded(size):
            raise RuntimeError(f"gather: parameter layout of {key} exceeds its arena region")
    backend.peer_copy(segs)
    torch.cuda.synchronize(backend.dev)
    dist.barrier()  # no rank changes its arena while another still reads it
    return full
