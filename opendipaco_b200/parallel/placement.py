"""Path -> rank placement.

The reference's ``TorchDistBackend`` gives rank r the contiguous block
``[r*P/W, (r+1)*P/W)`` and refuses ``P % W != 0`` (``src/opendipaco/backend/
torch_dist.py:31-45``). Here blocks are contiguous and balanced for any P >= W:
the first ``P % W`` ranks take one extra path (36 paths over 8 GPUs -> 5,5,5,5,4,4,
4,4). For divisible counts this is exactly the reference placement.
"""

from __future__ import annotations


def block_sizes(num_paths: int, world: int) -> list[int]:
    if world < 1 or num_paths < world:
        raise ValueError(f"need at least one path per rank (paths={num_paths}, world={world})")
    base, extra = divmod(num_paths, world)
    return [base + (1 if r < extra else 0) for r in range(world)]


def path_ranks(num_paths: int, world: int) -> list[int]:
    """rank of each path index."""
    out = []
    for r, n in enumerate(block_sizes(num_paths, world)):
        out += [r] * n
    return out


def rank_paths(num_paths: int, world: int, rank: int) -> list[int]:
    sizes = block_sizes(num_paths, world)
    start = sum(sizes[:rank])
    return list(range(start, start + sizes[rank]))
