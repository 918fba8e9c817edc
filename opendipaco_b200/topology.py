"""Path / module topology: which modules a path runs through and who shares them.

A DiPaCo model is an ordered list of segments: token embedding, body block groups,
head. A body segment with ``num_experts > 1`` is a *routing level* (a path picks
one expert); every other segment is either SHARED (one instance averaged over all
paths) or PRIVATE (one copy per path, never communicated). A *path* is the tuple of
expert choices over the routing levels.

Module-key grammar (part of the checkpoint format, so it is kept verbatim from
the reference, ``src/opendipaco/topology.py:18-23``)::

    "embed" / "embed.p{i}"   shared / private embedding
    "head"  / "head.p{i}"    shared / private head
    "L{j}E{e}"               expert e of routing level j
    "B{s}"  / "B{s}.p{i}"    shared / private body block at segment s

Besides the reference API this module emits a *sharing table*
(:meth:`PathTopology.sharing_table`): for every shared key the sorted list of
path indices through it, which the device outer-step planner turns into per-GPU
reduction groups.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from itertools import product
from math import prod

Path = tuple[int, ...]


class Sharing(str, Enum):
    SHARED = "shared"
    PRIVATE = "private"


@dataclass(frozen=True)
class Segment:
    """One position along a path (reference: ``src/opendipaco/topology.py:42-53``)."""

    role: str                 # "embed" | "body" | "head"
    layers: int = 0
    num_experts: int = 1
    sharing: Sharing = Sharing.SHARED

    @property
    def is_routing(self) -> bool:
        return self.num_experts > 1


def embed_key() -> str:
    return "embed"


def head_key() -> str:
    return "head"


def expert_key(level: int, expert: int) -> str:
    return f"L{level}E{expert}"


def is_private_key(key: str) -> bool:
    return ".p" in key


def _parse_expert(key: str) -> tuple[int, int]:
    lvl, exp = key[1:].split("E")
    return int(lvl), int(exp)


def _is_expert(key: str) -> bool:
    return key.startswith("L") and "E" in key


class PathTopology:
    """Enumerates paths and the sharing structure they induce.

    ``PathTopology(level_sizes)`` builds the all-shared topology; ``segments=``
    gives full control. Behaviour mirrors ``src/opendipaco/topology.py:72-221``.
    """

    def __init__(
        self,
        level_sizes: tuple[int, ...] | None = None,
        share_embedding: bool = True,
        share_head: bool = True,
        *,
        segments: list[Segment] | None = None,
        layers_per_level: tuple[int, ...] | None = None,
        embedding: str = "shared",
        head: str = "shared",
    ):
        if segments is None:
            if level_sizes is None:
                raise ValueError("provide either level_sizes or segments")
            sizes = tuple(level_sizes)
            lpl = tuple(layers_per_level) if layers_per_level is not None else (1,) * len(sizes)
            emb = Sharing(embedding) if share_embedding else Sharing.PRIVATE
            hd = Sharing(head) if share_head else Sharing.PRIVATE
            segments = [Segment("embed", 0, 1, emb)]
            segments += [Segment("body", n, k, Sharing.SHARED) for k, n in zip(sizes, lpl)]
            segments.append(Segment("head", 0, 1, hd))
        self.segments: tuple[Segment, ...] = tuple(segments)
        self.routing_indices = [i for i, s in enumerate(self.segments) if s.is_routing]
        self.level_sizes = tuple(self.segments[i].num_experts for i in self.routing_indices)
        self._offset: dict[int, int] = {}
        running = 0
        for i, s in enumerate(self.segments):
            self._offset[i] = running
            running += s.layers
        self.total_layers = running

    # counts ---------------------------------------------------------------
    @property
    def num_levels(self) -> int:
        return len(self.routing_indices)

    @property
    def num_paths(self) -> int:
        return prod(self.level_sizes) if self.level_sizes else 1

    # paths ----------------------------------------------------------------
    def paths(self) -> list[Path]:
        if not self.level_sizes:
            return [()]
        return [tuple(p) for p in product(*[range(k) for k in self.level_sizes])]

    def path_index(self, path: Path) -> int:
        """Mixed-radix index, most significant level first."""
        idx = 0
        for k, c in zip(self.level_sizes, path):
            idx = idx * k + c
        return idx

    def path_from_index(self, index: int) -> Path:
        digits = []
        for k in reversed(self.level_sizes):
            digits.append(index % k)
            index //= k
        return tuple(reversed(digits))

    # keys -----------------------------------------------------------------
    def _base_name(self, seg: int) -> str:
        role = self.segments[seg].role
        return role if role in ("embed", "head") else f"B{seg}"

    def _segment_key(self, seg: int, path: Path) -> str:
        s = self.segments[seg]
        if s.is_routing:
            lvl = self.routing_indices.index(seg)
            return expert_key(lvl, path[lvl])
        base = self._base_name(seg)
        if s.sharing == Sharing.PRIVATE:
            return f"{base}.p{self.path_index(path)}"
        return base

    def module_keys(self) -> list[str]:
        out: list[str] = []
        for i, s in enumerate(self.segments):
            if s.is_routing:
                lvl = self.routing_indices.index(i)
                out += [expert_key(lvl, e) for e in range(s.num_experts)]
            elif s.sharing == Sharing.SHARED:
                out.append(self._base_name(i))
            else:
                out += [f"{self._base_name(i)}.p{p}" for p in range(self.num_paths)]
        return out

    def path_module_keys(self, path: Path) -> list[str]:
        return [self._segment_key(i, path) for i in range(len(self.segments))]

    # sharing --------------------------------------------------------------
    def paths_through_module(self, key: str) -> list[Path]:
        if is_private_key(key):
            return [self.path_from_index(int(key.split(".p")[1]))]
        if _is_expert(key):
            lvl, e = _parse_expert(key)
            return [p for p in self.paths() if p[lvl] == e]
        return self.paths()

    def sharing_count(self, key: str) -> int:
        if is_private_key(key):
            return 1
        if _is_expert(key):
            lvl, _ = _parse_expert(key)
            return self.num_paths // self.level_sizes[lvl]
        return self.num_paths

    def sharing_table(self) -> dict[str, list[int]]:
        """Shared key -> sorted path indices through it (private keys omitted)."""
        return {
            k: sorted(self.path_index(p) for p in self.paths_through_module(k))
            for k in self.module_keys()
            if not is_private_key(k)
        }

    # construction info -----------------------------------------------------
    def _segment_index_of_key(self, key: str) -> int:
        base = key.split(".p")[0]
        if base in ("embed", "head"):
            return next(i for i, s in enumerate(self.segments) if s.role == base)
        if _is_expert(base):
            lvl, _ = _parse_expert(base)
            return self.routing_indices[lvl]
        return int(base[1:])

    def role_of_key(self, key: str) -> str:
        return self.segments[self._segment_index_of_key(key)].role

    def layers_of_key(self, key: str) -> int:
        return self.segments[self._segment_index_of_key(key)].layers

    def offset_of_key(self, key: str) -> int:
        return self._offset[self._segment_index_of_key(key)]
