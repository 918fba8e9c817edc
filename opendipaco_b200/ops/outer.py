"""Fused DiLoCo outer step (``csrc/outer.cu``) driven by a segment table.

A *segment* is one shared module (its flat fp32 global buffer, momentum buffer,
pseudo-gradient buffer and the list of local working copies that share it on this GPU,
with their weights).
:class:`OuterPlan` packs the table once (device pointers are stable because every
buffer is a view into the executor's persistent flat arenas) and each round is one
kernel launch.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from ._ext import ext

SEG_DTYPE = np.dtype([("glob", "<u8"), ("mom", "<u8"), ("delta", "<u8"), ("n", "<i8"), ("first_local", "<i4"),
                      ("nlocal", "<i4"), ("mode", "<i4"), ("scale", "<f4"), ("inv_den", "<f4"),
                      ("pad", "<i4"), ("chunk0", "<i8")])
LOC_DTYPE = np.dtype([("w32", "<u8"), ("w16", "<u8"), ("weight", "<f4"), ("pad", "<i4")])
assert SEG_DTYPE.itemsize == 64 and LOC_DTYPE.itemsize == 24

MODE_OUTER, MODE_COPY, MODE_BCAST, MODE_ACC, MODE_APPLY = 0, 1, 2, 3, 4


@dataclass
class Segment:
    key: str
    glob: torch.Tensor                      # fp32 flat view
    mom: torch.Tensor | None                # fp32 flat view (None for COPY/BCAST)
    locals32: list[torch.Tensor]
    locals16: list[torch.Tensor | None]
    weights: list[float] = field(default_factory=list)
    mode: int = MODE_OUTER
    scale: float = 1.0
    inv_den: float = 1.0
    delta: torch.Tensor | None = None       # fp32 flat buffer for the ACC / APPLY phases


class OuterPlan:
    def __init__(self, segments: list[Segment], device):
        self.segments = segments
        self.device = torch.device(device)
        self.chunk = int(ext().outer_chunk_elems())
        self._tables = None
        self.total_chunks = 0
        self.key_chunks: list[tuple[str, int, int]] = []

    def build(self) -> None:
        segs = np.zeros(len(self.segments), dtype=SEG_DTYPE)
        locs = []
        chunk0 = 0
        self.key_chunks = []
        for i, s in enumerate(self.segments):
            n = s.glob.numel()
            if n % 4 or s.glob.data_ptr() % 16:
                raise ValueError(f"outer step: module {s.key} must be 16-byte aligned with a multiple of 4 elements")
            nch = (n + self.chunk - 1) // self.chunk
            segs[i] = (s.glob.data_ptr(), s.mom.data_ptr() if s.mom is not None else 0,
                       s.delta.data_ptr() if s.delta is not None else 0, n, len(locs),
                       len(s.locals32), s.mode, s.scale, s.inv_den, 0, chunk0)
            for j, l32 in enumerate(s.locals32):
                assert l32.numel() == n
                l16 = s.locals16[j]
                w = s.weights[j] if j < len(s.weights) else 0.0
                locs.append((l32.data_ptr(), l16.data_ptr() if l16 is not None else 0, w, 0))
            self.key_chunks.append((s.key, chunk0, nch))
            chunk0 += nch
        self.total_chunks = chunk0
        loc_arr = np.array(locs, dtype=LOC_DTYPE) if locs else np.zeros(1, dtype=LOC_DTYPE)
        seg_t = torch.from_numpy(segs.view(np.int64).copy()).to(self.device)
        loc_t = torch.from_numpy(loc_arr.view(np.int64).copy()).to(self.device)
        self._tables = (seg_t, loc_t)
        self.sq_part = torch.zeros(max(self.total_chunks, 1), device=self.device, dtype=torch.float32)

    def set_weights(self, weights: dict[str, list[float]], inv_den: dict[str, float] | None = None) -> None:
        changed = False
        for s in self.segments:
            if s.key in weights and list(weights[s.key]) != list(s.weights):
                s.weights = list(weights[s.key])
                changed = True
            if inv_den and s.key in inv_den and inv_den[s.key] != s.inv_den:
                s.inv_den = inv_den[s.key]
                changed = True
        if changed or self._tables is None:
            self.build()

    def tables(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(segment table, local table) on the device."""
        if self._tables is None:
            self.build()
        return self._tables

    def run(self, lr: float, momentum: float, nesterov: bool, first: bool,
            status: torch.Tensor | None = None) -> None:
        """One launch. ``status`` (int32 [1]) counts elements whose pseudo-gradient was not
        finite and were therefore left unchanged."""
        seg_t, loc_t = self.tables()
        ext().outer_step(seg_t, len(self.segments), loc_t, self.total_chunks, lr, momentum, nesterov, first,
                         self.sq_part, status)

    def with_mode(self, mode_for_outer: int) -> "OuterPlan":
        """A copy of this plan whose outer segments (OUTER or APPLY) run in
        ``mode_for_outer`` (ACC, APPLY or BCAST), sharing the same buffers. ACC and BCAST
        plans keep only those segments (private-module copies are dropped)."""
        segs = [Segment(s.key, s.glob, s.mom, s.locals32, s.locals16, s.weights,
                        mode_for_outer if s.mode in (MODE_OUTER, MODE_APPLY) else s.mode, s.scale, s.inv_den,
                        s.delta)
                for s in self.segments]
        if mode_for_outer in (MODE_ACC, MODE_BCAST):
            segs = [s for s in segs if s.mode == mode_for_outer]
        plan = OuterPlan(segs, self.device)
        plan.build()
        return plan

    def hbm_bytes(self) -> int:
        """Bytes one launch must move through HBM (each buffer read / written once): the
        algorithmic traffic the roofline of this plan's launch is computed from."""
        total = 0
        for s in self.segments:
            n, nl = s.glob.numel(), len(s.locals32)
            n16 = sum(1 for t in s.locals16 if t is not None)
            write_back = 4 * nl + 2 * n16
            if s.mode == MODE_COPY:
                per = 8
            elif s.mode == MODE_BCAST:
                per = 4 + write_back
            elif s.mode == MODE_ACC:
                per = 4 + 4 * nl + 4
            elif s.mode == MODE_APPLY:
                per = 3 * 4 + 2 * 4 + write_back       # delta, global, momentum in; momentum, global out
            else:
                per = 4 + 4 * nl + 4 + 2 * 4 + write_back
            total += per * n
        return total

    def delta_norms(self) -> dict[str, float]:
        """Per-key ||delta|| of the last run (read back once per round)."""
        part = self.sq_part.cpu()
        return {k: float(part[c0:c0 + n].double().sum().sqrt()) for k, c0, n in self.key_chunks}
