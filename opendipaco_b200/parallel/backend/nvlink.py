"""NVLink / NVSwitch backend: the DiLoCo outer step over peer memory, no NCCL.

Placement and the generic ``global_reduce`` API are inherited from
:class:`TorchDistBackend` (contiguous balanced path blocks, one NCCL subgroup per
module key, used only off the hot path). The fused executor instead calls
:meth:`NVLinkBackend.fused_outer_step` once per round, which runs three kernels:

1. ACC (local, ``csrc/outer.cu``): this rank's weighted pseudo-gradient partial
   ``sum_j w_j (global - local_j)`` for every shared key it owns, written into a
   symmetric DELTA buffer (and private keys copied into the bank);
2. APPLY (``csrc/outer_nvlink.cu``): cross-GPU barrier, then for the slice of every
   shared key this rank owns: peer loads of all sharers' partials (rank order),
   Nesterov on the momentum shard, peer stores of the new global into every
   sharer's GLOB;
3. BCAST: cross-GPU barrier, then the fresh globals are copied into the local
   working copies (fp32 master + bf16).

``NVLinkBackend(..., compress="int4")`` adds a QUANT kernel between 1 and 2: every rank
turns its partial plus an error-feedback residual (kept locally, carried to the next
round) into 4-bit codes with one absmax/7 scale per 128 elements, in symmetric QD / QS
buffers, and APPLY reads those codes instead of the fp32 partials and dequantises them
in registers: 0.53 instead of 4 bytes per element cross NVLink. Keys held by a single
GPU are not compressed. This is the NVLink counterpart of the int4 wire compression
of outer gradients in the reference's control plane (src/opendipaco/schedule/compress.py:92);
the residual is not checkpointed and restarts at zero after a resume.

``compress="topk"`` (with ``density``, default 0.01) keeps instead, in every 4096-element
block of a rank's partial plus residual, the ``ceil(density * len)`` entries of largest
magnitude as (uint16 index, fp32 value) pairs (a TOPK kernel, exact radix select); APPLY
sums the sharers' pairs of its block in shared memory. This is the blockwise analogue of
the reference's per-row top-k sparsification with error feedback
(src/opendipaco/schedule/compress.py:183); key regions and slices are 4096-aligned so an
APPLY chunk is one block.

Buffers are allocated with ``torch.distributed._symmetric_memory`` (``empty`` +
``rendezvous`` over the world group): the bank's GLOB, DELTA and momentum arenas
(identical offsets on every rank: one region per module key in ``module_keys()``
order) and a small flag pad for the epoch barriers. Device waits are bounded; a
peer that never arrives makes the kernels record ``ERR_TIMEOUT_PEER`` and the host
raises :class:`~opendipaco_b200.ops.KernelTimeout` after the round.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.distributed as dist

from ...ops._ext import err_word, ext
from ...ops.outer import MODE_ACC, MODE_BCAST, MODE_COPY, MODE_OUTER
from ...topology import is_private_key
from .torch_dist import TorchDistBackend

NVKEY = np.dtype([("off", "<i8"), ("s0", "<i8"), ("s1", "<i8"), ("chunk0", "<i8"), ("nsh", "<i4"),
                  ("sh", "<i4", (8,)), ("scale", "<f4"), ("inv_den", "<f4"), ("quant", "<i4")])
assert NVKEY.itemsize == 80
NVREGION = np.dtype([("off", "<i8"), ("n", "<i8"), ("group0", "<i8")])
ALIGN = 256
QGROUP = 128
SPBLOCK = 4096  # top-k block = one APPLY chunk


def _ru(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


class NVLinkBackend(TorchDistBackend):

    def __init__(self, topology, device: torch.device | None = None, dp: int = 1, compress: str | None = None,
                 density: float = 0.01):
        super().__init__(topology, device, dp=dp)
        if compress not in (None, "none", "int4", "topk"):
            raise ValueError(f"unknown NVLink outer-step compression {compress!r} (None, 'int4' or 'topk')")
        if not 0.0 < density <= 1.0:
            raise ValueError("density must be in (0, 1]")
        self.compress = compress if compress != "none" else None
        self.density = float(density)
        self.kcap = max(1, math.ceil(self.density * SPBLOCK))
        self._align = SPBLOCK if self.compress == "topk" else ALIGN
        self._dp_handles: list = []
        self._offs: dict[str, int] | None = None
        self._tables = None
        self._epoch = 0
        self._sq_keys: list[tuple[str, int, int]] = []
        # timing=True brackets the outer step's launches with CUDA events (phase_times())
        self.timing = False
        self._tev: list = []
        self.nvlink_bytes = {"in": 0, "out": 0}

    # ------------------------------------------------------------------ arenas
    def bank_arena(self, sizes: dict[str, int], device) -> tuple[dict, dict]:
        """Symmetric GLOB / momentum arenas; returns per-key views for owned keys."""
        import torch.distributed._symmetric_memory as symm

        self._offs, off = {}, 0
        for k in self.topology.module_keys():
            self._offs[k] = off
            off += _ru(sizes[k], self._align)
        self._sizes = dict(sizes)
        total = max(off, ALIGN)
        group = dist.group.WORLD.group_name
        self.dev = torch.device(device)

        def sym(n, dtype):
            t = symm.empty(n, dtype=dtype, device=self.dev)
            t.zero_()
            h = symm.rendezvous(t, group)
            return t, h

        self.GLOB, self._hg = sym(total, torch.float32)
        self.DELTA, self._hd = sym(total, torch.float32)
        self.MOM, self._hm = sym(total, torch.float32)
        self.PAD, self._hp = sym(2 * self.world_size, torch.int32)
        if self.compress == "int4":
            self.QD, self._hqd = sym(total // 8, torch.int32)       # 4-bit codes, two per byte
            self.QS, self._hqs = sym(total // QGROUP, torch.float32)  # one scale per 128 elements
        elif self.compress == "topk":
            nblk = total // SPBLOCK
            self.QD, self._hqd = sym((nblk * self.kcap + 1) // 2, torch.int32)  # uint16 indices
            self.QS, self._hqs = sym(nblk * self.kcap, torch.float32)         # values
        if self.compress:
            self.RES = torch.zeros(total, dtype=torch.float32, device=self.dev)
        torch.cuda.synchronize(self.dev)
        dist.barrier()
        as_dev = lambda ptrs: torch.tensor(list(ptrs), dtype=torch.int64, device=self.dev)  # noqa: E731
        self._gptrs = as_dev(self._hg.buffer_ptrs)
        self._dptrs = as_dev(self._hd.buffer_ptrs)
        self._pptrs = as_dev(self._hp.buffer_ptrs)
        if self.compress:
            self._qdptrs = as_dev(self._hqd.buffer_ptrs)
            self._qsptrs = as_dev(self._hqs.buffer_ptrs)
        glob = {k: self.GLOB[o:o + sizes[k]] for k, o in self._offs.items() if self.owns_module(k)}
        mom = {k: self.MOM[o:o + sizes[k]] for k, o in self._offs.items()
               if self.owns_module(k) and not is_private_key(k)}
        return glob, mom

    # ------------------------------------------------------------------ data parallelism
    def dp_tensor(self, shape, dtype) -> torch.Tensor:
        """A zeroed tensor in memory every member of this rank's data-parallel group can
        address (symmetric allocation, rendezvous over the group)."""
        import math

        import torch.distributed._symmetric_memory as symm

        n = max(math.prod(shape), 1)
        t = symm.empty(n, dtype=dtype, device=self.device)
        t.zero_()
        h = symm.rendezvous(t, self.dp_group.group_name)
        self._dp_handles.append((t, h))
        return t.view(*shape)

    def dp_table(self, w32, w16, grad, m1, m2, G: int, opt8=None) -> torch.Tensor:
        """Device table int64 [12][8] of every member's W32, W16, GRAD, M1, M2 (AdamW),
        signal pad, norm-exchange buffer and the 8-bit Adam state ``opt8 = (MQ, MABS,
        VQ, VLO, VSC)`` -- the layout the ``dp_*`` kernels read; absent rows are 0."""
        pad = self.dp_tensor((8,), torch.int32)
        norm = self.dp_tensor((8 * max(G, 1),), torch.float32)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.dp_group)
        handles = {t.data_ptr(): h for t, h in self._dp_handles}
        tab = torch.zeros(12, 8, dtype=torch.int64)
        rows = (w32, w16, grad, m1, m2, pad, norm) + tuple(opt8 or (None,) * 5)
        for row, t in enumerate(rows):
            if t is None:
                continue
            h = handles[t.data_ptr()]
            for m, ptr in enumerate(h.buffer_ptrs):
                tab[row, m] = ptr
        return tab.to(self.device)

    # ------------------------------------------------------------------ slices
    def slice_of(self, key: str, rank: int | None = None) -> tuple[int, int]:
        """[s0, s1) of ``key`` owned by ``rank`` (default: this rank) in the cross-GPU outer
        step: the key's sharers split it evenly, in multiples of 4 elements (of whole
        4096-element blocks in top-k mode)."""
        sh = self.sharing_ranks(key)
        n = self._sizes[key]
        per = _ru((n + len(sh) - 1) // len(sh), SPBLOCK if self.compress == "topk" else 4)
        i = sh.index(self.rank if rank is None else rank)
        return min(n, i * per), min(n, (i + 1) * per)

    def delta_view(self, key: str) -> torch.Tensor:
        """This rank's pseudo-gradient partial of ``key`` in the symmetric DELTA buffer (the
        peers read it during APPLY); the fused executor's last optimizer step writes it."""
        return self.DELTA[self._offs[key]:self._offs[key] + self._sizes[key]]

    def outer_launch_count(self, ex) -> int:
        """Kernels of one outer step: [ACC (+ private copies)] [QUANT | TOPK] APPLY BCAST."""
        t = self._tables
        acc = 0 if getattr(ex, "acc_fused", False) else 1 + (1 if t and t["cplan"] is not None else 0)
        return acc + (1 if self.compress else 0) + 2

    def _build(self, ex, plan) -> None:
        chunk = int(ext().outer_nvlink_chunk_elems())
        fused = getattr(ex, "acc_fused", False)
        # ACC plan: outer segments write their partial into DELTA; private copies run too
        # (unless the last inner step's optimizer kernel already did both)
        for s in plan.segments:
            if s.mode == MODE_OUTER:
                s.delta = self.delta_view(s.key)
        acc = None if fused else plan.with_mode(MODE_ACC)
        copies = [s for s in plan.segments if s.mode == MODE_COPY]
        if copies and not fused:
            from ...ops.outer import OuterPlan

            cplan = OuterPlan(copies, self.dev)
            cplan.build()
        else:
            cplan = None
        keys, chunk0 = [], 0
        apply_elems = 0
        regs, g0 = [], 0
        b_in = b_out = 0
        self._sq_keys = []
        for s in plan.segments:
            if s.mode != MODE_OUTER:
                continue
            sh = self.sharing_ranks(s.key)
            if len(sh) > 8:
                raise ValueError("NVLink outer step supports at most 8 sharer GPUs per module")
            s0, s1 = self.slice_of(s.key)
            nch = (s1 - s0 + chunk - 1) // chunk if s1 > s0 else 0
            rec = np.zeros(1, dtype=NVKEY)
            rec["off"], rec["s0"], rec["s1"], rec["chunk0"], rec["nsh"] = self._offs[s.key], s0, s1, chunk0, len(sh)
            rec["sh"][0, :len(sh)] = sh
            rec["scale"], rec["inv_den"] = s.scale, s.inv_den
            if self.compress and len(sh) > 1:
                r = np.zeros(1, dtype=NVREGION)
                if self.compress == "int4":
                    rec["quant"] = 1
                    ng = _ru(s.glob.numel(), QGROUP) // QGROUP
                    r["off"], r["n"], r["group0"] = self._offs[s.key], ng * QGROUP, g0
                else:
                    rec["quant"] = 2
                    ng = _ru(s.glob.numel(), SPBLOCK) // SPBLOCK
                    r["off"], r["n"], r["group0"] = self._offs[s.key], s.glob.numel(), g0
                regs.append(r)
                g0 += ng
            # bytes of this rank's APPLY slice that cross NVLink: the other sharers' partials
            # come in (fp32, int4 codes + scales, or top-k pairs), the new global goes out
            L = max(s1 - s0, 0)
            apply_elems += L
            if rec["quant"][0] == 1:
                bpe = 0.5 + 4.0 / QGROUP
            elif rec["quant"][0] == 2:
                bpe = 6.0 * self.kcap / SPBLOCK
            else:
                bpe = 4.0
            b_in += int(L * (len(sh) - 1) * bpe)
            b_out += L * (len(sh) - 1) * 4
            if nch:
                keys.append(rec)
                self._sq_keys.append((s.key, chunk0, nch))
            chunk0 += nch
        key_arr = np.concatenate(keys) if keys else np.zeros(1, dtype=NVKEY)
        to_dev = lambda a: torch.from_numpy(a.view(np.int64).copy()).to(self.dev)  # noqa: E731
        reg_arr = np.concatenate(regs) if regs else np.zeros(1, dtype=NVREGION)
        # BCAST: one segment per shared key with all of this GPU's sharers (the global is
        # read once per key)
        bplan = plan.with_mode(MODE_BCAST)
        # local HBM bytes of each phase (for the roofline of the whole outer step): APPLY
        # reads this rank's partial, global and momentum of its slices and writes momentum
        # and global (20 bytes per element); the peers' partials and the peer stores cross
        # NVLink (counted in b_in / b_out)
        self.phase_hbm_bytes = {"acc": acc.hbm_bytes() if acc is not None else 0,
                                "apply": 20 * apply_elems, "bcast": bplan.hbm_bytes()}
        if cplan is not None:
            self.phase_hbm_bytes["acc"] += cplan.hbm_bytes()
        self._tables = dict(plan_id=id(plan), acc=acc, cplan=cplan, keys=to_dev(key_arr), nkeys=len(keys),
                            chunks=chunk0, bplan=bplan, sq=torch.zeros(max(chunk0, 1), device=self.dev),
                            regs=to_dev(reg_arr), nregs=len(regs), groups=g0)
        self._all_keys = [k for k in self.topology.module_keys() if not is_private_key(k)]
        self.nvlink_bytes = {"in": b_in, "out": b_out}

    # ------------------------------------------------------------------ the round
    def fused_outer_step(self, ex, plan, first: bool) -> None:
        if self._tables is None or self._tables["plan_id"] != id(plan):
            self._build(ex, plan)
        t = self._tables
        dl = ex.e.diloco
        err = err_word(self.dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if self.timing else None
        if ev:
            ev[0].record()
        if t["acc"] is not None:
            t["acc"].run(0.0, 0.0, False, False)
        if t["cplan"] is not None:
            t["cplan"].run(0.0, 0.0, False, False)
        if ev:
            ev[1].record()
        qd = qs = None
        if self.compress == "int4":
            ext().outer_nvlink_quant(t["regs"], t["nregs"], t["groups"], self.DELTA, self.RES,
                                     self.QD.view(torch.uint8), self.QS)
        elif self.compress == "topk":
            ext().outer_nvlink_topk(t["regs"], t["nregs"], t["groups"], self.density, self.kcap, self.DELTA,
                                    self.RES, self.QD.view(torch.int16), self.QS)
        if self.compress:
            qd, qs = self._qdptrs, self._qsptrs
        if ev:
            ev[2].record()
        self._epoch += 1
        ext().outer_nvlink_apply(t["keys"], t["nkeys"], t["chunks"], self._dptrs, self._gptrs, self._pptrs,
                                 self.MOM, self.rank, self.world_size, self._epoch, dl.outer_lr,
                                 dl.outer_momentum, dl.outer_nesterov, first, t["sq"], err, qd, qs, self.kcap,
                                 getattr(ex, "OUTER_STATUS", None))
        if ev:
            ev[3].record()
        bp = t["bplan"]
        seg_t, loc_t = bp.tables()
        ext().outer_nvlink_bcast(seg_t, len(bp.segments), loc_t, bp.total_chunks, self._pptrs, self.rank,
                                 self.world_size, self._epoch, err)
        if ev:
            ev[4].record()
            self._tev.append(ev)

    def outer_roofline_ms(self, hbm_gbps: float, link_gbps: float) -> dict[str, float]:
        """Roofline time (ms) of each outer-step phase: its local HBM bytes at ``hbm_gbps``
        or, for APPLY, the slower of that and its bytes over NVLink at ``link_gbps`` per
        direction; "total" sums the phases (they run one after another)."""
        hb = getattr(self, "phase_hbm_bytes", {"acc": 0, "apply": 0, "bcast": 0})
        link = max(self.nvlink_bytes["in"], self.nvlink_bytes["out"]) / link_gbps / 1e6
        out = {"acc": hb["acc"] / hbm_gbps / 1e6, "apply": max(hb["apply"] / hbm_gbps / 1e6, link),
               "bcast": hb["bcast"] / hbm_gbps / 1e6}
        out["total"] = sum(out.values())
        return out

    def phase_times(self) -> dict[str, float]:
        """Mean device time (ms) of the outer step's phases over the timed calls since the
        last read: acc (local partials), quant (compression), apply (cross-GPU barrier +
        peer-memory reduce, Nesterov, write-back), bcast (barrier + local copies)."""
        torch.cuda.synchronize(self.dev)
        n = len(self._tev)
        out = {k: 0.0 for k in ("acc", "quant", "apply", "bcast")}
        for ev in self._tev:
            for i, k in enumerate(out):
                out[k] += ev[i].elapsed_time(ev[i + 1]) / n
        self._tev = []
        return out

    def delta_norms(self) -> dict[str, float]:
        """Per shared key ||delta||, summed over the key's slices on every rank."""
        sq = self._tables["sq"].cpu() if self._tables else torch.zeros(1)
        vec = torch.zeros(len(self._all_keys), dtype=torch.float64)
        idx = {k: i for i, k in enumerate(self._all_keys)}
        for k, c0, n in self._sq_keys:
            vec[idx[k]] = sq[c0:c0 + n].double().sum()
        v = vec.to(self.dev)
        dist.all_reduce(v)
        v = v.cpu()
        return {k: float(v[idx[k]].sqrt()) for k in self._all_keys if self.owns_module(k)}

    def peer_copy(self, segments: list[tuple[int, int, int]]) -> None:
        """One launch of our pull-copy kernel over (source address, destination address,
        fp32 elements) segments; sources may be peer addresses of the symmetric arenas.
        Addresses must be 16-byte aligned."""
        if not segments:
            return
        from ...ops._ext import ext

        for src, dst, n in segments:
            if src % 16 or dst % 16:
                raise ValueError("peer_copy: 16-byte aligned addresses only")
        for i in range(0, len(segments), 65535):
            part = segments[i:i + 65535]
            tab = torch.tensor(part, dtype=torch.int64).to(self.dev)
            ext().peer_copy(tab, max(n for _, _, n in part))

    def gather_momentum(self, ex) -> None:
        """Fill the non-owned slices of each owned key's momentum from its owners (peer
        loads in one launch, between two barriers)."""
        torch.cuda.synchronize(self.dev)
        dist.barrier()
        segs = []
        for key, buf in ex.mom.items():
            off = self._offs[key]
            for r in self.sharing_ranks(key):
                if r == self.rank:
                    continue
                s0, s1 = self.slice_of(key, r)
                if s1 > s0:
                    segs.append((self._hm.buffer_ptrs[r] + 4 * (off + s0), buf.data_ptr() + 4 * s0, s1 - s0))
        self.peer_copy(segs)
        torch.cuda.synchronize(self.dev)
        dist.barrier()

    def bank_sources(self) -> dict[str, tuple[int, int]] | None:
        """key -> (peer address of the key's region in the GLOB arena of the rank that
        serves it, region length): the rank owning the key's lowest-index path, as in the
        broadcast gather. None before the arenas exist."""
        if self._offs is None:
            return None
        topo = self.topology
        out = {}
        for key in topo.module_keys():
            src = self.rank_of_path(min(topo.paths_through_module(key), key=topo.path_index))
            out[key] = (self._hg.buffer_ptrs[src] + 4 * self._offs[key], self._sizes[key])
        return out

    def close(self) -> None:
        torch.cuda.synchronize(self.dev) if self._offs is not None else None
