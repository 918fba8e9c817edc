"""Fused B200 executor for :class:`~opendipaco_b200.train.loop.DiPaCoEngine`.

Memory layout (per GPU, G = owned paths):

* one flat fp32 arena per quantity, shape ``[G, P]``: master weights, gradients,
  AdamW moments (or the blockwise 8-bit state), plus a bf16 working copy of the
  weights for the GEMMs. ``P`` is one path's parameter count with every tensor
  padded to a multiple of 256 elements (so 8-bit blocks never straddle two tensors
  and every TMA base is 512-byte aligned). Tensors appear in ``PathModel.parameters()``
  order, so a path's modules are contiguous regions and ``q|k|v`` and ``gate|up``
  are single ``[3H, H]`` / ``[2F, H]`` matrices.
* the global bank: one flat fp32 buffer (+ momentum) per owned module key with the
  same module-relative layout, so the outer step is elementwise over regions.
* every ``nn.Parameter`` of ``engine.bank`` and of the per-path ``PathModel``s is a
  view into these arenas: checkpoints, ``global_modules()`` and evaluation see the
  live weights without copies.

One inner step for all G paths = embedding gather, per layer RMSNorm -> QKV GEMM ->
attention (RoPE fused) -> O GEMM (+residual) -> RMSNorm -> gate|up GEMM (SwiGLU
epilogue) -> down GEMM (+residual), final RMSNorm -> LM-head GEMM (log-sum-exp
partials in the epilogue) -> CE, and the mirror-image backward, then the
deterministic grad-norm clip and one AdamW (or 8-bit Adam) launch over the whole
arena. Every GEMM is the grouped tcgen05 kernel over the G paths' weights. A round
(``inner_steps`` steps) is captured once in a CUDA graph; each round then costs one
host->device copy of its token batches + schedule, one graph launch, one outer-step
kernel and one device->host read of the last step's losses.

Semantics match the module executor: same batch indices (drawn from the engine's
CPU generator path by path), same cosine schedule, bf16 compute with fp32 master
weights (the reference's ``inner_autocast`` numerics), fp32 pseudo-gradients and
outer SGD-Nesterov.
"""

from __future__ import annotations

import logging
import math
import os
from collections import defaultdict
from dataclasses import dataclass

import numpy as np

import torch
from torch import nn

from ..models.llama import rope_cos_sin
from ..models.path import build_path_model
from ..ops import attention as attn
from ..ops._ext import check_errors, err_word, ext
from ..ops.outer import MODE_APPLY, MODE_COPY, MODE_OUTER, OuterPlan, Segment
from ..optim.adam8bit import Adam8bit
from ..optim.diloco import inner_lr_at, make_inner_optimizer
from ..topology import Path, is_private_key

ALIGN = 256
log = logging.getLogger(__name__)

# tables of the last inner step's AdamW + pseudo-gradient kernel (csrc/adam.cu)
ACC_REGION = np.dtype([("begin", "<i8"), ("end", "<i8"), ("first", "<i4"), ("count", "<i4"), ("cta0", "<i8")])
ACC_CTA_ELEMS = 1024  # elements of one region per CTA of adamw_acc_step
ACC_MAX_ENTRIES = 128  # (path, key) entries of one region
ACC_ENTRY = np.dtype([("delta", "<u8"), ("glob", "<u8"), ("g", "<i4"), ("flags", "<i4"), ("weight", "<f4"),
                      ("pad", "<i4")])
assert ACC_REGION.itemsize == 32 and ACC_ENTRY.itemsize == 32


def _ru(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


@dataclass
class _LayerOffsets:
    qkv: int
    o: int
    gu: int
    down: int
    ln1: int
    ln2: int


class PathLayout:
    """Flat layout of one path's parameters (``PathModel.named_parameters`` order)."""

    def __init__(self, pm: nn.Module, cfg):
        self.entries: list[tuple[str, tuple, int, int]] = []
        off = 0
        for name, p in pm.named_parameters():
            self.entries.append((name, tuple(p.shape), off, p.numel()))
            off += _ru(p.numel())
        self.P = off
        self.by_name = {n: (s, o, k) for n, s, o, k in self.entries}
        bb = cfg.backbone
        self.layers: list[_LayerOffsets] = []
        for i, _ in enumerate(pm._body_keys):
            for j in range(len(pm.body[i].layers)):
                pre = f"body.{i}.layers.{j}."
                o = {k: self.by_name[pre + k][1] for k in (
                    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                    "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                    "mlp.down_proj.weight", "input_layernorm.weight", "post_attention_layernorm.weight")}
                H, Fd, D = bb.hidden_size, bb.intermediate_size, bb.head_dim
                nq, nkv = bb.num_attention_heads, bb.kv_heads()
                if (o["self_attn.k_proj.weight"] != o["self_attn.q_proj.weight"] + nq * D * H
                        or o["self_attn.v_proj.weight"] != o["self_attn.k_proj.weight"] + nkv * D * H
                        or o["mlp.up_proj.weight"] != o["mlp.gate_proj.weight"] + Fd * H):
                    raise ValueError("fused executor needs q|k|v and gate|up to be contiguous "
                                     "(hidden/intermediate sizes must keep 256-element alignment)")
                self.layers.append(_LayerOffsets(o["self_attn.q_proj.weight"], o["self_attn.o_proj.weight"],
                                                 o["mlp.gate_proj.weight"], o["mlp.down_proj.weight"],
                                                 o["input_layernorm.weight"],
                                                 o["post_attention_layernorm.weight"]))
        self.emb = self.by_name["embed.embed_tokens.weight"][1]
        self.normf = self.by_name["head.norm.weight"][1]
        self.lm = self.by_name["head.lm_head.weight"][1]


def acc_region_table(regions: dict) -> tuple[np.ndarray, list, int]:
    """Region records of ``adamw_acc_step`` for ``{(begin, end): [entries]}``: each region
    gets ceil((end - begin) / ACC_CTA_ELEMS) CTAs, in ascending order of ``begin``.
    Returns (records, an empty entry list to fill in the same order, total CTAs)."""
    reg = np.zeros(len(regions), dtype=ACC_REGION)
    first = cta = 0
    for ri, ((a, b), lst) in enumerate(sorted(regions.items())):
        if len(lst) > ACC_MAX_ENTRIES:
            raise ValueError(f"adamw_acc_step: {len(lst)} (path, key) entries in one region (max {ACC_MAX_ENTRIES})")
        if a % 4:
            raise ValueError("adamw_acc_step: regions must begin at a multiple of 4 elements")
        reg[ri] = (a, b, first, len(lst), cta)
        first += len(lst)
        cta += (b - a + ACC_CTA_ELEMS - 1) // ACC_CTA_ELEMS
    return reg, [], cta


def _rebind(module: nn.Module, prefix_map, flat: torch.Tensor, layout_by_name, prefix: str) -> None:
    """Point every parameter of ``module`` at its slice of ``flat`` (copying values)."""
    for name, p in module.named_parameters():
        shape, off, n = layout_by_name[prefix + name]
        view = flat[off:off + n].view(shape)
        view.copy_(p.data)
        p.data = view


class FusedExecutor:
    def __init__(self, engine):
        self.e = engine
        cfg, dl = engine.config, engine.diloco
        if cfg.tie_word_embeddings:
            raise ValueError("the fused executor does not support tie_word_embeddings; "
                             "use ExecOptions(fused=False)")
        bb = cfg.backbone
        if bb.head_dim != 64:
            raise ValueError("the fused executor's attention kernel needs head_dim 64")
        if bb.hidden_size % 128:
            raise ValueError("the fused executor needs hidden_size % 128 == 0")
        self.dev = engine.device
        from ..ops.gemm import sm_count

        self.sms = sm_count(self.dev)
        self.topo = engine.topology
        self.paths: list[Path] = list(engine.backend.owned_paths())
        self.G = len(self.paths)
        if self.G == 0:
            raise ValueError("no owned paths")
        self.bb = bb
        self.eps = bb.rms_norm_eps
        self.opt8 = bool(getattr(dl, "optim_8bit", False))

        # -- per-path models (views into the flat arenas) ------------------------------
        pms = [build_path_model(cfg, p, engine.bank, deepcopy=True).to(self.dev) for p in self.paths]
        self.layout = PathLayout(pms[0], cfg)
        P, G = self.layout.P, self.G
        self.P = P
        be = engine.backend
        # intra-path data parallelism: this path group's batch is split over `dp` GPUs whose
        # masters, bf16 copies, gradients and moments sit in peer-addressable memory
        self.dp = int(getattr(be, "dp", 1))
        if self.dp > 1:
            if not hasattr(be, "dp_tensor"):
                raise NotImplementedError("intra-path data parallelism needs a peer-memory backend (NVLinkBackend)")
            zeros = lambda *shape, dtype=torch.float32: be.dp_tensor(shape, dtype)  # noqa: E731
        else:
            zeros = lambda *shape, dtype=torch.float32: torch.zeros(*shape, device=self.dev, dtype=dtype)  # noqa: E731
        self.W32 = zeros(G, P)
        self.W16 = zeros(G, P, dtype=torch.bfloat16)
        self.GRAD = zeros(G, P)
        if self.opt8:
            nb = P // ALIGN
            self.MQ = zeros(G * nb, ALIGN, dtype=torch.int8)
            self.MABS = zeros(G * nb)
            self.VQ = zeros(G * nb, ALIGN, dtype=torch.uint8)
            self.VLO = zeros(G * nb)
            self.VSC = zeros(G * nb)
            self.MOM1 = self.MOM2 = None
        else:
            self.MOM1 = zeros(G, P)
            self.MOM2 = zeros(G, P)
        for g, pm in enumerate(pms):
            _rebind(pm, None, self.W32[g], self.layout.by_name, "")
        self.W16.copy_(self.W32)
        if self.dp > 1:
            # member j of the group updates shard [j * PS, (j + 1) * PS) of every path
            self.dp_index = be.dp_index
            ps = _ru((P + self.dp - 1) // self.dp)
            self.dp_s0, self.dp_s1 = min(P, self.dp_index * ps), min(P, (self.dp_index + 1) * ps)
            opt8 = (self.MQ, self.MABS, self.VQ, self.VLO, self.VSC) if self.opt8 else None
            self.dp_tab = be.dp_table(self.W32, self.W16, self.GRAD, self.MOM1, self.MOM2, G, opt8)
            self.dp_counter = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.pms = dict(zip(self.paths, pms))
        if engine.materialize == "eager" and hasattr(engine, "_eager_views"):
            engine._eager_views.update(self.pms)
        self.steps_taken = [0] * G
        self._inner_opts: dict[Path, torch.optim.Optimizer] = {}

        # -- global bank as flat buffers -------------------------------------------
        self.glob: dict[str, torch.Tensor] = {}
        self.mom: dict[str, torch.Tensor] = {}
        # solo: a one-path task trainer (worker) -- the engine's bank is only read, never
        # rebound, and there is no outer step
        self.solo = bool(getattr(engine, "solo", False))
        arena = None
        if hasattr(engine.backend, "bank_arena") and not self.solo:
            # cross-GPU backends place the bank in peer-addressable (symmetric) memory
            sizes = {k: self._region_size(k) for k in self.topo.module_keys()}
            arena = engine.backend.bank_arena(sizes, self.dev)
        for key, mod in ({} if self.solo else engine.bank).items():
            n = self._region_size(key)
            buf = arena[0][key] if arena else torch.zeros(n, device=self.dev, dtype=torch.float32)
            self._rebind_bank(key, mod, buf)
            self.glob[key] = buf
            if not is_private_key(key):
                self.mom[key] = (arena[1][key] if arena else
                                 torch.zeros(n, device=self.dev, dtype=torch.float32))
        self.outer_steps = 0
        self._plan: OuterPlan | None = None
        self._plan_weights = None
        # the last inner step's AdamW also accumulates the outer pseudo-gradient of every
        # module key (plain AdamW, one GPU per path group); the outer step then reads one
        # partial per key instead of every working copy again
        self.acc_fused = (not self.opt8 and self.dp == 1 and not self.solo
                          and os.environ.get("ODP_ACC_FUSED", "1") != "0")
        self._deltas: dict[str, torch.Tensor] = {}
        self._acc_w: dict[tuple[str, int], float] = {}
        self.ACC_REG = self.ACC_ENT = None
        self.acc_nregs = self.acc_ctas = 0
        # elements the outer step's guard skipped because their pseudo-gradient was not finite
        self.OUTER_STATUS = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.outer_nonfinite = 0

        # -- step buffers are sized on the first round ---------------------------------
        self._shape = None
        self.wg_split: dict[str, int] = {}
        # ODP_HEAD_DW_CTAS=n > 0: LM-head weight gradient on a side stream with n CTAs
        self._side_ctas = int(os.environ.get("ODP_HEAD_DW_CTAS", "0"))
        self._side = torch.cuda.Stream(device=self.dev) if self._side_ctas > 0 else None
        self._ev_fork = torch.cuda.Event() if self._side_ctas > 0 else None
        self._ev_join = torch.cuda.Event() if self._side_ctas > 0 else None
        self._ahead = None  # (round key, host slot, active flags) sampled ahead of time
        self._slot = 0
        self._graph = None
        self._warm = False
        self.sq_bases = None

    # ------------------------------------------------------------------ layout helpers
    # Every path has the same segment structure, hence the same flat layout: module
    # key -> parameter-name prefix -> one region, identical on all paths.
    def _prefix(self, key: str) -> str:
        role = self.topo.role_of_key(key)
        if role in ("embed", "head"):
            return role + "."
        return f"body.{self.topo._segment_index_of_key(key) - 1}."

    def _entries(self, key: str):
        pre = self._prefix(key)
        return pre, [(n, s, o, k) for n, s, o, k in self.layout.entries if n.startswith(pre)]

    def _region(self, key: str) -> tuple[int, int]:
        _, ents = self._entries(key)
        return min(o for _, _, o, _ in ents), max(o + _ru(k) for _, _, o, k in ents)

    def _rel_entries(self, key: str):
        """(name within the module, shape, offset from the region start, numel)."""
        pre, ents = self._entries(key)
        start = self._region(key)[0]
        return [(n[len(pre):], s, o - start, k) for n, s, o, k in ents]

    def _region_size(self, key: str) -> int:
        a, b = self._region(key)
        return b - a

    def _local_region(self, g: int, key: str) -> tuple[int, int]:
        return self._region(key)

    def _rebind_bank(self, key: str, mod: nn.Module, buf: torch.Tensor) -> None:
        rel = {n: (s, o, k) for n, s, o, k in self._rel_entries(key)}
        for name, p in mod.named_parameters():
            s, o, k = rel[name]
            view = buf[o:o + k].view(s)
            view.copy_(p.data)
            p.data = view

    # ------------------------------------------------------------------ buffers
    def _alloc(self, B: int, S: int, steps: int) -> None:
        bb, G, dev = self.bb, self.G, self.dev
        H, Fd, V = bb.hidden_size, bb.intermediate_size, bb.vocab_size
        nh, nkv = bb.num_attention_heads, bb.kv_heads()
        C = (nh + 2 * nkv) * 64
        M = B * S
        L = len(self.layout.layers)
        if S % 64:
            raise ValueError("fused executor needs sequence_length % 64 == 0")
        if V % 8:
            raise ValueError("fused executor needs vocab_size % 8 == 0")
        f32, b16 = torch.float32, torch.bfloat16
        z = lambda *s, dt=f32: torch.zeros(*s, device=dev, dtype=dt)  # noqa: E731
        self.B, self.S, self.M, self.C, self.L = B, S, M, C, L
        self.T = 2 * ((V + 127) // 128)  # (max, sum exp) partials: two per 128-column tile
        # activation checkpointing: only the layer inputs X are kept; each layer's other
        # activations live in one shared slot and are recomputed before its backward
        self.ckpt = bool(getattr(self.e.diloco, "activation_checkpoint", False)) and L > 1
        nslot = 1 if self.ckpt else max(L, 1)
        self.X = z(L + 1, G, M, H)
        self.HR = z(nslot, G, M, H)
        self.XN1 = z(nslot, G, M, H, dt=b16)
        self.XN2 = z(nslot, G, M, H, dt=b16)
        self.RS1 = z(nslot, G, M)
        self.RS2 = z(nslot, G, M)
        self.QKV = z(nslot, G, M, C, dt=b16)
        self.O = z(nslot, G, M, H, dt=b16)
        self.LSEA = z(nslot, G * B, nh, S)
        self.GU = z(nslot, G, M, 2 * Fd, dt=b16)
        self.ACT = z(nslot, G, M, Fd, dt=b16)
        self.XNF = z(G, M, H, dt=b16)
        self.RSF = z(G, M)
        # loss_chunks > 1: the LM head runs over chunks of each path's sequences (as
        # torch.chunk splits the batch), so the logits buffer holds one chunk
        k = max(1, int(getattr(self.e.diloco, "loss_chunks", 1) or 1))
        per = -(-B // k)
        self.chunks = [(b0 * S, min(B, b0 + per) * S) for b0 in range(0, B, per)] if k > 1 else [(0, M)]
        self.MCH = self.chunks[0][1] - self.chunks[0][0]  # rows of the logits buffer
        self.LOGITS = z(G, self.MCH, V, dt=b16)
        # one-pass CE keeps a row in registers (<= 32768 columns); wider vocabularies use GEMM partials
        self.ce_fused = V % 8 == 0 and V <= 32768 and os.environ.get("ODP_CE_IMPL", "fused") == "fused"
        self.PART = z(1) if self.ce_fused else z(G, self.MCH, self.T, 2)
        # the LM-head gradient GEMMs form the dlogits from the logits (CTA-pair kernel:
        # at least 256 rows per chunk and vocabulary, hidden a multiple of 192 or 256)
        pairable = H >= 256 and (H % 256 == 0 or H % 192 == 0)
        self.ce_xf = (self.ce_fused and pairable and self.MCH >= 256 and V >= 256 and self._side_ctas == 0
                      and os.environ.get("ODP_CE_GRAD_FUSED", "0") == "1")
        self.CEOB = z(G, M) if self.ce_xf else None
        self.LSEC = z(G, M)
        self.ROWLOSS = z(G, M)
        self.LOSSSUM = z(G)
        self.INVCNT = z(G)
        self.DX = z(G, M, H)
        self.DX16 = z(G, M, H, dt=b16)
        self.DXN = z(G, M, H)
        self.DGU = z(G, M, 2 * Fd, dt=b16)
        self.DOUT = z(G, M, H, dt=b16)
        self.DQKV = z(G, M, C, dt=b16)
        # Weight gradients on a second stream: each is needed only by the optimizer, and the
        # grids of the backward's GEMMs, norms and attention leave SMs idle (with few paths per
        # GPU, most of them) that the weight-gradient GEMMs can use. Measured inner step: 2
        # paths 2.07 -> 1.85 ms, 4 paths 3.51 -> 3.44, 16 paths 13.23 -> 13.05. The buffers they
        # read (dY of each projection) are rewritten by the next layer, so each gets a ring of
        # two slots; the main stream waits for the side stream to finish reading a slot before
        # writing it again, and joins the side stream before the optimizer. ODP_WGRAD_STREAM=0
        # keeps them on the main stream. (Not with activation checkpointing, whose one
        # activation slot the next layer's recomputation overwrites, nor with a chunked LM head.)
        self.wg_side = (os.environ.get("ODP_WGRAD_STREAM", "1") != "0" and not self.ckpt and len(self.chunks) == 1
                        and self._side_ctas == 0)
        self._wgs = torch.cuda.Stream(device=dev) if self.wg_side else None
        self._rings, self._ring_i, self._ring_ev, self._ring_busy = {}, {}, {}, {}
        for name, buf in (("dx16", self.DX16), ("dgu", self.DGU), ("dqkv", self.DQKV)):
            slots = [buf, torch.empty_like(buf)] if self.wg_side else [buf]
            self._rings[name], self._ring_i[name] = slots, 0
            self._ring_ev[name] = [torch.cuda.Event() for _ in slots] if self.wg_side else []
            self._ring_busy[name] = [False] * len(slots)
        self._wg_fork = torch.cuda.Event() if self.wg_side else None
        self._wg_join = torch.cuda.Event() if self.wg_side else None
        self.DELTA = z(G * B, nh, S)
        # flash attention (S > 128): q|k rotated once per call into this scratch
        shp = attn.qkr_shape(G * B, S, nh, nkv)
        self.QKR = z(*shp, dt=b16) if shp else None
        self.NORMWORK = z(G * ((M + 7) // 8) * H)  # RMSNorm weight-gradient partials (8-row blocks at most)
        self.CLIPWORK = z(G * ((self.P + (1 << 16) - 1) // (1 << 16)))
        self.COEF = z(G)
        self.GNORM = z(G)
        self.IDS = z(steps, G, M, dt=torch.int32)
        self.LABELS = z(steps, G, M, dt=torch.int32)
        self.SCHED = z(steps, G, 4)
        self.LOSSES = z(steps, G)
        self.INVC = z(steps, G)  # 1 / valid labels of each (step, path) batch, for split batches
        self.EMBKEYS = z(G, M, dt=torch.int32)  # sorted (token, row) keys of the embedding backward
        # touched-row flags of the embedding gradient: rows of tokens absent from a step are
        # neither zeroed nor read (the norm and AdamW kernels take them as gradient 0);
        # plain AdamW on one GPU per path group with the sorted embedding backward
        self.emb_rows = (z(G, V, dt=torch.uint8) if (M <= 4096 and V < (1 << 20) and V * H < (1 << 31) and self.dp == 1 and not self.opt8
                                                     and os.environ.get("ODP_EMB_ROWS", "1") != "0") else None)
        # K splits of the weight-gradient GEMMs (tokens are K) that cannot fill the GPU alone
        # (few paths per GPU), and their shared workspace
        from ..ops.gemm import splitk_factor

        self.wg_shapes = {"lm": (V, H)}
        for i in range(L):
            self.wg_shapes.update({f"down{i}": (H, Fd), f"gu{i}": (2 * Fd, H), f"o{i}": (H, H), f"qkv{i}": (C, H)})
        self.wg_split = {k: splitk_factor(m, n, M, G, self.sms) for k, (m, n) in self.wg_shapes.items()}
        ws = max([G * sp * self.wg_shapes[k][0] * self.wg_shapes[k][1] for k, sp in self.wg_split.items()
                  if sp > 1] or [1])
        self.WGWS = z(ws)
        # gradient-norm clip without re-reading the gradients: the weight-gradient GEMMs
        # write a sum of squares per 32 x 32 output box, the embedding backward one per
        # written row, and the norm weights are read directly (same condition as the row
        # flags: the embedding backward must be the sorted one)
        self.sq_bases = None
        if self.emb_rows is not None and os.environ.get("ODP_FUSED_NORM", "1") != "0":
            lay = self.layout
            cb = lambda m, n: ((m + 31) // 32) * ((n + 31) // 32)  # noqa: E731
            bases, nslot = {}, 0
            for name, (m, n) in [("lm", (V, H))] + [(f"{k}{i}", mn) for i in range(L) for k, mn in
                                                    (("down", (H, Fd)), ("gu", (2 * Fd, H)), ("o", (H, H)),
                                                     ("qkv", (C, H)))]:
                bases[name] = nslot
                nslot += cb(m, n)
            covered = 2 * V * H + L * (C * H + H * nh * 64 + 3 * Fd * H + 2 * H) + H
            total = sum(k for _, _, _, k in lay.entries)
            if covered == total:  # every parameter has a producer that reports its squares
                self.sq_bases, self.sq_nslot = bases, nslot
        if self.sq_bases is not None:
            lay = self.layout
            self.SQPARTS = z(G, self.sq_nslot)
            self.EMBSQ = z(G, M)
            offs = [o for lo in lay.layers for o in (lo.ln1, lo.ln2)] + [lay.normf]
            self.NORMOFFS = torch.tensor(offs, dtype=torch.int64, device=dev)
        # two sets of pinned round inputs: while the GPU runs round r from one set, the host
        # samples round r + 1 into the other (engine.fit looks ahead when the next round is
        # certain to follow; the generator is consumed in the same order either way)
        self._host = [dict(ids=torch.zeros(steps, G, M, dtype=torch.int32).pin_memory(),
                           labels=torch.zeros(steps, G, M, dtype=torch.int32).pin_memory(),
                           sched=torch.zeros(steps, G, 4, dtype=torch.float32).pin_memory(),
                           invc=torch.zeros(steps, G, dtype=torch.float32).pin_memory()) for _ in range(2)]
        self._slot = 0
        self._ahead = None
        self.ids_host, self.labels_host = self._host[0]["ids"], self._host[0]["labels"]
        self.sched_host = self._host[0]["sched"]
        self.loss_host = torch.zeros(G, dtype=torch.float32).pin_memory()
        self.status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.invc_host = self._host[0]["invc"]
        self.cos, self.sin = rope_cos_sin(64, bb.rope_theta, S, dev)
        self.err = err_word(dev)
        self._shape = (B, S, steps)
        self._graph = None
        self._warm = False

    # ------------------------------------------------------------------ GEMM helper
    def _bn(self, M: int, N: int) -> int:
        # 128-wide tiles once they fill about two thirds of a wave (100 tiles on 148 SMs);
        # 64-wide below that
        tiles128 = self.G * ((M + 127) // 128) * ((N + 127) // 128)
        return 128 if tiles128 * 148 >= 100 * self.sms else 64

    def _sq(self, name: str) -> dict:
        """GEMM keyword arguments that make a weight-gradient GEMM write its box sums of
        squares into this step's slots (none when the fused clip norm is off)."""
        if self.sq_bases is None:
            return {}
        return {"sq": self.SQPARTS.view(-1)[self.sq_bases[name]:], "sq_ld": self.sq_nslot}

    def _wgrad(self, name: str, A, lda, sa, B, ldb, sb, C, ldc, sc, M, N, K) -> None:
        """fp32 weight gradient (both operands MN-major, K = tokens), split over K when
        few paths per GPU leave the tile grid short of the SM count."""
        from ..ops.gemm import gemm_wgrad

        sq = self._sq(name)
        gemm_wgrad(A, lda, sa, B, ldb, sb, C, ldc, sc, M, N, K, self.G, self.wg_split[name], self.WGWS,
                   sq.get("sq"), sq.get("sq_ld", 0), self.err, bn=self._bn(M, N))

    def _ring_write(self, name: str) -> torch.Tensor:
        """The ring slot to write next for buffer ``name``: the main stream first waits
        until the side stream has read what that slot held."""
        slots = self._rings[name]
        if len(slots) == 1:
            return slots[0]
        i = (self._ring_i[name] + 1) % len(slots)
        self._ring_i[name] = i
        if self._ring_busy[name][i]:
            torch.cuda.current_stream(self.dev).wait_event(self._ring_ev[name][i])
            self._ring_busy[name][i] = False
        return slots[i]

    def _wgrad_async(self, ring: str | None, name: str, *args) -> None:
        """``_wgrad`` on the side stream (when enabled), after everything issued so far on
        the main stream; marks the ring slot it reads as busy until it has run."""
        if self._wgs is None:
            self._wgrad(name, *args)
            return
        cur = torch.cuda.current_stream(self.dev)
        self._wg_fork.record(cur)
        self._wgs.wait_event(self._wg_fork)
        with torch.cuda.stream(self._wgs):
            self._wgrad(name, *args)
        if ring is not None:
            i = self._ring_i[ring]
            self._ring_ev[ring][i].record(self._wgs)
            self._ring_busy[ring][i] = True

    def _wgrad_join(self) -> None:
        """The main stream waits for every weight gradient issued on the side stream."""
        if self._wgs is None:
            return
        self._wg_join.record(self._wgs)
        torch.cuda.current_stream(self.dev).wait_event(self._wg_join)
        for name in self._ring_busy:
            self._ring_busy[name] = [False] * len(self._ring_busy[name])

    def _gemm(self, A, lda, sa, amn, B, ldb, sb, bmn, C, ldc, sc, M, N, K, epi, bn=None, **kw):
        from ..ops.gemm import EPI

        ext().gemm_bf16(A, lda, sa, amn, B, ldb, sb, bmn, C, ldc, sc, M, N, K, self.G, EPI[epi],
                        bn or self._bn(M, N), kw.get("R"), kw.get("ldr", 0), kw.get("sr", 0),
                        kw.get("aux"), kw.get("ldx", 0), kw.get("sx", 0), kw.get("part"),
                        kw.get("beta", 0.0), kw.get("f_half", 0), self.err, kw.get("max_ctas", 0), kw.get("sq"),
                        kw.get("sq_ld", 0))

    # ------------------------------------------------------------------ one inner step
    def _step(self, s: int, last: bool = False) -> None:
        X_ = ext()
        bb, G, P = self.bb, self.G, self.P
        H, Fd, V = bb.hidden_size, bb.intermediate_size, bb.vocab_size
        nh, nkv = bb.num_attention_heads, bb.kv_heads()
        M, C, S, B = self.M, self.C, self.S, self.B
        w32, w16, gr = self.W32.view(-1), self.W16.view(-1), self.GRAD.view(-1)
        lay = self.layout
        ids, labels = self.IDS[s], self.LABELS[s]
        MH, MC, MF, MF2 = M * H, M * C, M * Fd, M * 2 * Fd

        # ---------------- forward
        X_.embedding_fwd(ids, w32[lay.emb:], P, self.X[0], M, H, G, V)
        for l in range(self.L):
            self._layer_fwd(l, down=True)
        L = self.L
        X_.rmsnorm_fwd(self.X[L], MH, w32[lay.normf:], P, self.XNF, MH, self.RSF, M, H, G, self.eps)
        if len(self.chunks) > 1:
            self._lm_head_chunked(s, labels)
        elif self.ce_fused:
            # plain bf16 logits (TMA-stored), then loss + dlogits in one pass over each row --
            # or, when the gradient GEMMs form the dlogits themselves, a read-only pass that
            # leaves the logits in place and writes each row's exponent offset
            self._gemm(self.XNF, H, MH, False, w16[lay.lm:], H, P, False, self.LOGITS, V, M * V, M, V, H, "bf16",
                       bn=128)
            X_.ce_fused(self.LOGITS, V, M * V, labels, M, V, G, self.LSEC, self.ROWLOSS, self.LOSSSUM, self.INVCNT,
                        self.LOSSES[s], self.err, self.INVC[s] if self.dp > 1 else None,
                        self.CEOB if self.ce_xf else None)
        else:
            self._gemm(self.XNF, H, MH, False, w16[lay.lm:], H, P, False, self.LOGITS, V, M * V, M, V, H, "logits",
                       bn=128, part=self.PART)
            given = self.INVC[s] if self.dp > 1 else None
            X_.ce_forward(self.PART, self.T, self.LOGITS, V, M * V, labels, M, G, self.LSEC, self.ROWLOSS,
                          self.LOSSSUM, self.INVCNT, self.LOSSES[s], given)
            X_.ce_backward(self.LOGITS, V, M * V, self.LSEC, labels, self.INVCNT if given is None else given, M, V,
                           G)
        # ---------------- backward
        side = self._side if len(self.chunks) == 1 and not self.ce_xf else None
        if len(self.chunks) == 1:
            if self.ce_xf:
                self._ce_grad_gemms(labels, self.INVC[s] if self.dp > 1 else self.INVCNT)
            else:
                self._gemm(self.LOGITS, V, M * V, False, w16[lay.lm:], H, P, True, self.DXN, H, MH, M, H, V, "f32")
        if len(self.chunks) > 1 or self.ce_xf:
            pass  # the chunks (or the softmax-gradient GEMMs) already wrote DXN and the LM-head weight gradient
        elif side is not None:
            # the LM-head weight gradient is needed only by the optimizer: on a side stream
            # with a capped grid it runs under the layers' backward, whose small GEMMs and
            # attention leave SMs idle; joined before the gradient norm
            cur = torch.cuda.current_stream(self.dev)
            self._ev_fork.record(cur)
            side.wait_event(self._ev_fork)
            with torch.cuda.stream(side):
                self._gemm(self.LOGITS, V, M * V, True, self.XNF, H, MH, True, gr[lay.lm:], H, P, V, H, M, "f32",
                           max_ctas=self._side_ctas, **self._sq("lm"))
                self._ev_join.record(side)
        else:
            self._wgrad_async(None, "lm", self.LOGITS, V, M * V, self.XNF, H, MH, gr[lay.lm:], H, P, V, H, M)
        dx16 = self._ring_write("dx16")
        X_.rmsnorm_bwd(self.X[L], MH, w32[lay.normf:], P, self.RSF, self.DXN, MH, None, self.DX, MH, dx16,
                       gr[lay.normf:], P, self.NORMWORK, M, H, G, 0.0)
        for l in range(L - 1, -1, -1):
            lo = lay.layers[l]
            if self.ckpt:
                self._layer_fwd(l, down=False)  # the layer's activations, recomputed into the slot
            k = 0 if self.ckpt else l
            dgu = self._ring_write("dgu")
            self._gemm(dx16, H, MH, False, w16[lo.down:], Fd, P, True, dgu, 2 * Fd, MF2, M, Fd, H,
                       "swiglu_bwd", aux=self.GU[k], ldx=2 * Fd, sx=MF2, f_half=Fd)
            self._wgrad_async("dx16", f"down{l}", dx16, H, MH, self.ACT[k], Fd, MF, gr[lo.down:], Fd, P, H, Fd, M)
            self._gemm(dgu, 2 * Fd, MF2, False, w16[lo.gu:], H, P, True, self.DXN, H, MH, M, H, 2 * Fd, "f32")
            self._wgrad_async("dgu", f"gu{l}", dgu, 2 * Fd, MF2, self.XN2[k], H, MH, gr[lo.gu:], H, P, 2 * Fd, H, M)
            dx16 = self._ring_write("dx16")
            X_.rmsnorm_bwd(self.HR[k], MH, w32[lo.ln2:], P, self.RS2[k], self.DXN, MH, self.DX, self.DX, MH,
                           dx16, gr[lo.ln2:], P, self.NORMWORK, M, H, G, 0.0)
            self._gemm(dx16, H, MH, False, w16[lo.o:], H, P, True, self.DOUT, H, MH, M, H, H, "bf16")
            self._wgrad_async("dx16", f"o{l}", dx16, H, MH, self.O[k], H, MH, gr[lo.o:], H, P, H, H, M)
            dqkv = self._ring_write("dqkv")
            attn.bwd(self.QKV[k], G * B, S, nh, nkv, self.cos, self.sin, self.O[k], self.LSEA[k], self.DOUT,
                     self.DELTA, dqkv, self.err, self.QKR)
            self._gemm(dqkv, C, MC, False, w16[lo.qkv:], H, P, True, self.DXN, H, MH, M, H, C, "f32")
            self._wgrad_async("dqkv", f"qkv{l}", dqkv, C, MC, self.XN1[k], H, MH, gr[lo.qkv:], H, P, C, H, M)
            dx16 = self._ring_write("dx16")
            X_.rmsnorm_bwd(self.X[l], MH, w32[lo.ln1:], P, self.RS1[k], self.DXN, MH, self.DX, self.DX, MH,
                           dx16, gr[lo.ln1:], P, self.NORMWORK, M, H, G, 0.0)
        emb_n = bb.vocab_size * H
        rows = self.emb_rows
        if rows is None:
            self.GRAD[:, lay.emb:lay.emb + emb_n].zero_()
        X_.embedding_bwd_sorted(ids, self.DX, MH, gr[lay.emb:], P, M, H, G, V, self.EMBKEYS, rows,
                                self.EMBSQ if self.sq_bases is not None else None)
        if side is not None:
            torch.cuda.current_stream(self.dev).wait_event(self._ev_join)
        self._wgrad_join()
        # ---------------- optimizer
        clip = self.e.diloco.inner_grad_clip
        clipv = float(clip) if clip is not None else 0.0
        dl = self.e.diloco
        b1, b2 = dl.inner_betas
        if self.dp > 1:
            # reduce-scatter of the group's gradients + global clip norm, then AdamW on this
            # member's shard storing weights and moments into every member (all-gather)
            X_.dp_grad_reduce_norm(self.dp_tab, self.dp_counter, self.dp_index, self.dp, G, P, P, self.dp_s0,
                                   self.dp_s1, self.CLIPWORK, clipv, self.COEF, self.GNORM, self.err)
            if self.opt8:
                X_.dp_adam8bit(self.dp_tab, self.dp_counter, self.dp_index, self.dp, G, P, self.dp_s0, self.dp_s1,
                               self.COEF, self.SCHED[s], b1, b2, 1e-8, dl.inner_weight_decay, self.err)
            else:
                X_.dp_adamw(self.dp_tab, self.dp_counter, self.dp_index, self.dp, G, P, P, self.dp_s0, self.dp_s1,
                            self.COEF, self.SCHED[s], b1, b2, 1e-8, dl.inner_weight_decay, self.err)
            return
        if self.sq_bases is not None:
            X_.grad_clip_coef_parts(self.SQPARTS, self.sq_nslot, self.EMBSQ, M, self.GRAD, P, self.NORMOFFS, H, G,
                                    clipv, self.COEF, self.GNORM)
        else:
            X_.grad_clip_coef(self.GRAD, P, P, G, clipv, self.CLIPWORK, self.COEF, self.GNORM, rows, lay.emb, H, V)
        if self.opt8:
            X_.adam8bit_step(self.W32.view(-1), self.GRAD.view(-1), self.MQ, self.MABS, self.VQ, self.VLO,
                             self.VSC, self.COEF, self.SCHED[s], b1, b2, 1e-8, dl.inner_weight_decay,
                             False, self.W16.view(-1), P // ALIGN)
        elif self.acc_fused:
            # region-per-CTA AdamW (faster than one path per thread); the round's last
            # step also accumulates the outer pseudo-gradients
            X_.adamw_acc_step(self.W32, self.GRAD, self.MOM1, self.MOM2, self.W16, self.acc_ctas, P, P, self.COEF,
                              self.SCHED[s], b1, b2, 1e-8, dl.inner_weight_decay, rows, lay.emb, H, V, self.ACC_REG,
                              self.acc_nregs, self.ACC_ENT, last)
        else:
            X_.adamw_step(self.W32, self.GRAD, self.MOM1, self.MOM2, self.W16, P, P, P, G, self.COEF,
                          self.SCHED[s], b1, b2, 1e-8, dl.inner_weight_decay, rows, lay.emb, H, V)

    def _layer_fwd(self, l: int, down: bool) -> None:
        """Forward of layer ``l`` from ``X[l]``: RMSNorm -> QKV -> attention -> O (+residual)
        -> RMSNorm -> gate|up (SwiGLU) [-> down (+residual) into ``X[l + 1]``]. Its
        activations go to slot ``l``, or to the one shared slot when checkpointing."""
        X_ = ext()
        bb, G, P = self.bb, self.G, self.P
        H, Fd = bb.hidden_size, bb.intermediate_size
        nh, nkv = bb.num_attention_heads, bb.kv_heads()
        M, C, S, B = self.M, self.C, self.S, self.B
        MH, MC, MF, MF2 = M * H, M * C, M * Fd, M * 2 * Fd
        w32, w16 = self.W32.view(-1), self.W16.view(-1)
        lo = self.layout.layers[l]
        k = 0 if self.ckpt else l
        X_.rmsnorm_fwd(self.X[l], MH, w32[lo.ln1:], P, self.XN1[k], MH, self.RS1[k], M, H, G, self.eps)
        self._gemm(self.XN1[k], H, MH, False, w16[lo.qkv:], H, P, False, self.QKV[k], C, MC, M, C, H, "bf16")
        attn.fwd(self.QKV[k], G * B, S, nh, nkv, self.cos, self.sin, self.O[k], self.LSEA[k], self.err,
                 getattr(self, "QKR", None))
        self._gemm(self.O[k], H, MH, False, w16[lo.o:], H, P, False, self.HR[k], H, MH, M, H, H, "resid",
                   R=self.X[l], ldr=H, sr=MH)
        X_.rmsnorm_fwd(self.HR[k], MH, w32[lo.ln2:], P, self.XN2[k], MH, self.RS2[k], M, H, G, self.eps)
        self._gemm(self.XN2[k], H, MH, False, w16[lo.gu:], H, P, False, self.ACT[k], Fd, MF, M, 2 * Fd, H,
                   "swiglu", bn=128, aux=self.GU[k], ldx=2 * Fd, sx=MF2, f_half=Fd)
        if down:
            self._gemm(self.ACT[k], Fd, MF, False, w16[lo.down:], Fd, P, False, self.X[l + 1], H, MH, M, H, Fd,
                       "resid", R=self.HR[k], ldr=H, sr=MH)

    def _ce_grad_gemms(self, labels, scale, r0: int = 0, rows: int | None = None, beta: float = 0.0,
                       last: bool = True) -> None:
        """The LM-head input and weight gradients straight from the logits: the GEMMs turn
        each staged logits tile into dlogits (exp(x - lse) / count, label column minus
        1 / count; the same bits as the CE kernel's in-place form) before the MMAs read it,
        so the logits are never rewritten. Rows [r0, r0 + rows) of every path; the weight
        gradient is accumulated when ``beta`` is 1 (row chunks)."""
        from ..ops.gemm import gemm_ce_wgrad

        X_ = ext()
        bb, G, P = self.bb, self.G, self.P
        H, V, M = bb.hidden_size, bb.vocab_size, self.M
        mc = M - r0 if rows is None else rows
        lm = self.layout.lm
        w16, gr = self.W16.view(-1), self.GRAD.view(-1)
        lab, ob = labels.view(-1)[r0:], self.CEOB.view(-1)[r0:]
        mch = self.LOGITS.shape[1]
        X_.gemm_ce_grad(self.LOGITS, V, mch * V, False, w16[lm:], H, P, True, self.DXN.view(-1)[r0 * H:], H, M * H,
                        mc, H, V, G, 0.0, self.err, None, 0, 1, ob, lab, scale, M, 1)
        sq = self._sq("lm") if last else {}
        gemm_ce_wgrad(self.LOGITS, V, mch * V, self.XNF.view(-1)[r0 * H:], H, M * H, gr[lm:], H, P, V, H, mc, G,
                      1 if rows is not None else self.wg_split["lm"], self.WGWS, ob, lab, scale, M, sq.get("sq"),
                      sq.get("sq_ld", 0), self.err, beta=beta)

    def _lm_head_chunked(self, s: int, labels) -> None:
        """LM head + loss over row chunks: per chunk the logits GEMM, the chunk's loss rows
        and in-place dlogits (scaled by the WHOLE batch's 1 / count), the input gradient of
        its rows and the weight gradient accumulated over the chunks (fp32, the clip-norm
        box sums on the last chunk); then the loss sum over all rows. The reference's
        chunked loss (src/opendipaco/model.py:157-174) splits the batch the same way."""
        from ..ops.gemm import gemm_wgrad

        X_ = ext()
        bb, G, P = self.bb, self.G, self.P
        H, V = bb.hidden_size, bb.vocab_size
        M, MH, mch = self.M, self.M * bb.hidden_size, self.MCH
        w16, gr = self.W16.view(-1), self.GRAD.view(-1)
        lm = self.layout.lm
        given = self.INVC[s] if self.dp > 1 else None
        if given is None:
            X_.ce_label_count(labels, M, G, self.INVCNT)
        inv = given if given is not None else self.INVCNT
        xnf, dxn = self.XNF.view(-1), self.DXN.view(-1)
        lab, lse, rloss = labels.view(-1), self.LSEC.view(-1), self.ROWLOSS.view(-1)
        last = len(self.chunks) - 1
        for ci, (r0, r1) in enumerate(self.chunks):
            mc = r1 - r0
            a = xnf[r0 * H:]
            if self.ce_fused:
                self._gemm(a, H, MH, False, w16[lm:], H, P, False, self.LOGITS, V, mch * V, mc, V, H, "bf16", bn=128)
                part = None
            else:
                self._gemm(a, H, MH, False, w16[lm:], H, P, False, self.LOGITS, V, mch * V, mc, V, H, "logits",
                           bn=128, part=self.PART)
                part = self.PART
            X_.ce_rows_chunk(self.LOGITS, V, mch * V, lab[r0:], mc, M, V, G, lse[r0:], rloss[r0:], inv, part,
                             self.T, self.err, self.CEOB.view(-1)[r0:] if self.ce_xf else None)
            if self.ce_xf:
                self._ce_grad_gemms(labels, inv, r0, mc, beta=0.0 if ci == 0 else 1.0, last=ci == last)
                continue
            self._gemm(self.LOGITS, V, mch * V, False, w16[lm:], H, P, True, dxn[r0 * H:], H, MH, mc, H, V, "f32")
            sq = self._sq("lm") if ci == last else {}
            gemm_wgrad(self.LOGITS, V, mch * V, a, H, MH, gr[lm:], H, P, V, H, mc, G, 1, self.WGWS, sq.get("sq"),
                       sq.get("sq_ld", 0), self.err, beta=0.0 if ci == 0 else 1.0, bn=self._bn(V, H))
        X_.ce_group_sum(self.ROWLOSS, labels, M, G, self.LOSSSUM, self.INVCNT, self.LOSSES[s], given)

    # ------------------------------------------------------------------ round inputs
    def _prepare(self, corpus, batch_size: int, round_idx: int, slot: int = 0):
        """Sample a round of every owned path's batches (path by path from the engine's
        generator, like the module executor) into host slot ``slot``."""
        steps = self.e.diloco.inner_steps
        shards = [corpus.shard(self.topo.path_index(p)) for p in self.paths]
        return self._prepare_rows(shards, corpus.seq_len, batch_size, [self.e._gen] * self.G,
                                  [round_idx * steps] * self.G, steps, slot)

    def _prepare_rows(self, shards, S: int, batch_size: int, gens, base_steps, steps: int, slot: int = 0):
        """Batches of ``steps`` inner steps for path g from ``shards[g]`` with generator
        ``gens[g]`` (drawn in path order), learning rates from global step
        ``base_steps[g]``; returns the paths' active flags."""
        e = self.e
        active = [sh.size(0) > 0 for sh in shards]
        if batch_size % self.dp:
            raise ValueError(f"batch_size {batch_size} must be divisible by the data-parallel degree {self.dp}")
        B = batch_size // self.dp  # sequences of each step's batch trained on this GPU
        j0 = (self.dp_index if self.dp > 1 else 0) * B
        if self._shape != (B, S, steps):
            self._alloc(B, S, steps)
        hs = self._host[slot]
        ids = hs["ids"].view(steps, self.G, B, S)
        lab = hs["labels"].view(steps, self.G, B, S)
        from .loop import batch_indices

        total = e.total_rounds * steps if e.total_rounds else None
        dl = e.diloco
        b1, b2 = dl.inner_betas
        sched = hs["sched"]
        invc = hs["invc"]
        for g, (sh, act) in enumerate(zip(shards, active)):
            sched[:, g].zero_()
            invc[:, g].fill_(1.0)
            if not act:
                ids[:, g].zero_()
                lab[:, g].fill_(-100)
                continue
            # every step of a round samples the same number of rows: gather the round at once
            idx = torch.stack(batch_indices(sh.size(0), batch_size, steps, gens[g]))  # [steps, rows]
            # the whole batch is sampled (same generator calls on every member), this GPU
            # trains rows [j0, j0 + B); the loss is normalised by the whole batch
            invc[:, g] = 1.0 / max(1, idx.size(1) * (S - 1))
            seqs = sh[idx[:, j0:j0 + B]].to(torch.int32)  # [steps, b, S]
            b = seqs.size(1)
            ids[:, g, :b] = seqs
            lab[:, g, :b, :-1] = seqs[..., 1:]
            lab[:, g, :b, -1] = -100
            if b < B:
                ids[:, g, b:] = 0
                lab[:, g, b:] = -100
            rows = []
            for i in range(steps):
                t = self.steps_taken[g] + i + 1
                lr = inner_lr_at(base_steps[g] + i, total, dl)
                # active flag 2.0 marks a path's very first optimizer step (8-bit Adam
                # then treats the second moment as zero, like the reference)
                rows.append([lr, lr / (1 - b1 ** t), math.sqrt(1 - b2 ** t), 2.0 if t == 1 else 1.0])
            sched[:, g] = torch.tensor(rows, dtype=sched.dtype)
        return active

    def _upload(self, slot: int = 0) -> None:
        hs = self._host[slot]
        self.INVC.copy_(hs["invc"], non_blocking=True)
        self.IDS.copy_(hs["ids"], non_blocking=True)
        self.LABELS.copy_(hs["labels"], non_blocking=True)
        self.SCHED.copy_(hs["sched"], non_blocking=True)

    # ------------------------------------------------------------------ round
    def run_round(self, corpus, batch_size: int, round_idx: int, next_round: int | None = None):
        """One round. ``next_round``: index of the round the caller will certainly run next
        with the same corpus and batch size; its batches are then sampled on the host while
        the GPU runs this round."""
        e = self.e
        steps = e.diloco.inner_steps
        key = (id(corpus), batch_size, round_idx)
        if self._ahead is not None and self._ahead[0] == key and self._shape is not None:
            slot, active = self._ahead[1], self._ahead[2]
        else:
            slot = self._slot
            active = self._prepare(corpus, batch_size, round_idx, slot)
        self._ahead = None
        self._ensure_plan(corpus, active)
        self._upload(slot)
        self._run_inner(steps)
        for g, a in enumerate(active):
            if a:
                self.steps_taken[g] += steps
        if next_round is not None:
            nxt = 1 - slot  # the set this round's copies are not reading from
            self._ahead = ((id(corpus), batch_size, next_round), nxt,
                           self._prepare(corpus, batch_size, next_round, nxt))
            self._slot = nxt
        norms = self._outer(corpus, active)
        last = self.LOSSES[steps - 1]
        if self.dp > 1:
            last = last.clone()
            self.e.backend.dp_allreduce(last)  # partial losses of the group's batch slices
        self.loss_host.copy_(last, non_blocking=True)
        self.status_host.copy_(self.OUTER_STATUS, non_blocking=True)
        self.OUTER_STATUS.zero_()
        torch.cuda.current_stream(self.dev).synchronize()
        check_errors(self.dev)
        bad = int(self.status_host[0])
        if bad:
            self.outer_nonfinite += bad
            log.warning("outer step: %d element(s) with a non-finite pseudo-gradient were left unchanged "
                        "(a path diverged)", bad)
        losses = {p: float(self.loss_host[g]) for g, p in enumerate(self.paths) if active[g]}
        return losses, norms

    def _run_inner(self, steps: int) -> None:
        """Run a round's inner steps: eagerly on the first round (initialises kernel
        attributes), then from one captured CUDA graph."""
        if not self.e.exec.cuda_graphs:
            for s in range(steps):
                self._step(s, last=s == steps - 1)
            return
        if self._graph is None:
            if not self._warm:
                for s in range(steps):
                    self._step(s, last=s == steps - 1)
                self._warm = True
                return
            torch.cuda.synchronize(self.dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for s in range(steps):
                    self._step(s, last=s == steps - 1)
            self._graph = graph
        self._graph.replay()

    # ------------------------------------------------------------------ outer step
    def _delta(self, key: str) -> torch.Tensor:
        """The pseudo-gradient buffer of a shared key: the backend's peer-addressable one
        when it has one (cross-GPU outer step), else a local buffer."""
        if key not in self._deltas:
            be = self.e.backend
            if hasattr(be, "delta_view"):
                self._deltas[key] = be.delta_view(key)
            else:
                self._deltas[key] = torch.zeros(self._region_size(key), device=self.dev, dtype=torch.float32)
        return self._deltas[key]

    def _ensure_plan(self, corpus, active) -> None:
        """Build the outer plan (and the fused-optimizer tables) for these shard weights
        before the round's inner steps run."""
        wkey = (id(corpus), tuple(active))
        if self._plan is None or self._plan_weights != wkey:
            self._plan = self._build_plan(corpus, active)
            self._plan_weights = wkey
            if self.acc_fused:
                self._build_acc_tables()

    def _build_acc_tables(self) -> None:
        """Region / entry tables of ``adamw_acc_step``: per region of the path layout, every
        (path, key) pair sorted by key then path, with the key's pseudo-gradient and global
        buffers and the path's outer weight."""
        order = {k: i for i, k in enumerate(self.topo.module_keys())}
        regions = defaultdict(list)
        for g, path in enumerate(self.paths):
            for key in self.topo.path_module_keys(path):
                regions[self._region(key)].append((order[key], g, key))
        reg, ents, ctas = acc_region_table(regions)
        for ri, ((a, b), lst) in enumerate(sorted(regions.items())):
            lst.sort()
            for idx, (_, g, key) in enumerate(lst):
                last = idx + 1 == len(lst) or lst[idx + 1][2] != key
                delta = 0 if is_private_key(key) else self._delta(key).data_ptr()
                ents.append((delta, self.glob[key].data_ptr(), g, 1 if last else 0, self._acc_w.get((key, g), 0.0),
                             0))
        ent = np.array(ents, dtype=ACC_ENTRY)
        r_t = torch.from_numpy(reg.view(np.int64).copy())
        e_t = torch.from_numpy(ent.view(np.int64).copy())
        if self.ACC_REG is not None and self.ACC_REG.shape == r_t.shape and self.ACC_ENT.shape == e_t.shape:
            # same storage: a captured graph reads the new weights on its next replay
            self.ACC_REG.copy_(r_t)
            self.ACC_ENT.copy_(e_t)
        else:
            self.ACC_REG, self.ACC_ENT = r_t.to(self.dev), e_t.to(self.dev)
            self._graph, self._warm = None, False
        self.acc_nregs, self.acc_ctas = len(reg), ctas

    def _build_plan(self, corpus, active) -> OuterPlan:
        e = self.e
        segs = []
        single = getattr(e.backend, "world_size", 1) == 1
        for key in self.topo.module_keys():
            if key not in e.bank:
                continue
            users = [g for g, p in enumerate(self.paths) if key in self.topo.path_module_keys(p)]
            loc32, loc16, w = [], [], []
            for g in users:
                a, b = self._local_region(g, key)
                loc32.append(self.W32[g, a:b])
                loc16.append(self.W16[g, a:b])
                pidx = self.topo.path_index(self.paths[g])
                lead = self.dp == 1 or self.dp_index == 0  # a path's DP replicas hold the same delta
                w.append(e._outer_weight(key, pidx, corpus) if active[g] and lead else 0.0)
                self._acc_w[(key, g)] = w[-1]
            if is_private_key(key):
                # with the fused optimizer the last inner step already copied it
                if users and not self.acc_fused:
                    segs.append(Segment(key, self.glob[key], None, loc32[:1], [None], [1.0], mode=MODE_COPY))
                continue
            # the normaliser is global: every path through the key with a non-empty shard
            den = 0.0
            for p in self.topo.paths_through_module(key):
                pi = self.topo.path_index(p)
                if corpus.shard(pi).size(0) > 0:
                    den += e._outer_weight(key, pi, corpus)
            inv = 1.0 / max(den, 1e-12) if e.diloco.normalize_outer_delta else 1.0
            # one GPU with the fused optimizer: the pseudo-gradient is ready, apply it;
            # cross-GPU backends split OUTER segments into their own phases
            mode = MODE_APPLY if (self.acc_fused and single) else MODE_OUTER
            segs.append(Segment(key, self.glob[key], self.mom[key], loc32, loc16, w, mode,
                                e.outer_scale(key), inv, self._delta(key) if self.acc_fused else None))
        plan = OuterPlan(segs, self.dev)
        plan.build()
        return plan

    def _outer(self, corpus, active):
        e = self.e
        self._ensure_plan(corpus, active)
        backend = e.backend
        dl = e.diloco
        if getattr(backend, "world_size", 1) > 1:
            if not hasattr(backend, "fused_outer_step"):
                raise NotImplementedError("multi-rank fused outer step needs a backend with fused_outer_step")
            backend.fused_outer_step(self, self._plan, first=self.outer_steps == 0)
            norms = backend.delta_norms()
        else:
            self._plan.run(dl.outer_lr, dl.outer_momentum, dl.outer_nesterov, first=self.outer_steps == 0,
                           status=self.OUTER_STATUS)
            norms = self._plan.delta_norms()
        self.outer_steps += 1
        return [v for k, v in norms.items() if not is_private_key(k)]

    # ------------------------------------------------------------------ benchmarking hooks
    def device_round(self) -> None:
        """Replay one round's device work (inner-step graph + outer step) on the inputs
        already resident on the device: no host preparation, copies or reads."""
        self._run_inner(self.e.diloco.inner_steps)
        self.device_outer()

    def device_outer(self) -> None:
        """Only the outer step (pseudo-gradient reduce + Nesterov + write-back) of a round."""
        dl = self.e.diloco
        if getattr(self.e.backend, "world_size", 1) > 1:
            self.e.backend.fused_outer_step(self, self._plan, first=False)
        else:
            self._plan.run(dl.outer_lr, dl.outer_momentum, dl.outer_nesterov, first=False, status=self.OUTER_STATUS)

    def launches_per_round(self) -> int:
        """Kernels of this package launched per round (inner steps + outer step)."""
        per_step = (14 + 22 * self.L + (2 if self.dp > 1 else 0) - (1 if self.sq_bases is not None else 0)
                    + sum(1 for sp in self.wg_split.values() if sp > 1))
        if self.ckpt:  # recomputed layer forwards (all but the down projection): 6 launches each
            per_step += 6 * self.L
        if self.QKR is not None:  # flash attention: rotation pass in forward and backward, two backward kernels
            per_step += 3 * self.L + (self.L if self.ckpt else 0)
        if len(self.chunks) > 1:
            # chunked LM head: label count + per chunk (logits, CE rows (two kernels from
            # GEMM partials), dX, dW) + group sum, against 6 launches (+ a split-K reduce)
            per_chunk = 4 if self.ce_fused else 5
            per_step += per_chunk * len(self.chunks) + 2 - 6 - (1 if self.wg_split.get("lm", 1) > 1 else 0)
        be = self.e.backend
        outer = be.outer_launch_count(self) if getattr(be, "world_size", 1) > 1 else 1
        return self.e.diloco.inner_steps * per_step + outer

    def h2d_bytes_per_round(self) -> int:
        return int(self.IDS.numel() * 4 + self.LABELS.numel() * 4 + self.SCHED.numel() * 4 + self.INVC.numel() * 4)

    def d2h_bytes_per_round(self) -> int:
        chunks = self._plan.total_chunks if self._plan is not None else 0
        return int(self.G * 4 + 4 + chunks * 4 + 4)  # losses, error word, delta-norm partials, guard status

    # ------------------------------------------------------------------ API glue
    def path_model(self, path: Path) -> nn.Module:
        return self.pms[path]

    def sync_bank_views(self) -> None:
        """Bank parameters already alias the flat buffers; nothing to copy."""
        torch.cuda.current_stream(self.dev).synchronize()

    def _inner_opt(self, path: Path) -> torch.optim.Optimizer:
        if path not in self._inner_opts:
            self._inner_opts[path] = make_inner_optimizer(self.pms[path], self.e.diloco)
        return self._inner_opts[path]

    def inner_state_dicts(self) -> dict[Path, dict]:
        from .loop import _opt_state_cpu

        out = {}
        for g, path in enumerate(self.paths):
            opt = self._inner_opt(path)
            opt.state.clear()
            t = self.steps_taken[g]
            if t > 0:
                for name, p in self.pms[path].named_parameters():
                    s, o, n = self.layout.by_name[name]
                    if self.opt8:
                        nb0, nbn = o // ALIGN, (n + ALIGN - 1) // ALIGN
                        base = g * (self.P // ALIGN)
                        sl = slice(base + nb0, base + nb0 + nbn)
                        opt.state[p] = {"step": t, "m_q": self.MQ[sl], "m_absmax": self.MABS[sl],
                                        "v_q": self.VQ[sl], "v_lo": self.VLO[sl], "v_scale": self.VSC[sl]}
                    else:
                        opt.state[p] = {"step": torch.tensor(float(t)),
                                        "exp_avg": self.MOM1[g, o:o + n].view(s),
                                        "exp_avg_sq": self.MOM2[g, o:o + n].view(s)}
            out[path] = _opt_state_cpu(opt.state_dict())
            opt.state.clear()
        return out

    def outer_state_dict(self) -> dict:
        from .loop import _opt_state_cpu

        opt = self.e.outer_opt
        opt.state.clear()
        if self.outer_steps > 0 and hasattr(self.e.backend, "gather_momentum"):
            self.e.backend.gather_momentum(self)
        if self.outer_steps > 0:
            for key, mod in self.e.bank.items():
                if is_private_key(key):
                    continue
                rel = {n: (s, o, k) for n, s, o, k in self._rel_entries(key)}
                for name, p in mod.named_parameters():
                    s, o, k = rel[name]
                    opt.state[p] = {"momentum_buffer": self.mom[key][o:o + k].view(s)}
        sd = _opt_state_cpu(opt.state_dict())
        opt.state.clear()
        return sd

    @torch.no_grad()
    def load_states(self, outer_sd: dict, inner: dict) -> None:
        e = self.e
        opt = e.outer_opt
        opt.load_state_dict(outer_sd)
        self.outer_steps = 0
        for key, mod in e.bank.items():
            if is_private_key(key):
                continue
            rel = {n: (s, o, k) for n, s, o, k in self._rel_entries(key)}
            for name, p in mod.named_parameters():
                st = opt.state.get(p, {})
                if "momentum_buffer" in st and st["momentum_buffer"] is not None:
                    s, o, k = rel[name]
                    self.mom[key][o:o + k].copy_(st["momentum_buffer"].reshape(-1))
                    self.outer_steps = 1
        opt.state.clear()
        # working copies = bank for shared keys; private keys = bank (authoritative)
        for g, path in enumerate(self.paths):
            for key in self.pms[path].modules_by_key():
                if key in self.glob:
                    a, b = self._local_region(g, key)
                    self.W32[g, a:b].copy_(self.glob[key])
        self.W16.copy_(self.W32)
        if not self.opt8:
            self.MOM1.zero_()
            self.MOM2.zero_()
        for g, path in enumerate(self.paths):
            self.steps_taken[g] = 0
            if path not in inner:
                continue
            iopt = self._inner_opt(path)
            iopt.load_state_dict(inner[path])
            for name, p in self.pms[path].named_parameters():
                st = iopt.state.get(p)
                if not st:
                    continue
                s, o, n = self.layout.by_name[name]
                step = st["step"]
                self.steps_taken[g] = int(step.item() if torch.is_tensor(step) else step)
                if self.opt8:
                    nb0, nbn = o // ALIGN, (n + ALIGN - 1) // ALIGN
                    base = g * (self.P // ALIGN)
                    sl = slice(base + nb0, base + nb0 + nbn)
                    self.MQ[sl].copy_(st["m_q"])
                    self.MABS[sl].copy_(st["m_absmax"])
                    self.VQ[sl].copy_(st["v_q"])
                    self.VLO[sl].copy_(st["v_lo"])
                    self.VSC[sl].copy_(st["v_scale"])
                else:
                    self.MOM1[g, o:o + n].copy_(st["exp_avg"].reshape(-1))
                    self.MOM2[g, o:o + n].copy_(st["exp_avg_sq"].reshape(-1))
            iopt.state.clear()
        self._graph = None
        self._warm = False


__all__ = ["FusedExecutor", "PathLayout", "Adam8bit"]
