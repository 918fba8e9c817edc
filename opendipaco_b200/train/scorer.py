"""Scoring many paths at once: forward-only CE of token batches under G paths in one
set of grouped launches.

EM re-sharding scores every document under every candidate path, and routed evaluation
scores each path's routed sequences; run path by path through the module forward, that
is G times the launches of one small forward (reference ``src/opendipaco/em.py:36-70``,
``src/opendipaco/inference.py:55-104``). :class:`GroupedScorer` instead keeps the G
paths' weights side by side in flat ``[G, P]`` arenas (the fused executor's layout) and
runs one forward for all of them with the same grouped kernels as training: embedding
gather, per layer RMSNorm -> QKV GEMM -> tcgen05 attention (RoPE fused) -> O GEMM
(+residual) -> RMSNorm -> gate|up GEMM (SwiGLU) -> down GEMM (+residual), final RMSNorm,
then the LM head over row chunks (bf16 logits GEMM, per-row CE kernel) so at most one
chunk of logits exists. Activations are kept for one layer only (nothing runs backward),
the residual stream ping-pongs between two buffers.

The layer forward and the GEMM dispatch are the fused executor's own methods, so the
scorer computes exactly what a training step's forward computes (bf16 GEMMs, fp32
residual stream and norms).
"""

from __future__ import annotations

import torch
from torch import nn

from ..config import DiPaCoConfig
from ..models.llama import rope_cos_sin
from ..models.path import build_path_model
from ..ops._ext import check_errors, err_word, ext
from ..ops.loss import cross_entropy_rows
from ..topology import Path
from .fused import FusedExecutor, PathLayout


class _PingPong:
    """``X[l]`` of the layer forward over two buffers (layer l reads l % 2, writes (l+1) % 2)."""

    def __init__(self, buf: torch.Tensor):
        self.buf = buf

    def __getitem__(self, i: int) -> torch.Tensor:
        return self.buf[i % 2]


class GroupedScorer:
    """Forward-only per-token CE of ``G`` paths over batches of ``B`` sequences of length
    ``S`` (a multiple of 64)."""

    _layer_fwd = FusedExecutor._layer_fwd
    _gemm = FusedExecutor._gemm
    _bn = FusedExecutor._bn

    @staticmethod
    def supported(config: DiPaCoConfig, device: torch.device) -> bool:
        bb = config.backbone
        if device.type != "cuda" or config.tie_word_embeddings or bb.head_dim != 64 or bb.hidden_size % 128:
            return False
        from ..ops._ext import available

        return available()

    def __init__(self, config: DiPaCoConfig, bank: dict[str, nn.Module], device: torch.device, groups: int,
                 batch: int, seq_len: int, logit_bytes: int = 1 << 30):
        if seq_len % 64:
            raise ValueError("GroupedScorer needs seq_len % 64 == 0")
        self.config, self.bank, self.dev = config, bank, device
        self.topo = config.build_topology()
        bb = self.bb = config.backbone
        from ..ops.gemm import sm_count

        self.sms = sm_count(device)
        probe = build_path_model(config, self.topo.path_from_index(0), bank, deepcopy=False)
        self.layout = PathLayout(probe, config)
        self.G, self.P, self.B, self.S = groups, self.layout.P, batch, seq_len
        G, P, B, S = self.G, self.P, self.B, self.S
        H, Fd, V = bb.hidden_size, bb.intermediate_size, bb.vocab_size
        nh, nkv = bb.num_attention_heads, bb.kv_heads()
        self.C = (nh + 2 * nkv) * 64
        self.M = M = B * S
        self.L = len(self.layout.layers)
        self.eps = bb.rms_norm_eps
        self.ckpt = True  # one activation slot: every layer's activations land in slot 0
        f32, b16 = torch.float32, torch.bfloat16
        z = lambda *s, dt=f32: torch.empty(*s, device=device, dtype=dt)  # noqa: E731
        self.W32 = torch.zeros(G, P, device=device)
        self.W16 = torch.zeros(G, P, device=device, dtype=b16)
        self.X = _PingPong(z(2, G, M, H))
        self.HR, self.RS1, self.RS2 = z(1, G, M, H), z(1, G, M), z(1, G, M)
        self.XN1, self.XN2 = z(1, G, M, H, dt=b16), z(1, G, M, H, dt=b16)
        self.QKV, self.O = z(1, G, M, self.C, dt=b16), z(1, G, M, H, dt=b16)
        self.LSEA = z(1, G * B, nh, S)
        self.GU, self.ACT = z(1, G, M, 2 * Fd, dt=b16), z(1, G, M, Fd, dt=b16)
        self.XNF, self.RSF = z(G, M, H, dt=b16), z(G, M)
        # LM head over chunks of whole sequences: at most `logit_bytes` of bf16 logits
        rows = max(S, min(M, (logit_bytes // (2 * V * G)) // S * S))
        self.chunks = [(r0, min(M, r0 + rows)) for r0 in range(0, M, rows)]
        self.LOGITS = z(G, rows, V, dt=b16)
        self.cos, self.sin = rope_cos_sin(64, bb.rope_theta, S, device)
        self.err = err_word(device)
        self.paths: list[Path | None] = [None] * G

    @torch.no_grad()
    def load(self, g: int, path: Path) -> None:
        """Copy ``path``'s modules from the bank into group ``g``."""
        if self.paths[g] == path:
            return
        pm = build_path_model(self.config, path, self.bank, deepcopy=False)
        for name, p in pm.named_parameters():
            shape, off, n = self.layout.by_name[name]
            self.W32[g, off:off + n].copy_(p.detach().reshape(-1))
        self.W16[g].copy_(self.W32[g])
        self.paths[g] = path

    def invalidate(self) -> None:
        """Forget which paths are loaded (the bank's weights changed)."""
        self.paths = [None] * self.G

    @torch.no_grad()
    def token_losses(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """``ids`` [G, B, S] token ids, ``targets`` [G, B, S] next-token targets (< 0:
        not scored) -> [G, B, S] fp32 CE per position (0 where not scored)."""
        G, B, S = self.G, self.B, self.S
        if ids.shape != (G, B, S) or targets.shape != (G, B, S):
            raise ValueError(f"GroupedScorer: expected [{G}, {B}, {S}] ids and targets")
        X_ = ext()
        H, V, M, P = self.bb.hidden_size, self.bb.vocab_size, self.M, self.P
        lay = self.layout
        ids32 = ids.to(self.dev, torch.int32).reshape(G, M).contiguous()
        tgt = targets.to(self.dev, torch.long).reshape(G, M)
        w32, w16 = self.W32.view(-1), self.W16.view(-1)
        X_.embedding_fwd(ids32, w32[lay.emb:], P, self.X[0], M, H, G, V)
        for l in range(self.L):
            self._layer_fwd(l, down=True)
        X_.rmsnorm_fwd(self.X[self.L], M * H, w32[lay.normf:], P, self.XNF, M * H, self.RSF, M, H, G, self.eps)
        out = torch.empty(G, M, device=self.dev)
        xnf = self.XNF.view(-1)
        rows = self.LOGITS.size(1)
        for r0, r1 in self.chunks:
            mc = r1 - r0
            self._gemm(xnf[r0 * H:], H, M * H, False, w16[lay.lm:], H, P, False, self.LOGITS, V, rows * V, mc, V, H,
                       "bf16", bn=128)
            if mc == rows:
                out[:, r0:r1] = cross_entropy_rows(self.LOGITS.view(G * mc, V), tgt[:, r0:r1].reshape(-1)).view(G, mc)
            else:  # a shorter last chunk: rows of one group are contiguous
                for g in range(G):
                    out[g, r0:r1] = cross_entropy_rows(self.LOGITS[g, :mc], tgt[g, r0:r1])
        check_errors(self.dev)
        return out.view(G, B, S)


def padded_len(n: int) -> int:
    return max(64, (n + 63) // 64 * 64)


def group_count(config: DiPaCoConfig, bank: dict[str, nn.Module], wanted: int, budget: int = 8 << 30) -> int:
    """How many paths to score side by side: ``wanted``, capped so the weight arenas (6
    bytes per parameter per path) stay within ``budget``."""
    topo = config.build_topology()
    n = sum(p.numel() for k in topo.path_module_keys(topo.path_from_index(0)) for p in bank[k].parameters())
    return max(1, min(wanted, budget // max(1, 6 * n)))


def shifted_targets(ids: torch.Tensor, valid: torch.Tensor, first: int = 1) -> torch.Tensor:
    """Next-token targets of [B, S] ``ids``: position t predicts ids[t + 1] when that token
    is valid and t + 1 >= ``first``; every other position is -100 (not scored)."""
    tgt = torch.full_like(ids, -100)
    ok = valid[:, 1:].clone()
    if first > 1:
        ok[:, :first - 1] = False
    tgt[:, :-1] = torch.where(ok, ids[:, 1:], torch.full_like(ids[:, 1:], -100))
    return tgt


__all__ = ["GroupedScorer", "group_count", "padded_len", "shifted_targets"]
