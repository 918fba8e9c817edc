"""Blockwise 8-bit AdamW: moments stored in int8 blocks of 256.

Reference: ``src/opendipaco/optim/adam8bit.py:23-156``. The state-dict layout is
part of the checkpoint format and is kept: per parameter ``step`` (int),
``m_q [nb, 256] int8`` + ``m_absmax [nb]`` (symmetric absmax/127 per block) and
``v_q [nb, 256] uint8`` + ``v_lo [nb]`` + ``v_scale [nb]`` (the second moment
quantised in the *log* domain, floor 1e-20, so small values in a
mixed-magnitude block never collapse to zero).

The update is AdamW (decoupled weight decay, bias correction, eps 1e-8) on the
dequantised moments. On CUDA parameters the whole dequantise -> update ->
requantise runs in one sm_100a kernel (``opendipaco_b200/csrc/adam.cu``, one
warp per 256-element block, moments never leave registers); on CPU it runs the
same math in chunked PyTorch ops.
"""

from __future__ import annotations

import torch
from torch.optim import Optimizer

BLOCK = 256
V_FLOOR = 1e-20
_CHUNK = 1 << 22


def _blocks(t: torch.Tensor, bs: int) -> torch.Tensor:
    flat = t.reshape(-1)
    pad = (-flat.numel()) % bs
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    return flat.view(-1, bs)


def quantize_m(m: torch.Tensor, bs: int = BLOCK):
    b = _blocks(m, bs)
    absmax = b.abs().amax(dim=1)
    scale = torch.where(absmax > 0, absmax / 127.0, torch.ones_like(absmax))
    q = torch.round(b / scale[:, None]).clamp_(-127, 127).to(torch.int8)
    return q, absmax


def dequantize_m(q: torch.Tensor, absmax: torch.Tensor) -> torch.Tensor:
    return (q.float() * (absmax / 127.0)[:, None]).reshape(-1)


def quantize_v(v: torch.Tensor, bs: int = BLOCK):
    lv = torch.log(_blocks(v, bs).clamp_min(V_FLOOR))
    lo = lv.amin(dim=1)
    scale = ((lv.amax(dim=1) - lo) / 255.0).clamp_min(1e-12)
    q = torch.round((lv - lo[:, None]) / scale[:, None]).clamp_(0, 255).to(torch.uint8)
    return q, lo, scale


def dequantize_v(q: torch.Tensor, lo: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return torch.exp(q.float() * scale[:, None] + lo[:, None]).reshape(-1)


class Adam8bit(Optimizer):
    """AdamW with blockwise-int8 moment storage."""

    def __init__(self, params, lr: float, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, block_size: int = BLOCK):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      block_size=block_size))

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        for st in self.state.values():
            if "m_q" in st:
                st["m_q"] = st["m_q"].to(torch.int8)
                st["v_q"] = st["v_q"].to(torch.uint8)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            b1, b2 = group["betas"]
            lr, eps, wd, bs = group["lr"], group["eps"], group["weight_decay"], group["block_size"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    nb = (p.numel() + bs - 1) // bs
                    st["step"] = 0
                    st["m_q"] = torch.zeros((nb, bs), dtype=torch.int8, device=p.device)
                    st["m_absmax"] = torch.zeros(nb, device=p.device)
                    st["v_q"] = torch.zeros((nb, bs), dtype=torch.uint8, device=p.device)
                    st["v_lo"] = torch.zeros(nb, device=p.device)
                    st["v_scale"] = torch.zeros(nb, device=p.device)
                first = st["step"] == 0
                st["step"] += 1
                t = st["step"]
                bc1, bc2s = 1 - b1 ** t, (1 - b2 ** t) ** 0.5
                if p.is_cuda and bs == BLOCK:
                    from ..ops import adam as K

                    K.adam8bit_step(p, p.grad, st, lr=lr, b1=b1, b2=b2, eps=eps, wd=wd,
                                    bc1=bc1, bc2_sqrt=bc2s, first=first)
                else:
                    _step_cpu(p, st, b1, b2, lr, eps, wd, bs, bc1, bc2s, first)
        return loss


def _step_cpu(p, st, b1, b2, lr, eps, wd, bs, bc1, bc2s, first):
    g, flat = p.grad.reshape(-1), p.data.reshape(-1)
    nb, n = st["m_q"].shape[0], p.numel()
    per = max(1, _CHUNK // bs)
    for c0 in range(0, nb, per):
        c1 = min(c0 + per, nb)
        e0, e1 = c0 * bs, min(c1 * bs, n)
        gc = g[e0:e1]
        if gc.numel() < (c1 - c0) * bs:
            gc = torch.cat([gc, gc.new_zeros((c1 - c0) * bs - gc.numel())])
        m = dequantize_m(st["m_q"][c0:c1], st["m_absmax"][c0:c1])
        v = torch.zeros_like(gc) if first else dequantize_v(
            st["v_q"][c0:c1], st["v_lo"][c0:c1], st["v_scale"][c0:c1])
        m.mul_(b1).add_(gc, alpha=1 - b1)
        v.mul_(b2).addcmul_(gc, gc, value=1 - b2)
        st["m_q"][c0:c1], st["m_absmax"][c0:c1] = quantize_m(m, bs)
        st["v_q"][c0:c1], st["v_lo"][c0:c1], st["v_scale"][c0:c1] = quantize_v(v, bs)
        k = e1 - e0
        denom = (v[:k].sqrt() / bc2s).add_(eps)
        flat[e0:e1].mul_(1 - lr * wd).addcdiv_(m[:k], denom, value=-lr / bc1)
