"""Wire compression for DiLoCo traffic (reference ``src/opendipaco/schedule/compress.py``).

Modes ``none | bf16 | int8 | int4``. Weights travel bf16 in any non-"none" mode;
pseudo-gradients travel int8 (per-tensor symmetric, absmax/127) or int4 (one scale
per group of 128, values in [-7, 7] stored +8, two per byte, high nibble first),
optionally top-k sparsified (per output row for 2-D tensors), with worker-side
error feedback (the residual is added to the next round's delta). Down-link deltas
against a keyframe (``encode_state_delta`` / ``apply_state_delta``) and
self-describing decode (``maybe_dequantize``, Byzantine-hardened: every length and
index is validated before use).

The payload dicts (``{"q","s"}``, ``{"q4","s","g","n","shape"}``,
``{"sp","i","v"}``) are the wire contract and match the reference exactly. On CUDA
tensors quantisation, residual and decode run in the ``csrc/codec.cu`` kernels;
on CPU the same math runs in PyTorch.
"""

from __future__ import annotations

import hashlib
import math
import struct

import torch

MODES = ("none", "bf16", "int8", "int4")
INT4_GROUP = 128


def check_mode(mode: str) -> str:
    if mode not in MODES:
        raise ValueError(f"compress must be one of {MODES}, got {mode!r}")
    return mode


def compress_state(sd: dict, mode: str) -> dict:
    if mode == "none":
        return sd
    return {n: v.to(torch.bfloat16) if v.is_floating_point() else v for n, v in sd.items()}


def compress_shard(shard, mode: str):
    return shard if shard is None or mode == "none" else shard.to(torch.int32)


def restore_shard(shard):
    return None if shard is None else shard.long()


def _quantize_int8(t: torch.Tensor) -> tuple[dict, torch.Tensor]:
    t = t.detach().float()
    if t.is_cuda and t.numel():
        from ..ops import codec

        q, scale, r = codec.quant_int8(t)
        return {"q": q.cpu(), "s": scale}, r
    absmax = float(t.abs().max()) if t.numel() else 0.0
    scale = absmax / 127.0
    if scale == 0.0:
        return {"q": torch.zeros(t.shape, dtype=torch.int8), "s": 0.0}, t.clone()
    q = torch.round(t / scale).clamp_(-127, 127).to(torch.int8)
    return {"q": q, "s": scale}, t - q.float() * scale


def _quantize_int4(t: torch.Tensor, group_size: int = INT4_GROUP):
    flat = t.detach().reshape(-1).float()
    n = flat.numel()
    if flat.is_cuda and group_size == INT4_GROUP and n:
        from ..ops import codec

        packed, scale, resid = codec.quant_int4(flat)
        return ({"q4": packed, "s": scale, "g": group_size, "n": n, "shape": list(t.shape)},
                resid.reshape(t.shape))
    pad = -n % group_size
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    grp = flat.reshape(-1, group_size)
    scale = grp.abs().amax(dim=1, keepdim=True) / 7.0
    q = torch.round(grp / torch.where(scale > 0, scale, torch.ones_like(scale))).clamp_(-7, 7)
    recon = (q * scale).reshape(-1)[:n].reshape(t.shape)
    qu = (q + 8).to(torch.uint8).reshape(-1)
    packed = (qu[0::2] << 4 | qu[1::2]).contiguous()
    return ({"q4": packed, "s": scale.reshape(-1).float(), "g": group_size, "n": n, "shape": list(t.shape)},
            t.detach().float() - recon)


def _dequant_int4(p: dict) -> torch.Tensor:
    packed, scale = p.get("q4"), p.get("s")
    g, n = int(p.get("g", 0)), int(p.get("n", -1))
    if not (torch.is_tensor(packed) and torch.is_tensor(scale)) or g <= 0 or n < 0:
        raise ValueError("malformed int4 payload")
    ng = (n + g - 1) // g
    if scale.numel() != ng or packed.numel() != ng * g // 2:
        raise ValueError("malformed int4 payload: length mismatch")
    if packed.is_cuda and g % 2 == 0:
        from ..ops import codec

        return codec.dequant_int4(packed, scale, n, g)
    pk = packed.to(torch.int16)
    qu = torch.stack([pk >> 4 & 15, pk & 15], dim=1).reshape(-1)
    q = (qu.float() - 8.0).reshape(-1, g)
    return (q * scale.reshape(-1, 1).float()).reshape(-1)[:n]


def _digest_update(h, t: torch.Tensor) -> None:
    payload, _ = _quantize_int8(t.detach().cpu())
    s = payload["s"]
    h.update(struct.pack(">q", round(math.log(s) * 1000.0) if s > 0 else 0))
    h.update(payload["q"].numpy().tobytes())


def pseudograd_digest(shared_delta: dict) -> str:
    """sha256 over int8-quantised tensors + log-scale buckets (agreement between
    redundant executions tolerates float noise below the int8 step)."""
    h = hashlib.sha256()
    for key in sorted(shared_delta):
        h.update(key.encode())
        for t in shared_delta[key]:
            _digest_update(h, t)
    return h.hexdigest()


def state_digest(state: dict) -> str:
    h = hashlib.sha256()
    for name in sorted(state):
        h.update(name.encode())
        t = state[name]
        if not torch.is_floating_point(t):
            h.update(t.cpu().numpy().tobytes())
        else:
            _digest_update(h, t)
    return h.hexdigest()


def _sparsify(d: torch.Tensor, density: float, mode: str):
    d = d.detach()
    if d.dim() == 2:
        rows, cols = d.shape
        k = max(1, math.ceil(density * cols))
        idx = d.abs().topk(k, dim=1).indices
        kept = torch.gather(d, 1, idx).reshape(-1)
        flat_idx = (torch.arange(rows, device=d.device).unsqueeze(1) * cols + idx).reshape(-1)
    else:
        flat = d.reshape(-1)
        k = max(1, math.ceil(density * flat.numel()))
        flat_idx = flat.abs().topk(k).indices
        kept = flat[flat_idx]
    if mode == "int8":
        enc, _ = _quantize_int8(kept)
        vals = enc["q"].float().to(d.device) * enc["s"]
    elif mode == "int4":
        enc, _ = _quantize_int4(kept)
        vals = _dequant_int4(enc)
    elif mode == "bf16":
        enc = kept.to(torch.bfloat16)
        vals = enc.float()
    else:
        enc = vals = kept.float()
    dense = torch.zeros(d.numel(), dtype=torch.float32, device=d.device)
    dense[flat_idx] = vals
    return {"sp": list(d.shape), "i": flat_idx.to(torch.int32), "v": enc}, dense.reshape(d.shape)


def compress_delta(delta, mode: str, carry=None, density: float = 1.0):
    """Encode one module's pseudo-gradient list; returns (payload list, residual list)."""
    if mode == "none" and density >= 1.0:
        return list(delta), None
    if carry is not None:
        delta = [d + c for d, c in zip(delta, carry)]
    payload, residual = [], []
    for d in delta:
        if density < 1.0:
            p, recon = _sparsify(d, density, mode)
            payload.append(p)
            residual.append(d.detach().float() - recon)
        elif mode == "bf16":
            c = d.detach().to(torch.bfloat16)
            payload.append(c)
            residual.append(d.detach().float() - c.float())
        elif mode == "int4":
            p, r = _quantize_int4(d)
            payload.append(p)
            residual.append(r)
        else:
            p, r = _quantize_int8(d)
            payload.append(p)
            residual.append(r)
    return payload, residual


def encode_state_delta(cur: dict, base: dict, mode: str = "int8") -> dict:
    out = {}
    for n, c in cur.items():
        b = base.get(n)
        if c.is_floating_point() and b is not None and b.shape == c.shape:
            d = c.float() - b.float()
            out[n] = _quantize_int4(d)[0] if mode == "int4" else _quantize_int8(d)[0]
        else:
            out[n] = c
    return out


def apply_state_delta(base: dict, tensors: dict) -> dict:
    out = {}
    for n, t in tensors.items():
        if isinstance(t, dict) and "q" in t and torch.is_tensor(t["q"]):
            b = base[n]
            if t["q"].shape != b.shape:
                raise ValueError(f"int8 delta shape {tuple(t['q'].shape)} != base {tuple(b.shape)}")
            out[n] = b.float() + t["q"].float().to(b.device) * float(t["s"])
        elif isinstance(t, dict) and "q4" in t:
            b = base[n]
            deq = _dequant_int4(t)
            if deq.numel() != b.numel():
                raise ValueError(f"int4 delta has {deq.numel()} elems != base {b.numel()}")
            out[n] = b.float() + deq.reshape(b.shape).to(b.device)
        elif torch.is_tensor(t):
            out[n] = t
        else:
            raise TypeError(f"not a state-delta entry: {type(t)}")
    return out


def maybe_dequantize(items) -> list[torch.Tensor]:
    """Self-describing decode of a pseudo-gradient list to fp32 (validated)."""
    out = []
    for it in items:
        if torch.is_tensor(it):
            out.append(it if it.dtype == torch.float32 else it.float())
        elif isinstance(it, dict) and "q" in it and torch.is_tensor(it["q"]):
            out.append(it["q"].float() * float(it["s"]))
        elif isinstance(it, dict) and "q4" in it:
            deq = _dequant_int4(it)
            shape = [int(s) for s in it["shape"]]
            if any(s < 0 for s in shape) or math.prod(shape) != deq.numel():
                raise ValueError("int4 payload: shape does not match element count")
            out.append(deq.reshape(shape))
        elif isinstance(it, dict) and "sp" in it and torch.is_tensor(it.get("i")):
            shape = [int(s) for s in it["sp"]]
            v = it["v"]
            if isinstance(v, dict) and "q" in v:
                vals = v["q"].float() * float(v["s"])
            elif isinstance(v, dict) and "q4" in v:
                vals = _dequant_int4(v)
            elif torch.is_tensor(v):
                vals = v.float()
            else:
                raise TypeError(f"not a sparse-payload value: {type(v)}")
            if any(s < 0 for s in shape):
                raise ValueError("sparse payload: negative shape dim")
            n = math.prod(shape)
            idx, vals = it["i"].long().reshape(-1), vals.reshape(-1)
            if idx.numel() != vals.numel():
                raise ValueError("sparse payload: index/value length mismatch")
            if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= n):
                raise ValueError("sparse payload: index out of range")
            dense = torch.zeros(n, dtype=torch.float32, device=vals.device)
            dense[idx.to(vals.device)] = vals
            out.append(dense.reshape(shape))
        else:
            raise TypeError(f"not a pseudo-gradient tensor: {type(it)}")
    return out
