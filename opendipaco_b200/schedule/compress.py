"""Compression of the DiLoCo traffic between workers and servers.

Modes: ``none | bf16 | int8 | int4``. Weights sent down travel bf16 in every mode but
"none". Pseudo-gradients sent up are encoded per tensor by one of three payload codecs,
optionally after top-k sparsification, and the worker keeps what the encoding lost as an
error-feedback residual that is added to its next round's delta. Down-link weight deltas
against a keyframe use the same codecs (``encode_state_delta`` / ``apply_state_delta``).

Payload dicts are a wire contract with the reference (``src/opendipaco/schedule/
compress.py``), so either framework decodes the other's uploads:

* int8:   ``{"q": int8 tensor (shape of the input), "s": float}`` -- one symmetric
  absmax / 127 scale per tensor;
* int4:   ``{"q4": uint8 [ceil(n / g) * g / 2], "s": fp32 [ceil(n / g)], "g": 128, "n": n,
  "shape": [...]}`` -- one absmax / 7 scale per group of g, codes q + 8 in [1, 15], two per
  byte with the even element in the HIGH nibble;
* sparse: ``{"sp": shape, "i": int32 flat indices, "v": values}`` where the values are a
  plain tensor (none / bf16) or an int8 / int4 payload; 2-D tensors keep the top
  ceil(density * columns) entries of every row, others the top ceil(density * n) overall.

Decoding validates every length, shape and index before use (uploads come from peers
that may be faulty or hostile). The digests used by redundant-execution audits are also
shared with the reference: sha256 over the key names and, per tensor, its int8 codes and
a scale bucket ``round(1000 ln s)``. On CUDA tensors the int8 / int4 encoders and the int4
decoder run in ``csrc/codec.cu``; on CPU the same arithmetic runs in PyTorch.
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


# ------------------------------------------------------------------ payload codecs
class _Int8:
    """Per-tensor symmetric int8."""

    @staticmethod
    def matches(obj) -> bool:
        return isinstance(obj, dict) and torch.is_tensor(obj.get("q"))

    @staticmethod
    def encode(t: torch.Tensor) -> tuple[dict, torch.Tensor]:
        x = t.detach().float()
        if x.is_cuda and x.numel():
            from ..ops import codec

            q, scale, resid = codec.quant_int8(x)
            return {"q": q.cpu(), "s": scale}, resid
        scale = (float(x.abs().max()) if x.numel() else 0.0) / 127.0
        if scale == 0.0:
            return {"q": torch.zeros(x.shape, dtype=torch.int8), "s": 0.0}, x.clone()
        q = (x / scale).round().clamp(-127, 127).to(torch.int8)
        return {"q": q, "s": scale}, x - q.float() * scale

    @staticmethod
    def decode(p: dict) -> torch.Tensor:
        return p["q"].float() * float(p["s"])


class _Int4:
    """Group-wise int4, two codes per byte."""

    @staticmethod
    def matches(obj) -> bool:
        return isinstance(obj, dict) and "q4" in obj

    @staticmethod
    def encode(t: torch.Tensor, group: int = INT4_GROUP) -> tuple[dict, torch.Tensor]:
        x = t.detach().reshape(-1).float()
        n = x.numel()
        meta = {"g": group, "n": n, "shape": list(t.shape)}
        if x.is_cuda and group == INT4_GROUP and n:
            from ..ops import codec

            packed, scale, resid = codec.quant_int4(x)
            return {"q4": packed, "s": scale, **meta}, resid.reshape(t.shape)
        groups = torch.nn.functional.pad(x, (0, -n % group)).view(-1, group)
        scale = groups.abs().amax(dim=1) / 7.0
        divisor = torch.where(scale > 0, scale, torch.ones_like(scale))
        q = (groups / divisor[:, None]).round().clamp(-7, 7)
        codes = (q + 8).to(torch.uint8).view(-1, 2)
        packed = ((codes[:, 0] << 4) | codes[:, 1]).contiguous()
        recon = (q * scale[:, None]).reshape(-1)[:n]
        return {"q4": packed, "s": scale.float(), **meta}, (x - recon).reshape(t.shape)

    @staticmethod
    def decode(p: dict) -> torch.Tensor:
        packed, scale = p.get("q4"), p.get("s")
        try:
            group, n = int(p.get("g", 0)), int(p.get("n", -1))
        except (TypeError, ValueError):
            raise ValueError("malformed int4 payload") from None
        if not (torch.is_tensor(packed) and torch.is_tensor(scale)) or group <= 0 or n < 0:
            raise ValueError("malformed int4 payload")
        ngroups = -(-n // group)
        if scale.numel() != ngroups or packed.numel() * 2 != ngroups * group:
            raise ValueError("malformed int4 payload: length mismatch")
        if packed.is_cuda and group % 2 == 0:
            from ..ops import codec

            return codec.dequant_int4(packed, scale, n, group)
        b = packed.reshape(-1).to(torch.int16)
        codes = torch.stack((b >> 4, b & 15), dim=1).reshape(ngroups, group)
        return ((codes.float() - 8.0) * scale.reshape(-1, 1).float()).reshape(-1)[:n]

    @staticmethod
    def decode_shaped(p: dict) -> torch.Tensor:
        flat = _Int4.decode(p)
        shape = [int(s) for s in p["shape"]]
        if any(s < 0 for s in shape) or math.prod(shape) != flat.numel():
            raise ValueError("int4 payload: shape does not match element count")
        return flat.reshape(shape)


def _encode_values(kept: torch.Tensor, mode: str):
    """(payload of the kept values, their decoded fp32 values)."""
    if mode == "int8":
        enc, _ = _Int8.encode(kept)
        return enc, enc["q"].float().to(kept.device) * enc["s"]
    if mode == "int4":
        enc, _ = _Int4.encode(kept)
        return enc, _Int4.decode(enc)
    if mode == "bf16":
        enc = kept.to(torch.bfloat16)
        return enc, enc.float()
    return kept.float(), kept.float()


def _decode_values(v) -> torch.Tensor:
    if _Int8.matches(v):
        return _Int8.decode(v)
    if _Int4.matches(v):
        return _Int4.decode(v)
    if torch.is_tensor(v):
        return v.float()
    raise TypeError(f"not a sparse-payload value: {type(v)}")


class _Sparse:
    """Top-k entries with flat int32 indices."""

    @staticmethod
    def matches(obj) -> bool:
        return isinstance(obj, dict) and "sp" in obj and torch.is_tensor(obj.get("i"))

    @staticmethod
    def encode(d: torch.Tensor, density: float, mode: str) -> tuple[dict, torch.Tensor]:
        d = d.detach()
        if d.dim() == 2:  # the top entries of every output row
            cols = d.shape[1]
            k = max(1, math.ceil(density * cols))
            top = d.abs().topk(k, dim=1).indices
            flat_idx = (top + torch.arange(d.shape[0], device=d.device)[:, None] * cols).reshape(-1)
        else:
            k = max(1, math.ceil(density * d.numel()))
            flat_idx = d.reshape(-1).abs().topk(k).indices
        enc, vals = _encode_values(d.reshape(-1)[flat_idx], mode)
        dense = torch.zeros(d.numel(), dtype=torch.float32, device=d.device).index_copy_(0, flat_idx, vals)
        return {"sp": list(d.shape), "i": flat_idx.to(torch.int32), "v": enc}, dense.reshape(d.shape)

    @staticmethod
    def decode(p: dict) -> torch.Tensor:
        shape = [int(s) for s in p["sp"]]
        if any(s < 0 for s in shape):
            raise ValueError("sparse payload: negative shape dim")
        vals = _decode_values(p["v"]).reshape(-1)
        idx = p["i"].long().reshape(-1)
        if idx.numel() != vals.numel():
            raise ValueError("sparse payload: index/value length mismatch")
        n = math.prod(shape)
        if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= n):
            raise ValueError("sparse payload: index out of range")
        dense = torch.zeros(n, dtype=torch.float32, device=vals.device)
        dense[idx.to(vals.device)] = vals
        return dense.reshape(shape)


# the int8 / int4 codecs under the names the rest of the package (and its tests) use
_quantize_int8 = _Int8.encode
_quantize_int4 = _Int4.encode
_dequant_int4 = _Int4.decode


# ------------------------------------------------------------------ down-link
def compress_state(sd: dict, mode: str) -> dict:
    """Weights for the down-link: floating tensors in bf16 unless ``mode`` is "none"."""
    if mode == "none":
        return sd
    return {name: t.to(torch.bfloat16) if t.is_floating_point() else t for name, t in sd.items()}


def compress_shard(shard, mode: str):
    """Token ids travel as int32 in the compressed modes."""
    return shard if shard is None or mode == "none" else shard.to(torch.int32)


def restore_shard(shard):
    return None if shard is None else shard.long()


def encode_state_delta(cur: dict, base: dict, mode: str = "int8") -> dict:
    """Quantised difference of ``cur`` against the keyframe ``base`` for every floating
    tensor with a same-shaped base; other entries are sent as they are."""
    codec = _Int4 if mode == "int4" else _Int8
    out = {}
    for name, t in cur.items():
        ref = base.get(name)
        if t.is_floating_point() and ref is not None and ref.shape == t.shape:
            out[name] = codec.encode(t.float() - ref.float())[0]
        else:
            out[name] = t
    return out


def apply_state_delta(base: dict, tensors: dict) -> dict:
    """Inverse of :func:`encode_state_delta` (validated against the keyframe's shapes)."""
    out = {}
    for name, t in tensors.items():
        if _Int8.matches(t):
            ref = base[name]
            if t["q"].shape != ref.shape:
                raise ValueError(f"int8 delta shape {tuple(t['q'].shape)} != base {tuple(ref.shape)}")
            out[name] = ref.float() + _Int8.decode(t).to(ref.device)
        elif _Int4.matches(t):
            ref = base[name]
            flat = _Int4.decode(t)
            if flat.numel() != ref.numel():
                raise ValueError(f"int4 delta has {flat.numel()} elems != base {ref.numel()}")
            out[name] = ref.float() + flat.reshape(ref.shape).to(ref.device)
        elif torch.is_tensor(t):
            out[name] = t
        else:
            raise TypeError(f"not a state-delta entry: {type(t)}")
    return out


# ------------------------------------------------------------------ up-link
def compress_delta(delta, mode: str, carry=None, density: float = 1.0):
    """Encode one module's pseudo-gradient list (``carry``: the previous round's residuals,
    added first). Returns (payload list, residual list); residual = input - decoded."""
    if mode == "none" and density >= 1.0:
        return list(delta), None
    if carry is not None:
        delta = [d + c for d, c in zip(delta, carry)]
    payloads, residuals = [], []
    for d in delta:
        if density < 1.0:
            p, recon = _Sparse.encode(d, density, mode)
            r = d.detach().float() - recon
        elif mode == "bf16":
            p = d.detach().to(torch.bfloat16)
            r = d.detach().float() - p.float()
        elif mode == "int4":
            p, r = _Int4.encode(d)
        else:
            p, r = _Int8.encode(d)
        payloads.append(p)
        residuals.append(r)
    return payloads, residuals


def maybe_dequantize(items) -> list[torch.Tensor]:
    """Decode a pseudo-gradient list of any payload kind to fp32 tensors."""
    out = []
    for it in items:
        if torch.is_tensor(it):
            out.append(it if it.dtype == torch.float32 else it.float())
        elif _Int8.matches(it):
            out.append(_Int8.decode(it))
        elif _Int4.matches(it):
            out.append(_Int4.decode_shaped(it))
        elif _Sparse.matches(it):
            out.append(_Sparse.decode(it))
        else:
            raise TypeError(f"not a pseudo-gradient tensor: {type(it)}")
    return out


# ------------------------------------------------------------------ digests
def declared_shape(payload):
    """The dense shape a pseudo-gradient payload claims, read without decoding it (None
    when it is not a payload)."""
    try:
        if torch.is_tensor(payload):
            return tuple(payload.shape)
        if isinstance(payload, dict):
            if torch.is_tensor(payload.get("q")):
                return tuple(payload["q"].shape)
            if "q4" in payload:
                return tuple(int(s) for s in payload["shape"])
            if "sp" in payload:
                return tuple(int(s) for s in payload["sp"])
    except (TypeError, ValueError, KeyError):
        return None
    return None


def decode_checked(items, shapes) -> list[torch.Tensor]:
    """Decode a pseudo-gradient list after checking that the shapes it declares are
    exactly ``shapes`` (before anything is allocated: a payload claiming a huge shape is
    refused, not materialised)."""
    if not isinstance(items, list) or len(items) != len(shapes) or any(
            declared_shape(p) != tuple(s) for p, s in zip(items, shapes)):
        raise ValueError("pseudo-gradient payload does not match the module's shapes")
    return maybe_dequantize(items)


def _digest_tensor(h, t: torch.Tensor) -> None:
    enc, _ = _Int8.encode(t.detach().cpu())
    s = enc["s"]
    h.update(struct.pack(">q", round(math.log(s) * 1000.0) if s > 0 else 0))
    h.update(enc["q"].numpy().tobytes())


def pseudograd_digest(shared_delta: dict) -> str:
    """Digest of a pseudo-gradient (key -> tensor list) that redundant executions agree
    on despite float noise below one int8 step."""
    h = hashlib.sha256()
    for key in sorted(shared_delta):
        h.update(key.encode())
        for t in shared_delta[key]:
            _digest_tensor(h, t)
    return h.hexdigest()


def state_digest(state: dict) -> str:
    """Digest of a named state dict (integer tensors hashed exactly)."""
    h = hashlib.sha256()
    for name in sorted(state):
        h.update(name.encode())
        t = state[name]
        if torch.is_floating_point(t):
            _digest_tensor(h, t)
        else:
            h.update(t.cpu().numpy().tobytes())
    return h.hexdigest()
