"""Pickle-free message codec, framing and authentication (reference ``schedule/wire.py``).

Body layout (the wire contract, kept byte-compatible so peers of either framework
interoperate)::

    [u32 json_len][json][u32 n_tensors] then n times:
        [u8 dtype_code][u8 ndim][u64 shape x ndim][u64 nbytes][raw little-endian bytes]

JSON holds dicts with string keys, lists and scalars; tensors become ``{"$t": i}``
and tuples ``{"$tup": [...]}``. Tensors are rebuilt from raw bytes against a
10-dtype allow-list -- nothing is executed on receipt. Frames carry an 8-byte
big-endian length; ``recv_msg_sized`` refuses lengths above ``max_bytes``.
Auth: HMAC-SHA256 challenge/response over shared secrets (several accepted keys
for rotation) or an Ed25519 ``PeerIdentity`` signature.
"""

from __future__ import annotations

import hashlib
import hmac
import json
import os
import socket
import struct

import torch

DEFAULT_MAX_MSG_BYTES = 4 * 1024 ** 3
_LEN = struct.Struct(">Q")
_U32 = struct.Struct(">I")
_U64 = struct.Struct(">Q")
_THDR = struct.Struct(">BB")
_DTYPES = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3, torch.int64: 4,
           torch.int32: 5, torch.int16: 6, torch.int8: 7, torch.uint8: 8, torch.bool: 9}
_CODES = {v: k for k, v in _DTYPES.items()}


def _flatten(obj, blobs: list):
    if torch.is_tensor(obj):
        blobs.append(obj.detach().cpu().contiguous())
        return {"$t": len(blobs) - 1}
    if isinstance(obj, tuple):
        return {"$tup": [_flatten(x, blobs) for x in obj]}
    if isinstance(obj, list):
        return [_flatten(x, blobs) for x in obj]
    if isinstance(obj, dict):
        out = {}
        for k, v in obj.items():
            if not isinstance(k, str):
                raise TypeError(f"wire dict keys must be str, got {type(k)}")
            out[k] = _flatten(v, blobs)
        return out
    if obj is None or isinstance(obj, (str, int, float, bool)):
        return obj
    raise TypeError(f"cannot serialize {type(obj)} over the wire")


def _unflatten(s, blobs: list):
    if isinstance(s, dict):
        if len(s) == 1 and "$t" in s:
            return blobs[s["$t"]]
        if len(s) == 1 and "$tup" in s:
            return tuple(_unflatten(x, blobs) for x in s["$tup"])
        return {k: _unflatten(v, blobs) for k, v in s.items()}
    if isinstance(s, list):
        return [_unflatten(x, blobs) for x in s]
    return s


def encode(obj) -> bytes:
    blobs: list = []
    js = json.dumps(_flatten(obj, blobs)).encode()
    parts = [_U32.pack(len(js)), js, _U32.pack(len(blobs))]
    for t in blobs:
        if t.dtype not in _DTYPES:
            raise TypeError(f"unsupported tensor dtype {t.dtype}")
        raw = t.reshape(-1).view(torch.uint8).numpy().tobytes()
        parts.append(_THDR.pack(_DTYPES[t.dtype], t.dim()))
        parts += [_U64.pack(d) for d in t.shape]
        parts += [_U64.pack(len(raw)), raw]
    return b"".join(parts)


def decode(data: bytes):
    mv = memoryview(data)
    (n,) = _U32.unpack_from(mv, 0)
    off = 4
    structure = json.loads(bytes(mv[off:off + n]))
    off += n
    (nt,) = _U32.unpack_from(mv, off)
    off += 4
    blobs = []
    for _ in range(nt):
        code, ndim = _THDR.unpack_from(mv, off)
        off += _THDR.size
        if code not in _CODES:
            raise ValueError(f"unknown tensor dtype code {code}")
        shape = list(struct.unpack_from(f">{ndim}Q", mv, off))
        off += 8 * ndim
        (nb,) = _U64.unpack_from(mv, off)
        off += 8
        raw = mv[off:off + nb]
        off += nb
        if len(raw) != nb:
            raise ValueError("truncated tensor blob")
        blobs.append(torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(_CODES[code]).reshape(shape).clone())
    return _unflatten(structure, blobs)


def send_msg(sock: socket.socket, obj) -> int:
    data = encode(obj)
    sock.sendall(_LEN.pack(len(data)) + data)
    return len(data) + _LEN.size


def _recv_n(sock: socket.socket, n: int) -> bytes | None:
    buf = bytearray()
    while len(buf) < n:
        b = sock.recv(min(n - len(buf), 1 << 20))
        if not b:
            return None
        buf += b
    return bytes(buf)


def recv_msg_sized(sock: socket.socket, max_bytes: int = DEFAULT_MAX_MSG_BYTES):
    hdr = _recv_n(sock, _LEN.size)
    if hdr is None:
        return None, 0
    (n,) = _LEN.unpack(hdr)
    if n > max_bytes:
        raise ValueError(f"incoming message of {n} bytes exceeds cap {max_bytes}")
    body = _recv_n(sock, n)
    return (None, 0) if body is None else (decode(body), n + _LEN.size)


def recv_msg(sock: socket.socket, max_bytes: int = DEFAULT_MAX_MSG_BYTES):
    return recv_msg_sized(sock, max_bytes)[0]


def _kb(key) -> bytes:
    return key.encode() if isinstance(key, str) else bytes(key)


def coerce_keys(auth_key) -> list[bytes] | None:
    if auth_key is None:
        return None
    if isinstance(auth_key, (str, bytes, bytearray)):
        return [_kb(auth_key)]
    keys = [_kb(k) for k in auth_key]
    return keys or None


def acceptable_keys(auth_key, accept_keys=None) -> list[bytes] | None:
    out: list[bytes] = []
    for src in (auth_key, accept_keys):
        for k in coerce_keys(src) or []:
            if k not in out:
                out.append(k)
    return out or None


def verify_mac(mac: str, nonce: bytes, keys: list[bytes]) -> bool:
    ok = False
    for k in keys:  # no early exit: timing does not reveal which key matched
        ok |= hmac.compare_digest(mac, hmac.new(k, nonce, hashlib.sha256).hexdigest())
    return ok


def server_handshake(sock: socket.socket, key) -> bool:
    keys = coerce_keys(key)
    if keys is None:
        return True
    nonce = os.urandom(32)
    try:
        send_msg(sock, {"type": "challenge", "nonce": nonce.hex()})
        reply = recv_msg(sock, max_bytes=4096)
    except (OSError, ValueError):
        return False
    if not reply or reply.get("type") != "auth" or not verify_mac(reply.get("mac", ""), nonce, keys):
        return False
    try:
        send_msg(sock, {"type": "welcome"})
    except OSError:
        return False
    return True


def client_handshake(sock: socket.socket, key) -> bool:
    if key is None:
        return True
    try:
        ch = recv_msg(sock, max_bytes=4096)
        if not ch or ch.get("type") != "challenge":
            return False
        nonce = bytes.fromhex(ch["nonce"])
        if hasattr(key, "auth_response"):
            send_msg(sock, {"type": "auth", **key.auth_response(nonce)})
        else:
            send_msg(sock, {"type": "auth", "mac": hmac.new(_kb(key), nonce, hashlib.sha256).hexdigest()})
        ok = recv_msg(sock, max_bytes=4096)
    except (OSError, ValueError):
        return False
    return bool(ok and ok.get("type") == "welcome")
