"""Messages of the control plane: a pickle-free body codec, length framing and the
challenge / response authentication.

The byte layout is a contract shared with the reference (``src/opendipaco/schedule/
wire.py``), so workers and servers of either framework talk to each other::

    frame = [u64 big-endian body length][body]
    body  = [u32 structure length][structure: UTF-8 JSON][u32 tensor count]
            tensor count x ([u8 dtype code][u8 ndim][u64 dim] x ndim [u64 nbytes][raw bytes])

The structure is ``json.dumps`` of the message with every tensor replaced by
``{"$t": <index into the tensor list>}`` (depth-first, in dict order) and every tuple by
``{"$tup": [...]}``; dict keys must be strings. Tensors travel as their raw little-endian
bytes under a fixed code table of ten dtypes; nothing in a received message is executed,
and a frame longer than the receiver's cap is refused before its body is read.

Authentication: the server sends ``{"type": "challenge", "nonce": <32 random bytes,
hex>}``; the client answers ``{"type": "auth", "mac": HMAC-SHA256(key, nonce)}`` (any of
the server's accepted keys, so keys can be rotated) or, with a ``PeerIdentity``,
``{"type": "auth", "pub": ..., "sig": ...}``; the server confirms with
``{"type": "welcome"}``.
"""

from __future__ import annotations

import functools
import hashlib
import hmac
import json
import os
import socket
import struct

import torch

DEFAULT_MAX_MSG_BYTES = 4 * 1024 ** 3  # above one large path's weights; bounds a garbage length prefix
_LEN = struct.Struct(">Q")             # frame length prefix
_U32 = struct.Struct(">I")
_U64 = struct.Struct(">Q")

# dtype code table (the wire contract); anything else is refused on both ends
_CODE_OF = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3, torch.int64: 4,
            torch.int32: 5, torch.int16: 6, torch.int8: 7, torch.uint8: 8, torch.bool: 9}
_DTYPE_OF = {c: d for d, c in _CODE_OF.items()}
_TENSOR, _TUPLE = "$t", "$tup"


# ------------------------------------------------------------------ body codec
def _tagged(obj, tensors: list):
    """The JSON-able structure of ``obj``; its tensors are appended to ``tensors``."""
    if torch.is_tensor(obj):
        tensors.append(obj)
        return {_TENSOR: len(tensors) - 1}
    if isinstance(obj, dict):
        out = {}
        for key, value in obj.items():
            if type(key) is not str:
                raise TypeError(f"wire dict keys must be str, got {type(key)}")
            out[key] = _tagged(value, tensors)
        return out
    if isinstance(obj, tuple):
        return {_TUPLE: [_tagged(x, tensors) for x in obj]}
    if isinstance(obj, list):
        return [_tagged(x, tensors) for x in obj]
    if obj is None or isinstance(obj, (bool, int, float, str)):
        return obj
    raise TypeError(f"cannot serialize {type(obj)} over the wire")


def _tensor_record(t: torch.Tensor) -> list:
    code = _CODE_OF.get(t.dtype)
    if code is None:
        raise TypeError(f"unsupported tensor dtype {t.dtype}")
    t = t.detach().to("cpu").contiguous()
    raw = t.reshape(-1).view(torch.uint8).numpy()
    head = struct.pack(f">BB{t.dim()}QQ", code, t.dim(), *t.shape, raw.nbytes)
    return [head, memoryview(raw)]


def encode(obj) -> bytes:
    """Message -> body bytes."""
    tensors: list = []
    structure = json.dumps(_tagged(obj, tensors)).encode("utf-8")
    pieces = [_U32.pack(len(structure)), structure, _U32.pack(len(tensors))]
    for t in tensors:
        pieces.extend(_tensor_record(t))
    return b"".join(pieces)


def _untag(tensors: list, node: dict):
    if len(node) == 1:
        if _TENSOR in node:
            return tensors[node[_TENSOR]]
        if _TUPLE in node:
            return tuple(node[_TUPLE])
    return node


def decode(data: bytes):
    """Body bytes -> message. Tensors are read first (they follow the structure) so the
    JSON parser can put them in place as it builds each dict."""
    view = memoryview(data)
    (slen,) = _U32.unpack_from(view, 0)
    structure = bytes(view[4:4 + slen])
    pos = 4 + slen
    (count,) = _U32.unpack_from(view, pos)
    pos += 4
    tensors = []
    for _ in range(count):
        code, ndim = view[pos], view[pos + 1]
        dtype = _DTYPE_OF.get(code)
        if dtype is None:
            raise ValueError(f"unknown tensor dtype code {code}")
        shape = struct.unpack_from(f">{ndim}Q", view, pos + 2)
        (nbytes,) = _U64.unpack_from(view, pos + 2 + 8 * ndim)
        pos += 2 + 8 * ndim + 8
        if pos + nbytes > len(view):
            raise ValueError("truncated tensor blob")
        if nbytes:
            flat = torch.frombuffer(bytearray(view[pos:pos + nbytes]), dtype=torch.uint8)  # owns its copy
        else:
            flat = torch.empty(0, dtype=torch.uint8)
        tensors.append(flat.view(dtype).reshape(shape))
        pos += nbytes
    return json.loads(structure, object_hook=functools.partial(_untag, tensors))


# ------------------------------------------------------------------ framing
def send_msg(sock: socket.socket, obj) -> int:
    """Frame and send one message; returns the bytes put on the wire."""
    body = encode(obj)
    sock.sendall(_LEN.pack(len(body)) + body)
    return _LEN.size + len(body)


def _read_exact(sock: socket.socket, n: int) -> bytearray | None:
    buf = bytearray(n)
    view, got = memoryview(buf), 0
    while got < n:
        k = sock.recv_into(view[got:], min(n - got, 1 << 20))
        if k == 0:
            return None  # peer closed
        got += k
    return buf


def recv_msg_sized(sock: socket.socket, max_bytes: int = DEFAULT_MAX_MSG_BYTES):
    """(message, bytes read) of the next frame, or (None, 0) when the peer closed."""
    head = _read_exact(sock, _LEN.size)
    if head is None:
        return None, 0
    (n,) = _LEN.unpack(head)
    if n > max_bytes:
        raise ValueError(f"incoming message of {n} bytes exceeds cap {max_bytes}")
    body = _read_exact(sock, n)
    if body is None:
        return None, 0
    return decode(body), _LEN.size + n


def recv_msg(sock: socket.socket, max_bytes: int = DEFAULT_MAX_MSG_BYTES):
    return recv_msg_sized(sock, max_bytes)[0]


# ------------------------------------------------------------------ shared-secret auth
def key_bytes(key) -> bytes:
    return key.encode() if isinstance(key, str) else bytes(key)


_kb = key_bytes


def coerce_keys(auth_key) -> list[bytes] | None:
    """One key or an iterable of keys -> list of byte strings (None: no auth)."""
    if auth_key is None:
        return None
    if isinstance(auth_key, (str, bytes, bytearray)):
        return [key_bytes(auth_key)]
    return [key_bytes(k) for k in auth_key] or None


def acceptable_keys(auth_key, accept_keys=None) -> list[bytes] | None:
    """The server's current key followed by the extra accepted ones, without repeats."""
    merged = dict.fromkeys((coerce_keys(auth_key) or []) + (coerce_keys(accept_keys) or []))
    return list(merged) or None


def _mac(key: bytes, nonce: bytes) -> str:
    return hmac.new(key, nonce, hashlib.sha256).hexdigest()


def verify_mac(mac: str, nonce: bytes, keys: list[bytes]) -> bool:
    """Constant-time check of ``mac`` against every accepted key (all are compared, so
    the timing does not tell which key matched)."""
    hits = [hmac.compare_digest(mac, _mac(k, nonce)) for k in keys]
    return any(hits)


def server_handshake(sock: socket.socket, key) -> bool:
    """Blocking server side of the challenge / response (True: authenticated)."""
    keys = coerce_keys(key)
    if keys is None:
        return True
    nonce = os.urandom(32)
    try:
        send_msg(sock, {"type": "challenge", "nonce": nonce.hex()})
        answer = recv_msg(sock, max_bytes=4096)
        if not (answer and answer.get("type") == "auth" and verify_mac(answer.get("mac", ""), nonce, keys)):
            return False
        send_msg(sock, {"type": "welcome"})
        return True
    except (OSError, ValueError):
        return False


def client_handshake(sock: socket.socket, key) -> bool:
    """Blocking client side: answers the challenge with an HMAC of ``key`` or, when
    ``key`` is a ``PeerIdentity``, its signature."""
    if key is None:
        return True
    try:
        challenge = recv_msg(sock, max_bytes=4096)
        if not challenge or challenge.get("type") != "challenge":
            return False
        nonce = bytes.fromhex(challenge["nonce"])
        proof = key.auth_response(nonce) if hasattr(key, "auth_response") else {"mac": _mac(key_bytes(key), nonce)}
        send_msg(sock, {"type": "auth", **proof})
        reply = recv_msg(sock, max_bytes=4096)
        return bool(reply and reply.get("type") == "welcome")
    except (OSError, ValueError, KeyError):
        return False
