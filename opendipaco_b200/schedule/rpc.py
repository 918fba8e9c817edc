"""Blocking client-side RPC helpers shared by workers, schedulers, trackers and owners
(the dial / request-reply half of reference ``src/opendipaco/schedule/sharded.py`` and
``src/opendipaco/schedule/tracker.py``)."""

from __future__ import annotations

import socket
import ssl
import threading
import time

from .wire import DEFAULT_MAX_MSG_BYTES, client_handshake, recv_msg, send_msg


def connect(addr, auth_key=None, max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES, timeout: float = 10.0, *, tls=None,
            server_hostname: str | None = None) -> socket.socket:
    """Dial ``(host, port)`` (retrying until ``timeout``), optionally wrap in TLS, authenticate."""
    host, port = addr[0], int(addr[1])
    deadline, last = time.monotonic() + timeout, None
    while time.monotonic() < deadline:
        s = None
        try:
            s = socket.create_connection((host, port), timeout=timeout)
            s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            if tls is not None:
                s = tls.wrap_socket(s, server_hostname=server_hostname or host)
            if not client_handshake(s, auth_key):
                s.close()
                raise PermissionError(f"{host}:{port} rejected authentication")
            return s
        except (ssl.SSLError, PermissionError):
            raise
        except OSError as exc:
            last = exc
            if s is not None:
                s.close()
            time.sleep(0.05)
    raise ConnectionError(f"could not connect to {host}:{port}: {last}")


def rpc(sock: socket.socket, msg: dict, max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES):
    send_msg(sock, msg)
    reply = recv_msg(sock, max_msg_bytes)
    if reply is None:
        raise ConnectionError("peer closed the connection")
    return reply


def rpc_locked(sock, lock: threading.Lock, msg: dict, max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES):
    with lock:
        return rpc(sock, msg, max_msg_bytes)


def one_shot(addr, msg: dict, *, auth_key=None, tls=None, timeout: float = 10.0,
             max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES):
    """Connect, send one request, return the reply, close."""
    s = connect(addr, auth_key, max_msg_bytes, timeout, tls=tls, server_hostname=addr[0])
    try:
        return rpc(s, msg, max_msg_bytes)
    finally:
        s.close()


def record_issued_at(record) -> float | None:
    ts = record.get("issued_at") if isinstance(record, dict) else None
    return float(ts) if isinstance(ts, (int, float)) and not isinstance(ts, bool) else None
