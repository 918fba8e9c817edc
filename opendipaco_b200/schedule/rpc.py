"""Blocking client-side RPC helpers shared by workers, schedulers, trackers and owners
(the dial / request-reply half of reference ``src/opendipaco/schedule/sharded.py`` and
``src/opendipaco/schedule/tracker.py``)."""

from __future__ import annotations

import socket
import ssl
import threading
import time

from .p2p import CIRCUIT_SEP
from .wire import DEFAULT_MAX_MSG_BYTES, client_handshake, recv_msg, send_msg


def connect(addr, auth_key=None, max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES, timeout: float = 10.0, *, tls=None,
            server_hostname: str | None = None) -> socket.socket:
    """Dial ``(host, port)`` (retrying until ``timeout``), optionally wrap in TLS, authenticate.

    ``addr`` may also be a relay circuit address (a NAT peer reached through a relay) or
    a list of addresses tried in order (a peer's several relays)."""
    if isinstance(addr, str):
        return _connect_circuit(addr, auth_key, timeout, tls, server_hostname)
    if _address_list(addr):
        last = None
        for a in addr:
            try:
                return connect(a, auth_key, max_msg_bytes, timeout, tls=tls, server_hostname=server_hostname)
            except (OSError, ConnectionError) as exc:
                if isinstance(exc, PermissionError):
                    raise
                last = exc
        raise ConnectionError(f"no address of {addr!r} answered: {last}")
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


def _address_list(addr) -> bool:
    """A list of addresses (circuit strings or ``(host, port)`` pairs), not one pair."""
    return (isinstance(addr, (list, tuple)) and len(addr) > 0
            and all((isinstance(a, str) and CIRCUIT_SEP in a) or isinstance(a, (list, tuple)) for a in addr))


def _hostname(addr):
    """The TLS server name of a ``(host, port)`` address (None for circuits and lists)."""
    if isinstance(addr, (list, tuple)) and not _address_list(addr) and isinstance(addr[0], str):
        return addr[0]
    return None


def _connect_circuit(addr: str, auth_key, timeout: float, tls, server_hostname):
    from .relay import dial_circuit

    s = dial_circuit(addr, timeout)
    try:
        if tls is not None:
            s = tls.wrap_socket(s, server_hostname=server_hostname or "localhost")
        s.settimeout(timeout)
        if not client_handshake(s, auth_key):
            raise PermissionError(f"{addr} rejected authentication")
        s.settimeout(None)
        return s
    except BaseException:
        s.close()
        raise


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
    s = connect(addr, auth_key, max_msg_bytes, timeout, tls=tls, server_hostname=_hostname(addr))
    try:
        return rpc(s, msg, max_msg_bytes)
    finally:
        s.close()


def record_issued_at(record) -> float | None:
    ts = record.get("issued_at") if isinstance(record, dict) else None
    return float(ts) if isinstance(ts, (int, float)) and not isinstance(ts, bool) else None
