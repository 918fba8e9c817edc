"""Selector-based TCP server core and transport metrics (reference ``schedule/reactor.py``).

``ReactorServer`` accepts connections on one thread and spreads them over
``io_threads`` selector loops (non-blocking sockets, optional non-blocking TLS
handshake). Each connection must first answer a challenge with an HMAC over one of
the accepted shared secrets or an Ed25519 signature from an admitted identity;
afterwards every complete frame is decoded with the pickle-free codec and handed to
the subclass hook :meth:`ReactorServer._handle`, whose optional reply is queued
back. Frames longer than ``max_msg_bytes`` close the connection; beyond
``max_connections`` new sockets are refused. ``TransportMetrics`` counts tasks,
submissions, bytes by category (``bytes_opt`` must stay 0: optimizer state never
crosses the wire), rejections and staleness, with Prometheus text output.
"""

from __future__ import annotations

import os
import selectors
import socket
import ssl
import threading
import time
from dataclasses import dataclass, field

import torch

from .identity import peer_id_of, verify_auth
from .wire import DEFAULT_MAX_MSG_BYTES, _LEN, acceptable_keys, decode, encode, verify_mac


def _pubkey_hex(p) -> str:
    return getattr(p, "public_key_hex", p).lower()


def _tensor_bytes(obj) -> int:
    if obj is None:
        return 0
    if torch.is_tensor(obj):
        return obj.numel() * obj.element_size()
    if isinstance(obj, dict):
        return sum(_tensor_bytes(v) for v in obj.values())
    if isinstance(obj, (list, tuple)):
        return sum(_tensor_bytes(v) for v in obj)
    return 0


def _fmt(n: float) -> str:
    for unit in ("B", "KB", "MB", "GB"):
        if n < 1024 or unit == "GB":
            return f"{int(n)}B" if unit == "B" else f"{n:.1f}{unit}"
        n /= 1024
    return f"{n:.1f}GB"


@dataclass
class TransportMetrics:
    _GAUGES = frozenset({"max_staleness", "mean_staleness", "throughput_tasks_per_s", "active_workers"})
    _LIVENESS_WINDOW = 60.0
    generations: int = 0
    tasks_sent: int = 0
    submits: int = 0
    heartbeats: int = 0
    nacks: int = 0
    idle: int = 0
    reclaims: int = 0
    dropped: int = 0
    tasks_with_shard: int = 0
    tasks_with_private_down: int = 0
    bytes_down: int = 0
    bytes_up: int = 0
    bytes_control: int = 0
    bytes_shared_weights: int = 0
    bytes_private_down: int = 0
    bytes_shard: int = 0
    bytes_shared_grad: int = 0
    bytes_private_up: int = 0
    bytes_opt: int = 0
    accepted_updates: int = 0
    stale_rejected: int = 0
    invalid_rejected: int = 0
    norm_clipped: int = 0
    poison_flagged: int = 0
    handler_errors: int = 0
    staleness_sum: int = 0
    max_staleness: int = 0
    _wall: float = 0.0
    _worker_seen: dict = field(default_factory=dict)
    _lock: threading.Lock = field(default_factory=threading.Lock)

    def _bump(self, name: str, by: int = 1) -> None:
        with self._lock:
            setattr(self, name, getattr(self, name) + by)

    def record_worker(self, worker_id) -> None:
        with self._lock:
            self._worker_seen[worker_id] = time.monotonic()

    def active_workers(self, window: float | None = None) -> int:
        w = self._LIVENESS_WINDOW if window is None else window
        now = time.monotonic()
        with self._lock:
            return sum(1 for t in self._worker_seen.values() if now - t <= w)

    def record_update(self, staleness: int) -> None:
        with self._lock:
            self.accepted_updates += 1
            self.staleness_sum += staleness
            self.max_staleness = max(self.max_staleness, staleness)

    def record_stale_reject(self) -> None:
        self._bump("stale_rejected")

    def record_invalid_reject(self) -> None:
        self._bump("invalid_rejected")

    def record_norm_clip(self) -> None:
        self._bump("norm_clipped")

    def record_poison_flag(self) -> None:
        self._bump("poison_flagged")

    def record_handler_error(self) -> None:
        self._bump("handler_errors")

    def record_out(self, msg: dict, nbytes: int) -> None:
        with self._lock:
            if msg.get("type") == "task":
                self.tasks_sent += 1
                self.bytes_down += nbytes
                self.bytes_shared_weights += _tensor_bytes(msg.get("shared_weights"))
                self.bytes_opt += _tensor_bytes(msg.get("opt_state"))
                if msg.get("private_weights"):
                    self.tasks_with_private_down += 1
                    self.bytes_private_down += _tensor_bytes(msg["private_weights"])
                if msg.get("shard") is not None:
                    self.tasks_with_shard += 1
                    self.bytes_shard += _tensor_bytes(msg["shard"])
                return
            if msg.get("type") == "idle":
                self.idle += 1
            self.bytes_control += nbytes

    def record_in(self, msg: dict, nbytes: int) -> None:
        with self._lock:
            kind = msg.get("type")
            if kind == "submit":
                self.submits += 1
                self.bytes_up += nbytes
                self.bytes_shared_grad += _tensor_bytes(msg.get("shared_grad"))
                self.bytes_private_up += _tensor_bytes(msg.get("private_weights"))
                self.bytes_opt += _tensor_bytes(msg.get("opt_state"))
                return
            if kind == "heartbeat":
                self.heartbeats += 1
            elif kind == "nack":
                self.nacks += 1
            self.bytes_control += nbytes

    def summary(self) -> dict:
        now = time.monotonic()
        with self._lock:
            d = {k: v for k, v in self.__dict__.items() if not k.startswith("_")}
            d["throughput_tasks_per_s"] = self.tasks_sent / self._wall if self._wall else 0.0
            d["mean_staleness"] = self.staleness_sum / self.accepted_updates if self.accepted_updates else 0.0
            d["active_workers"] = sum(1 for t in self._worker_seen.values() if now - t <= self._LIVENESS_WINDOW)
            return d

    def prometheus(self, namespace: str = "opendipaco_transport") -> str:
        out = []
        for k, v in self.summary().items():
            gauge = k in self._GAUGES
            name = f"{namespace}_{k}" if gauge else f"{namespace}_{k}_total"
            out += [f"# TYPE {name} {'gauge' if gauge else 'counter'}", f"{name} {v}"]
        return "\n".join(out) + "\n"

    def report(self) -> str:
        s = self.summary()
        return "\n".join([
            f"accepted={s['accepted_updates']} stale_rejected={s['stale_rejected']} "
            f"mean_staleness={s['mean_staleness']:.1f} max_staleness={s['max_staleness']} "
            f"tasks={s['tasks_sent']} throughput={s['throughput_tasks_per_s']:.1f}/s",
            f"reclaims={s['reclaims']} nacks={s['nacks']} heartbeats={s['heartbeats']}",
            f"bytes  down={_fmt(s['bytes_down'])}  up={_fmt(s['bytes_up'])}  control={_fmt(s['bytes_control'])}",
            f"  optimizer-on-wire={_fmt(s['bytes_opt'])}",
        ])


@dataclass(eq=False)
class _Conn:
    sock: socket.socket
    inbuf: bytearray = field(default_factory=bytearray)
    outbuf: bytearray = field(default_factory=bytearray)
    authed: bool = False
    peer_id: str | None = None
    nonce: bytes | None = None
    want_write: bool = False
    closed: bool = False
    tls: bool = False
    handshaking: bool = False


class _Loop:
    """One selector thread serving many non-blocking connections."""

    def __init__(self, server: "ReactorServer"):
        self.srv = server
        self.sel = selectors.DefaultSelector()
        self._rd, self._wr = socket.socketpair()
        self._rd.setblocking(False)
        self.sel.register(self._rd, selectors.EVENT_READ, data=None)
        self._pending: list[_Conn] = []
        self._plock = threading.Lock()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def add(self, conn: _Conn) -> None:
        with self._plock:
            self._pending.append(conn)
        self.wake()

    def wake(self) -> None:
        try:
            self._wr.send(b"!")
        except OSError:
            pass

    def _run(self) -> None:
        while not self.srv._io_stop and not self.srv._dead:
            try:
                events = self.sel.select(timeout=0.2)
            except OSError:
                break
            for key, mask in events:
                if key.data is None:
                    try:
                        self._rd.recv(65536)
                    except OSError:
                        pass
                    self._adopt()
                    continue
                conn = key.data
                if conn.handshaking:
                    self._tls_step(conn)
                    continue
                if mask & selectors.EVENT_READ:
                    self._read(conn)
                if not conn.closed and mask & selectors.EVENT_WRITE:
                    self._flush(conn)
        for key in list(self.sel.get_map().values()):
            if key.data is not None:
                self._close(key.data)
        try:
            self.sel.close()
        except OSError:
            pass

    def _adopt(self) -> None:
        with self._plock:
            new, self._pending = self._pending, []
        for conn in new:
            try:
                self.sel.register(conn.sock, selectors.EVENT_READ, data=conn)
            except (KeyError, ValueError, OSError):
                self._close(conn)
                continue
            self._tls_step(conn) if conn.handshaking else self._greet(conn)

    def _greet(self, conn: _Conn) -> None:
        if self.srv.auth_keys is not None or self.srv.admitted_peers is not None:
            conn.nonce = os.urandom(32)
            self._send(conn, {"type": "challenge", "nonce": conn.nonce.hex()})
        else:
            conn.authed = True

    def _tls_step(self, conn: _Conn) -> None:
        try:
            conn.sock.do_handshake()
        except ssl.SSLWantReadError:
            self._want_write(conn, False)
            return
        except ssl.SSLWantWriteError:
            self._want_write(conn, True)
            return
        except (ssl.SSLError, OSError):
            self._close(conn)
            return
        conn.handshaking = False
        self._want_write(conn, False)
        self._greet(conn)

    def _read(self, conn: _Conn) -> None:
        while not conn.closed:
            try:
                data = conn.sock.recv(1 << 20)
            except (BlockingIOError, ssl.SSLWantReadError):
                return
            except ssl.SSLWantWriteError:
                self._want_write(conn, True)
                return
            except OSError:
                self._close(conn)
                return
            if not data:
                self._close(conn)
                return
            conn.inbuf += data
            self._frames(conn)
            if not (conn.tls and conn.sock.pending()):
                return

    def _frames(self, conn: _Conn) -> None:
        while not conn.closed and len(conn.inbuf) >= _LEN.size:
            (n,) = _LEN.unpack_from(conn.inbuf, 0)
            if n > self.srv.max_msg_bytes:
                self._close(conn)
                return
            if len(conn.inbuf) < _LEN.size + n:
                return
            body = bytes(conn.inbuf[_LEN.size:_LEN.size + n])
            del conn.inbuf[:_LEN.size + n]
            try:
                msg = decode(body)
            except Exception:
                self._close(conn)
                return
            try:
                self._dispatch(conn, msg, n + _LEN.size)
            except Exception:
                self.srv.metrics.record_handler_error()
                self._close(conn)
                return

    def _dispatch(self, conn: _Conn, msg: dict, nin: int) -> None:
        srv = self.srv
        if not conn.authed:
            ok = False
            if conn.nonce is not None and msg.get("type") == "auth":
                if srv.auth_keys is not None and "mac" in msg:
                    ok = verify_mac(msg.get("mac", ""), conn.nonce, srv.auth_keys)
                if not ok and srv.admitted_peers is not None and "pub" in msg:
                    pub = msg.get("pub", "")
                    if srv.peer_admitted(pub) and verify_auth(pub, msg.get("sig", ""), conn.nonce):
                        ok, conn.peer_id = True, peer_id_of(pub)
            if ok:
                conn.authed = True
                self._send(conn, {"type": "welcome"})
            else:
                self._close(conn)
            return
        if msg.get("worker_id") is not None:
            srv.metrics.record_worker(msg["worker_id"])
        srv.metrics.record_in(msg, nin)
        reply = srv._handle(msg, nin, conn.peer_id)
        if reply is not None:
            srv.metrics.record_out(reply, self._send(conn, reply))

    def _send(self, conn: _Conn, msg: dict) -> int:
        data = encode(msg)
        frame = _LEN.pack(len(data)) + data
        conn.outbuf += frame
        self._flush(conn)
        return len(frame)

    def _flush(self, conn: _Conn) -> None:
        if conn.closed:
            return
        if conn.outbuf:
            try:
                sent = conn.sock.send(conn.outbuf)
                del conn.outbuf[:sent]
            except (BlockingIOError, ssl.SSLWantWriteError, ssl.SSLWantReadError):
                pass
            except OSError:
                self._close(conn)
                return
        self._want_write(conn, bool(conn.outbuf))

    def _want_write(self, conn: _Conn, on: bool) -> None:
        if conn.closed or conn.want_write == on:
            return
        try:
            self.sel.modify(conn.sock, selectors.EVENT_READ | (selectors.EVENT_WRITE if on else 0), data=conn)
            conn.want_write = on
        except (KeyError, OSError):
            self._close(conn)

    def _close(self, conn: _Conn) -> None:
        if conn.closed:
            return
        conn.closed = True
        for fn in (lambda: self.sel.unregister(conn.sock), conn.sock.close):
            try:
                fn()
            except (KeyError, OSError, ValueError):
                pass
        self.srv._conn_closed(conn)


class ReactorServer:
    """Base TCP server; subclasses implement :meth:`_handle`."""

    def __init__(self, *, host: str = "0.0.0.0", port: int = 0, auth_key=None, accept_keys=None,
                 admitted_peers=None, max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES, io_threads: int = 4,
                 max_connections: int = 1024, tls: "ssl.SSLContext | None" = None):
        self.auth_key = auth_key
        self.auth_keys = acceptable_keys(auth_key, accept_keys)
        self._peer_lock = threading.Lock()
        self.admitted_peers = {_pubkey_hex(p) for p in admitted_peers} if admitted_peers is not None else None
        self.max_msg_bytes = max_msg_bytes
        self.tls = tls
        self.io_threads = max(1, io_threads)
        self.max_connections = max_connections
        self.metrics = TransportMetrics()
        self._sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self._sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        deadline = time.monotonic() + 3.0
        while True:
            try:
                self._sock.bind((host, port))
                break
            except OSError:
                if time.monotonic() >= deadline:
                    raise
                time.sleep(0.1)
        self._sock.listen(128)
        self.port = self._sock.getsockname()[1]
        self._stop = self._io_stop = self._dead = False
        self._loops: list[_Loop] = []
        self._accept_thread = None
        self._conn_lock = threading.Lock()
        self._registry: set = set()
        self._open = 0
        self._rr = 0
        self._exporter = self._logger = None

    def _handle(self, msg: dict, nbytes: int, peer_id: str | None = None):
        raise NotImplementedError

    # identity admission
    def peer_admitted(self, pub: str) -> bool:
        with self._peer_lock:
            return self.admitted_peers is not None and pub.lower() in self.admitted_peers

    def peer_id_admitted(self, peer_id: str) -> bool:
        with self._peer_lock:
            return self.admitted_peers is None or peer_id in {peer_id_of(p) for p in self.admitted_peers}

    def admit_peer(self, pub) -> None:
        with self._peer_lock:
            if self.admitted_peers is None:
                self.admitted_peers = set()
            self.admitted_peers.add(_pubkey_hex(pub))

    def revoke_peer(self, pub) -> None:
        with self._peer_lock:
            if self.admitted_peers is not None:
                self.admitted_peers.discard(_pubkey_hex(pub))

    # observability
    def start_metrics_server(self, *, host: str = "0.0.0.0", port: int = 0,
                             namespace: str = "opendipaco_transport"):
        from .observability import MetricsExporter

        self._exporter = MetricsExporter(self.metrics, host=host, port=port, namespace=namespace).start()
        return self._exporter

    def start_metrics_logging(self, *, interval: float = 10.0, sink=None):
        from .observability import MetricsLogger

        self._logger = MetricsLogger(self.metrics, interval=interval, sink=sink).start()
        return self._logger

    # lifecycle
    def start(self) -> None:
        self._loops = [_Loop(self) for _ in range(self.io_threads)]
        for lp in self._loops:
            lp.thread.start()
        self._accept_thread = threading.Thread(target=self._accept, daemon=True)
        self._accept_thread.start()

    def _accept(self) -> None:
        while not self._stop and not self._dead:
            try:
                sock, _ = self._sock.accept()
            except OSError:
                return
            with self._conn_lock:
                if self._open >= self.max_connections:
                    sock.close()
                    continue
                self._open += 1
            sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            sock.setblocking(False)
            if self.tls is not None:
                try:
                    sock = self.tls.wrap_socket(sock, server_side=True, do_handshake_on_connect=False)
                except (ssl.SSLError, OSError):
                    sock.close()
                    with self._conn_lock:
                        self._open -= 1
                    continue
                conn = _Conn(sock=sock, tls=True, handshaking=True)
            else:
                conn = _Conn(sock=sock)
            with self._conn_lock:
                self._registry.add(conn)
            self._loops[self._rr % len(self._loops)].add(conn)
            self._rr += 1

    def _conn_closed(self, conn: _Conn) -> None:
        with self._conn_lock:
            if conn in self._registry:
                self._registry.discard(conn)
                self._open -= 1

    def shutdown(self) -> None:
        self._stop = True
        for obs in (self._exporter, self._logger):
            if obs is not None:
                obs.stop()
        try:
            self._sock.close()
        except OSError:
            pass
        time.sleep(0.2)
        self._io_stop = True
        for lp in self._loops:
            lp.wake()
        time.sleep(0.1)

    def simulate_crash(self) -> None:
        """Drop every connection abruptly (tests of restart / reconnect)."""
        self._dead = self._io_stop = True
        with self._conn_lock:
            conns = list(self._registry)
        for conn in conns:
            for fn in (lambda: conn.sock.shutdown(socket.SHUT_RDWR), conn.sock.close):
                try:
                    fn()
                except OSError:
                    pass
        try:
            self._sock.close()
        except OSError:
            pass
        for lp in self._loops:
            lp.wake()


_ReactorServer = ReactorServer
