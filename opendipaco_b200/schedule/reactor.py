"""TCP server core of the control plane and its transport metrics.

``ReactorServer`` is the base of the coordinator, the sharded scheduler, the parameter
servers and the tracker. It runs one asyncio event loop on a background thread: the loop
owns every socket (accepting, the optional TLS handshake, framed reads and writes with
back-pressure), and a pool of ``io_threads`` worker threads decodes each frame, runs the
subclass hook :meth:`ReactorServer._handle` and encodes its reply, so a large tensor
payload or a slow handler never stalls the other connections. Messages of one connection
are handled strictly in order; different connections are handled concurrently.

A connection that must authenticate (shared secrets and/or admitted Ed25519 identities)
gets a challenge first and is closed unless its first message answers it (wire.py has
the exchange). Frames longer than ``max_msg_bytes``, bodies that do not decode and
handler exceptions close the connection; beyond ``max_connections`` new sockets are
closed at once.

Behaviour follows the reference's selector-based reactor (``src/opendipaco/schedule/
reactor.py``): same handshake, limits and metrics names (Prometheus scrapes and the
``opendipaco`` report lines stay comparable); the event-loop design is this module's own.
"""

from __future__ import annotations

import asyncio
import os
import socket
import ssl
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import torch

from .identity import peer_id_of, verify_auth
from .wire import DEFAULT_MAX_MSG_BYTES, _LEN, acceptable_keys, decode, encode, verify_mac

# ---------------------------------------------------------------------- metrics
# Counters in exposition order. ``bytes_opt`` counts optimizer state seen on the wire in
# either direction: it must stay 0 (inner-optimizer state never leaves a worker).
_COUNTERS = (
    "generations", "tasks_sent", "submits", "heartbeats", "nacks", "idle", "reclaims", "dropped",
    "tasks_with_shard", "tasks_with_private_down",
    "bytes_down", "bytes_up", "bytes_control", "bytes_shared_weights", "bytes_private_down", "bytes_shard",
    "bytes_shared_grad", "bytes_private_up", "bytes_opt",
    "accepted_updates", "stale_rejected", "invalid_rejected", "norm_clipped", "poison_flagged", "handler_errors",
    "staleness_sum", "max_staleness",
)
_GAUGES = ("max_staleness", "mean_staleness", "throughput_tasks_per_s", "active_workers")
# per message type: (count counter, total-bytes counter, {payload field: bytes counter},
# {payload field: (counter of messages carrying it, whether a value counts as carried)})
_TRAFFIC_OUT = {"task": ("tasks_sent", "bytes_down",
                         {"shared_weights": "bytes_shared_weights", "opt_state": "bytes_opt",
                          "private_weights": "bytes_private_down", "shard": "bytes_shard"},
                         {"private_weights": ("tasks_with_private_down", bool),
                          "shard": ("tasks_with_shard", lambda x: x is not None)}),
                "idle": ("idle", "bytes_control", {}, {})}
_TRAFFIC_IN = {"submit": ("submits", "bytes_up",
                          {"shared_grad": "bytes_shared_grad", "private_weights": "bytes_private_up",
                           "opt_state": "bytes_opt"}, {}),
               "heartbeat": ("heartbeats", "bytes_control", {}, {}),
               "nack": ("nacks", "bytes_control", {}, {})}


def payload_bytes(obj) -> int:
    """Bytes of every tensor inside a (nested) message field."""
    if torch.is_tensor(obj):
        return obj.numel() * obj.element_size()
    if isinstance(obj, dict):
        obj = obj.values()
    elif not isinstance(obj, (list, tuple)):
        return 0
    return sum(payload_bytes(x) for x in obj)


def human_bytes(n: float) -> str:
    if n < 1024:
        return f"{int(n)}B"
    for unit in ("KB", "MB", "GB"):
        n /= 1024
        if n < 1024 or unit == "GB":
            return f"{n:.1f}{unit}"
    return f"{n:.1f}GB"


class TransportMetrics:
    """Thread-safe counters of one server's traffic and outcomes. Every counter is also
    an attribute (``metrics.reclaims += 1`` works); derived gauges come from
    :meth:`summary`."""

    LIVENESS_WINDOW = 60.0  # a worker counts as active for this long after its last message

    def __init__(self):
        object.__setattr__(self, "_values", dict.fromkeys(_COUNTERS, 0))
        object.__setattr__(self, "_lock", threading.Lock())
        object.__setattr__(self, "_last_seen", {})
        object.__setattr__(self, "_wall", 0.0)  # seconds the server spent serving (throughput)

    def __getattr__(self, name):
        values = self.__dict__["_values"]
        if name in values:
            return values[name]
        raise AttributeError(name)

    def __setattr__(self, name, value):
        if name in self._values:
            with self._lock:
                self._values[name] = value
        else:
            object.__setattr__(self, name, value)

    def _add(self, name: str, by: int = 1) -> None:
        with self._lock:
            self._values[name] += by

    # -- events
    def record_worker(self, worker_id) -> None:
        with self._lock:
            self._last_seen[worker_id] = time.monotonic()

    def active_workers(self, window: float | None = None) -> int:
        horizon = time.monotonic() - (self.LIVENESS_WINDOW if window is None else window)
        with self._lock:
            return sum(t >= horizon for t in self._last_seen.values())

    def record_update(self, staleness: int) -> None:
        with self._lock:
            v = self._values
            v["accepted_updates"] += 1
            v["staleness_sum"] += staleness
            v["max_staleness"] = max(v["max_staleness"], staleness)

    def record_stale_reject(self) -> None:
        self._add("stale_rejected")

    def record_invalid_reject(self) -> None:
        self._add("invalid_rejected")

    def record_norm_clip(self) -> None:
        self._add("norm_clipped")

    def record_poison_flag(self) -> None:
        self._add("poison_flagged")

    def record_handler_error(self) -> None:
        self._add("handler_errors")

    def _traffic(self, table: dict, msg: dict, nbytes: int) -> None:
        count, total, fields, carried = table.get(msg.get("type"), (None, "bytes_control", {}, {}))
        sizes = {f: payload_bytes(msg.get(f)) for f in fields}
        with self._lock:
            v = self._values
            if count:
                v[count] += 1
            v[total] += nbytes
            for f, counter in fields.items():
                v[counter] += sizes[f]
            for f, (counter, carries) in carried.items():
                if carries(msg.get(f)):
                    v[counter] += 1

    def record_out(self, msg: dict, nbytes: int) -> None:
        self._traffic(_TRAFFIC_OUT, msg, nbytes)

    def record_in(self, msg: dict, nbytes: int) -> None:
        self._traffic(_TRAFFIC_IN, msg, nbytes)

    # -- views
    def summary(self) -> dict:
        now = time.monotonic()
        with self._lock:
            out = dict(self._values)
            live = sum(now - t <= self.LIVENESS_WINDOW for t in self._last_seen.values())
        out["throughput_tasks_per_s"] = out["tasks_sent"] / self._wall if self._wall else 0.0
        out["mean_staleness"] = out["staleness_sum"] / out["accepted_updates"] if out["accepted_updates"] else 0.0
        out["active_workers"] = live
        return out

    def prometheus(self, namespace: str = "opendipaco_transport") -> str:
        """Prometheus text exposition: counters as ``<ns>_<name>_total``, gauges as
        ``<ns>_<name>``."""
        lines = []
        for name, value in self.summary().items():
            kind = "gauge" if name in _GAUGES else "counter"
            metric = f"{namespace}_{name}" if kind == "gauge" else f"{namespace}_{name}_total"
            lines.append(f"# TYPE {metric} {kind}\n{metric} {value}")
        return "\n".join(lines) + "\n"

    def report(self) -> str:
        s = self.summary()
        return (f"accepted={s['accepted_updates']} stale_rejected={s['stale_rejected']} "
                f"mean_staleness={s['mean_staleness']:.1f} max_staleness={s['max_staleness']} "
                f"tasks={s['tasks_sent']} throughput={s['throughput_tasks_per_s']:.1f}/s\n"
                f"reclaims={s['reclaims']} nacks={s['nacks']} heartbeats={s['heartbeats']}\n"
                f"bytes  down={human_bytes(s['bytes_down'])}  up={human_bytes(s['bytes_up'])}  "
                f"control={human_bytes(s['bytes_control'])}\n"
                f"  optimizer-on-wire={human_bytes(s['bytes_opt'])}")


# ---------------------------------------------------------------------- server
def _listen(host: str, port: int) -> socket.socket:
    """A listening socket on (host, port); a port still held by a closing predecessor
    is retried for up to 3 s (restart-in-place tests rebind the same port)."""
    sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
    sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
    give_up = time.monotonic() + 3.0
    while True:
        try:
            sock.bind((host, port))
            break
        except OSError:
            if time.monotonic() > give_up:
                sock.close()
                raise
            time.sleep(0.1)
    sock.listen(128)
    sock.setblocking(False)
    return sock


class _Closed(Exception):
    """The connection is to be dropped (protocol violation, peer gone, shutdown)."""


class ReactorServer:
    """Base TCP server; subclasses implement :meth:`_handle`."""

    def __init__(self, *, host: str = "0.0.0.0", port: int = 0, auth_key=None, accept_keys=None,
                 admitted_peers=None, max_msg_bytes: int = DEFAULT_MAX_MSG_BYTES, io_threads: int = 4,
                 max_connections: int = 1024, tls: "ssl.SSLContext | None" = None):
        self.auth_key = auth_key
        self.auth_keys = acceptable_keys(auth_key, accept_keys)
        self._admit_lock = threading.Lock()
        self.admitted_peers = None if admitted_peers is None else {self._hex(p) for p in admitted_peers}
        # peer ids admitted without their key at hand (the owners of a signed epoch list
        # peer ids, which hash from their public keys)
        self._admitted_ids: set = set()
        self.max_msg_bytes = max_msg_bytes
        self.tls = tls
        self.io_threads = max(1, io_threads)
        self.max_connections = max_connections
        self.metrics = TransportMetrics()
        self._listener = _listen(host, port)
        self.port = self._listener.getsockname()[1]
        self._stop = False  # graceful shutdown requested (handlers may answer "stop")
        self._dead = False  # crashed: every connection dropped
        self._loop: asyncio.AbstractEventLoop | None = None
        self._thread: threading.Thread | None = None
        self._workers: ThreadPoolExecutor | None = None
        self._server = None
        self._writers: set = set()
        self._observers: list = []

    @staticmethod
    def _hex(pub) -> str:
        return getattr(pub, "public_key_hex", pub).lower()

    def _handle(self, msg: dict, nbytes: int, peer_id: str | None = None):
        raise NotImplementedError

    # -------------------------------------------------------------- admission
    def _identity_auth_on(self) -> bool:
        return self.admitted_peers is not None or bool(self._admitted_ids)

    def peer_admitted(self, pub: str) -> bool:
        with self._admit_lock:
            if self.admitted_peers is not None and pub.lower() in self.admitted_peers:
                return True
            try:
                return bool(self._admitted_ids) and peer_id_of(pub) in self._admitted_ids
            except ValueError:  # not a hex key
                return False

    def peer_id_admitted(self, peer_id: str) -> bool:
        with self._admit_lock:
            if peer_id in self._admitted_ids:
                return True
            if self.admitted_peers is None:
                return not self._admitted_ids
            return any(peer_id_of(p) == peer_id for p in self.admitted_peers)

    def admit_peer_id(self, peer_id: str) -> None:
        """Admit the identity whose public key hashes to ``peer_id``."""
        with self._admit_lock:
            self._admitted_ids.add(str(peer_id))

    def admit_peer(self, pub) -> None:
        with self._admit_lock:
            if self.admitted_peers is None:
                self.admitted_peers = set()
            self.admitted_peers.add(self._hex(pub))

    def revoke_peer(self, pub) -> None:
        with self._admit_lock:
            if self.admitted_peers is not None:
                self.admitted_peers.discard(self._hex(pub))

    # -------------------------------------------------------------- observability
    def start_metrics_server(self, *, host: str = "0.0.0.0", port: int = 0, namespace: str = "opendipaco_transport"):
        from .observability import MetricsExporter

        exporter = MetricsExporter(self.metrics, host=host, port=port, namespace=namespace).start()
        self._observers.append(exporter)
        return exporter

    def start_metrics_logging(self, *, interval: float = 10.0, sink=None):
        from .observability import MetricsLogger

        logger = MetricsLogger(self.metrics, interval=interval, sink=sink).start()
        self._observers.append(logger)
        return logger

    # -------------------------------------------------------------- lifecycle
    def start(self) -> None:
        self._workers = ThreadPoolExecutor(max_workers=self.io_threads, thread_name_prefix="odp-io")
        self._loop = asyncio.new_event_loop()
        up = threading.Event()

        def run():
            asyncio.set_event_loop(self._loop)
            self._server = self._loop.run_until_complete(
                asyncio.start_server(self._session, sock=self._listener, limit=1 << 22,
                                     **({"ssl": self.tls, "ssl_handshake_timeout": 30.0} if self.tls else {})))
            up.set()
            try:
                self._loop.run_forever()
            finally:
                # sessions still waiting on a handler or a read end here, not at exit
                pending = [t for t in asyncio.all_tasks(self._loop) if not t.done()]
                for t in pending:
                    t.cancel()
                if pending:
                    self._loop.run_until_complete(asyncio.gather(*pending, return_exceptions=True))
                self._loop.run_until_complete(self._loop.shutdown_asyncgens())
                self._loop.close()

        self._thread = threading.Thread(target=run, name=f"odp-reactor-{self.port}", daemon=True)
        self._thread.start()
        if not up.wait(10.0):
            raise RuntimeError("reactor event loop did not start")

    def _on_loop(self, fn) -> None:
        loop = self._loop
        if loop is not None and loop.is_running():
            try:
                loop.call_soon_threadsafe(fn)
            except RuntimeError:  # the loop closed meanwhile
                pass

    def _teardown(self, abort: bool) -> None:
        """On the loop: stop accepting, drop every connection (RST when ``abort``), stop."""
        if self._server is not None:
            self._server.close()
        for w in list(self._writers):
            if abort:
                w.transport.abort()
            else:
                w.close()
        self._loop.call_later(0.05, self._loop.stop)

    def _finish(self) -> None:
        if self._thread is not None:
            self._thread.join(timeout=5.0)
        if self._workers is not None:
            self._workers.shutdown(wait=False, cancel_futures=True)
        try:
            self._listener.close()
        except OSError:
            pass

    def shutdown(self) -> None:
        """Graceful stop: no new connections; connections still being served get a short
        grace period (handlers answer "stop" from now on), then all are closed."""
        self._stop = True
        for obs in self._observers:
            obs.stop()
        self._on_loop(lambda: self._server.close() if self._server is not None else None)
        time.sleep(0.25)
        self._on_loop(lambda: self._teardown(abort=False))
        self._finish()

    def simulate_crash(self) -> None:
        """Drop every connection abruptly and stop serving, as a killed process would (for
        tests of failover, reconnect and restart-in-place)."""
        self._dead = True
        self._stop = True
        for obs in self._observers:
            obs.stop()
        self._on_loop(lambda: self._teardown(abort=True))
        self._finish()

    def adopt_socket(self, sock: socket.socket) -> None:
        """Serve an already-connected socket (a relayed circuit the server dialled out
        for) exactly like an accepted connection: TLS when configured, the challenge,
        then framed requests."""
        async def serve():
            loop = asyncio.get_running_loop()
            reader = asyncio.StreamReader(limit=1 << 22)
            protocol = asyncio.StreamReaderProtocol(reader)
            transport, _ = await loop.connect_accepted_socket(
                lambda: protocol, sock=sock, **({"ssl": self.tls, "ssl_handshake_timeout": 30.0} if self.tls else {}))
            await self._session(reader, asyncio.StreamWriter(transport, protocol, reader, loop))

        if self._loop is None or not self._loop.is_running() or self._stop:
            sock.close()
            return
        sock.setblocking(False)
        asyncio.run_coroutine_threadsafe(serve(), self._loop)

    # -------------------------------------------------------------- one connection
    async def _read_frame(self, reader: asyncio.StreamReader, cap: int) -> tuple[bytes, int]:
        head = await reader.readexactly(_LEN.size)
        (n,) = _LEN.unpack(head)
        if n > cap:
            raise _Closed(f"frame of {n} bytes above the cap {cap}")
        return await reader.readexactly(n), _LEN.size + n

    @staticmethod
    def _frame(msg: dict) -> bytes:
        body = encode(msg)
        return _LEN.pack(len(body)) + body

    async def _authenticate(self, reader, writer) -> tuple[bool, str | None]:
        """Challenge / response when the server requires it: (accepted, peer id)."""
        if self.auth_keys is None and not self._identity_auth_on():
            return True, None
        nonce = os.urandom(32)
        writer.write(self._frame({"type": "challenge", "nonce": nonce.hex()}))
        await writer.drain()
        body, _ = await self._read_frame(reader, self.max_msg_bytes)
        msg = decode(body)
        if msg.get("type") != "auth":
            return False, None
        if self.auth_keys is not None and "mac" in msg and verify_mac(msg.get("mac", ""), nonce, self.auth_keys):
            accepted, peer = True, None
        elif (self._identity_auth_on() and "pub" in msg and self.peer_admitted(msg.get("pub", ""))
              and verify_auth(msg["pub"], msg.get("sig", ""), nonce)):
            accepted, peer = True, peer_id_of(msg["pub"])
        else:
            return False, None
        writer.write(self._frame({"type": "welcome"}))
        await writer.drain()
        return accepted, peer

    def _serve_one(self, body: bytes, nbytes: int, peer_id):
        """Worker thread: decode, account, handle, encode. Returns (reply, frame) or None."""
        msg = decode(body)
        if msg.get("worker_id") is not None:
            self.metrics.record_worker(msg["worker_id"])
        self.metrics.record_in(msg, nbytes)
        try:
            reply = self._handle(msg, nbytes, peer_id)
        except Exception:
            self.metrics.record_handler_error()
            raise
        return None if reply is None else (reply, self._frame(reply))

    async def _session(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter) -> None:
        if self._stop or len(self._writers) >= self.max_connections:
            writer.transport.abort()
            return
        self._writers.add(writer)
        sock = writer.get_extra_info("socket")
        if sock is not None:
            try:
                sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            except OSError:
                pass
        loop = asyncio.get_running_loop()
        try:
            accepted, peer_id = await self._authenticate(reader, writer)
            while accepted and not self._dead:
                body, nbytes = await self._read_frame(reader, self.max_msg_bytes)
                out = await loop.run_in_executor(self._workers, self._serve_one, body, nbytes, peer_id)
                if out is not None:
                    reply, frame = out
                    writer.write(frame)
                    await writer.drain()
                    self.metrics.record_out(reply, len(frame))
        except (_Closed, asyncio.IncompleteReadError, ConnectionError, ssl.SSLError, OSError, ValueError,
                TypeError, KeyError, RuntimeError):
            pass
        except Exception:  # a handler failure: already counted; the connection is dropped
            pass
        finally:
            self._writers.discard(writer)
            if not writer.is_closing():
                writer.close()


_ReactorServer = ReactorServer
