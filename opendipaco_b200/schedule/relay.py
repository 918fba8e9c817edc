"""Circuit relay over plain TCP: reach peers behind NAT.

A peer that cannot accept inbound connections (``reachability: nat``) keeps an
outbound *reservation* on one or more relays and advertises circuit addresses
``/ip4/<relay host>/tcp/<relay port>/p2p/<relay id>/p2p-circuit/p2p/<peer id>`` in its
signed directory record. A client dials such an address through
:func:`dial_circuit`: the relay tells the reserved peer over its reservation channel,
the peer dials the relay back with the one-time token it received there, and from then
on the relay only copies bytes between the two sockets. What runs over the spliced pair
is the ordinary session (optional TLS, the challenge / response of the server, framed
RPCs), so a relayed peer is authenticated end to end exactly like a directly dialled
one and the relay never sees a key; without TLS the relay can read the frames, with TLS
it cannot.

This is the NAT tier of the reference (``src/opendipaco/schedule/p2p.py``: libp2p
circuit relay v2 with Noise and DCUtR hole punching), built here on the framework's own
TCP transport because the libp2p packages are not part of this image. The multiaddr
form of circuit addresses is kept; the relay protocol is this module's own, and hole
punching is not attempted (every relayed byte goes through the relay).

Relay protocol (framed messages of ``wire.py``):

* reservation: relay ``challenge{nonce}`` -> peer ``reserve{pub, sig}`` (an identity
  signature over the nonce) -> relay ``reserved{ttl}``; the connection stays open and
  carries ``incoming{token}`` notices and ``ping`` keep-alives;
* circuit: client ``circuit{target, nonce}`` -> relay ``connected{relay_pub, sig}``
  (the relay's signature over the client's nonce) once the target dialled back, or
  ``refused{reason}``;
* dial-back: peer ``accept{token}`` on a fresh connection -> spliced.
"""

from __future__ import annotations

import asyncio
import logging
import os
import socket
import threading
import time

from .identity import PeerIdentity, peer_id_of, verify_signature
from .p2p import CIRCUIT_SEP, parse_circuit_addr, parse_p2p_addr
from .wire import _LEN, decode, encode, recv_msg, send_msg

logger = logging.getLogger("opendipaco_b200.schedule")

# distinct signing contexts: a relay's proof to a client can never pass as a reservation
RESERVE_CONTEXT = b"opendipaco-relay-reserve:"
CIRCUIT_CONTEXT = b"opendipaco-relay-circuit:"
CONTROL_MAX_BYTES = 64 * 1024  # relay control frames are tiny


# ------------------------------------------------------------------ addresses
def relay_multiaddr(host: str, port: int, relay_id: str) -> str:
    kind = "ip6" if ":" in host else ("ip4" if host.replace(".", "").isdigit() else "dns4")
    return f"/{kind}/{host}/tcp/{int(port)}/p2p/{relay_id}"


def circuit_addr(relay: str, dest_id: str) -> str:
    """``relay`` (a relay multiaddr with its ``/p2p/<id>``) -> circuit address of ``dest_id``."""
    parse_p2p_addr(relay)
    return f"{relay}{CIRCUIT_SEP}/p2p/{dest_id}"


def parse_relay_multiaddr(addr: str) -> tuple[str, int, str]:
    """``/ip4|ip6|dns4|dns/<host>/tcp/<port>/p2p/<id>`` -> (host, port, relay peer id)."""
    head, rid = parse_p2p_addr(addr)
    parts = head.strip("/").split("/")
    if len(parts) != 4 or parts[0] not in ("ip4", "ip6", "dns4", "dns6", "dns") or parts[2] != "tcp":
        raise ValueError(f"unsupported relay multiaddr {addr!r} (want /ip4/<host>/tcp/<port>/p2p/<id>)")
    return parts[1], int(parts[3]), rid


def is_circuit(addr) -> bool:
    return isinstance(addr, str) and CIRCUIT_SEP in addr


# ------------------------------------------------------------------ relay server
class RelayServer:
    """A forwarding relay: reservations from NAT peers, circuits from clients.

    ``admitted`` (peer ids or identities) limits who may reserve; ``None`` lets any
    identity reserve (circuits carry only end-to-end authenticated sessions).
    ``max_circuits`` bounds the spliced pairs alive at once; a dial-back has
    ``connect_timeout`` seconds to arrive."""

    def __init__(self, identity: PeerIdentity | None = None, *, host: str = "0.0.0.0", port: int = 0,
                 admitted=None, max_circuits: int = 256, connect_timeout: float = 10.0,
                 reservation_ttl: float = 3600.0):
        self.identity = identity or PeerIdentity.generate()
        self.peer_id = self.identity.peer_id
        self.admitted = None if admitted is None else {getattr(a, "peer_id", a) for a in admitted}
        self.max_circuits, self.connect_timeout = max_circuits, connect_timeout
        self.reservation_ttl = reservation_ttl
        self._listener = socket.create_server((host, port), reuse_port=False)
        self._listener.setblocking(False)
        self.host, self.port = host, self._listener.getsockname()[1]
        self._loop = None
        self._thread = None
        self._server = None
        self._reserved: dict = {}     # peer id -> writer of its reservation channel
        self._pending: dict = {}      # token -> future resolved with the dial-back (reader, writer)
        self._circuits = 0
        self.stats = {"reservations": 0, "circuits": 0, "refused": 0, "bytes": 0}

    def multiaddr(self, host: str | None = None) -> str:
        return relay_multiaddr(host or ("127.0.0.1" if self.host in ("0.0.0.0", "") else self.host), self.port,
                               self.peer_id)

    # -- lifecycle
    def start(self) -> "RelayServer":
        self._loop = asyncio.new_event_loop()
        up = threading.Event()

        def run():
            asyncio.set_event_loop(self._loop)
            self._server = self._loop.run_until_complete(asyncio.start_server(self._conn, sock=self._listener))
            up.set()
            try:
                self._loop.run_forever()
            finally:
                pending = [t for t in asyncio.all_tasks(self._loop) if not t.done()]
                for t in pending:
                    t.cancel()
                if pending:
                    self._loop.run_until_complete(asyncio.gather(*pending, return_exceptions=True))
                self._loop.close()

        self._thread = threading.Thread(target=run, name=f"odp-relay-{self.port}", daemon=True)
        self._thread.start()
        if not up.wait(10.0):
            raise RuntimeError("relay event loop did not start")
        return self

    def shutdown(self) -> None:
        loop = self._loop
        if loop is None or not loop.is_running():
            return

        def stop():
            self._server.close()
            for w in list(self._reserved.values()):
                w.transport.abort()
            loop.call_later(0.05, loop.stop)

        loop.call_soon_threadsafe(stop)
        self._thread.join(timeout=5.0)
        try:
            self._listener.close()
        except OSError:
            pass

    def reserved_peers(self) -> list[str]:
        return sorted(self._reserved)

    # -- framing
    @staticmethod
    async def _read(reader) -> dict:
        (n,) = _LEN.unpack(await reader.readexactly(_LEN.size))
        if n > CONTROL_MAX_BYTES:
            raise ValueError("relay control frame too large")
        return decode(await reader.readexactly(n))

    @staticmethod
    async def _write(writer, msg: dict) -> None:
        body = encode(msg)
        writer.write(_LEN.pack(len(body)) + body)
        await writer.drain()

    # -- connections
    async def _conn(self, reader, writer) -> None:
        nonce = os.urandom(32)
        try:
            await self._write(writer, {"type": "challenge", "nonce": nonce.hex()})
            first = await asyncio.wait_for(self._read(reader), self.connect_timeout)
            kind = first.get("type")
            if kind == "reserve":
                await self._reservation(first, nonce, reader, writer)
            elif kind == "circuit":
                await self._circuit(first, reader, writer)
            elif kind == "accept":
                fut = self._pending.pop(str(first.get("token")), None)
                if fut is None or fut.done():
                    writer.transport.abort()
                    return
                fut.set_result((reader, writer))
                return  # the circuit task owns this connection now
            else:
                writer.transport.abort()
        except (asyncio.IncompleteReadError, asyncio.TimeoutError, ConnectionError, OSError, ValueError,
                TypeError, KeyError):
            writer.transport.abort()

    async def _reservation(self, msg, nonce, reader, writer) -> None:
        pub = msg.get("pub")
        if not (isinstance(pub, str) and verify_signature(pub, msg.get("sig"), RESERVE_CONTEXT + nonce)):
            await self._write(writer, {"type": "refused", "reason": "bad signature"})
            writer.transport.abort()
            return
        pid = peer_id_of(pub)
        if self.admitted is not None and pid not in self.admitted:
            self.stats["refused"] += 1
            await self._write(writer, {"type": "refused", "reason": "not admitted"})
            writer.transport.abort()
            return
        old = self._reserved.get(pid)
        if old is not None and old is not writer:
            old.transport.abort()
        self._reserved[pid] = writer
        self.stats["reservations"] += 1
        await self._write(writer, {"type": "reserved", "ttl": self.reservation_ttl, "relay": self.peer_id})
        try:
            while True:  # the peer only pings; the channel ends when it closes
                m = await asyncio.wait_for(self._read(reader), self.reservation_ttl)
                if m.get("type") == "ping":
                    await self._write(writer, {"type": "pong"})
        finally:
            if self._reserved.get(pid) is writer:
                del self._reserved[pid]
            writer.transport.abort()

    async def _circuit(self, msg, reader, writer) -> None:
        target = msg.get("target")
        ctl = self._reserved.get(target) if isinstance(target, str) else None
        if ctl is None or self._circuits >= self.max_circuits:
            self.stats["refused"] += 1
            await self._write(writer, {"type": "refused",
                                       "reason": "no reservation" if ctl is None else "relay full"})
            writer.transport.abort()
            return
        token = os.urandom(16).hex()
        fut = asyncio.get_running_loop().create_future()
        self._pending[token] = fut
        self._circuits += 1
        try:
            await self._write(ctl, {"type": "incoming", "token": token})
            t_reader, t_writer = await asyncio.wait_for(fut, self.connect_timeout)
            nonce = bytes.fromhex(str(msg.get("nonce", "")))
            await self._write(writer, {"type": "connected", "relay_pub": self.identity.public_key_hex,
                                       "sig": self.identity.sign(CIRCUIT_CONTEXT + nonce).hex()})
            self.stats["circuits"] += 1
            await asyncio.gather(self._pipe(reader, t_writer), self._pipe(t_reader, writer))
        except (asyncio.TimeoutError, ConnectionError, OSError, ValueError):
            try:
                await self._write(writer, {"type": "refused", "reason": "target did not answer"})
            except (ConnectionError, OSError):
                pass
            writer.transport.abort()
        finally:
            self._pending.pop(token, None)
            self._circuits -= 1

    async def _pipe(self, src, dst) -> None:
        try:
            while True:
                chunk = await src.read(1 << 16)
                if not chunk:
                    break
                self.stats["bytes"] += len(chunk)
                dst.write(chunk)
                await dst.drain()
        except (ConnectionError, OSError):
            pass
        finally:  # either side ending ends the circuit
            dst.close()


# ------------------------------------------------------------------ client side
def _dial(host: str, port: int, timeout: float) -> socket.socket:
    s = socket.create_connection((host, port), timeout=timeout)
    s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    return s


def dial_circuit(addr: str, timeout: float = 10.0) -> socket.socket:
    """Open a relayed connection to the destination of circuit address ``addr``; the
    returned socket carries the destination server's own session (its challenge
    first). The relay proves the identity named in ``addr``."""
    relay, dest = parse_circuit_addr(addr)
    host, port, relay_id = parse_relay_multiaddr(relay)
    s = _dial(host, port, timeout)
    try:
        s.settimeout(timeout)
        if (recv_msg(s, CONTROL_MAX_BYTES) or {}).get("type") != "challenge":
            raise ConnectionError(f"{relay}: not a relay")
        nonce = os.urandom(32)
        send_msg(s, {"type": "circuit", "target": dest, "nonce": nonce.hex()})
        reply = recv_msg(s, CONTROL_MAX_BYTES) or {}
        if reply.get("type") != "connected":
            raise ConnectionError(f"relay {relay_id[:12]} refused the circuit to {dest[:12]}: "
                                  f"{reply.get('reason', 'closed')}")
        pub = reply.get("relay_pub")
        if not (isinstance(pub, str) and peer_id_of(pub) == relay_id
                and verify_signature(pub, reply.get("sig"), CIRCUIT_CONTEXT + nonce)):
            raise PermissionError(f"the relay at {host}:{port} is not {relay_id[:12]}")
        s.settimeout(None)
        return s
    except BaseException:
        s.close()
        raise


class RelayReservation:
    """The NAT peer's side: keep a reservation on ``relay`` (a relay multiaddr) and hand
    every incoming circuit to ``server`` (a :class:`ReactorServer`) as if it had been
    accepted. Reconnects with backoff while running; ``addr`` is the circuit address
    to advertise."""

    def __init__(self, server, relay: str, identity: PeerIdentity, *, ping_interval: float = 20.0,
                 timeout: float = 10.0):
        self.server, self.relay, self.identity = server, relay, identity
        self.host, self.port, self.relay_id = parse_relay_multiaddr(relay)
        self.addr = circuit_addr(relay, identity.peer_id)
        self.ping_interval, self.timeout = ping_interval, timeout
        self.ready = threading.Event()
        self._stop = threading.Event()
        self._sock = None
        self._thread = threading.Thread(target=self._run, name="odp-relay-reservation", daemon=True)

    def start(self) -> "RelayReservation":
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        s = self._sock
        if s is not None:
            try:
                s.shutdown(socket.SHUT_RDWR)
            except OSError:
                pass
            s.close()
        self._thread.join(timeout=5.0)

    def _reserve(self) -> socket.socket:
        s = _dial(self.host, self.port, self.timeout)
        s.settimeout(self.timeout)
        ch = recv_msg(s, CONTROL_MAX_BYTES) or {}
        if ch.get("type") != "challenge":
            s.close()
            raise ConnectionError("not a relay")
        sig = self.identity.sign(RESERVE_CONTEXT + bytes.fromhex(ch["nonce"])).hex()
        send_msg(s, {"type": "reserve", "pub": self.identity.public_key_hex, "sig": sig})
        reply = recv_msg(s, CONTROL_MAX_BYTES) or {}
        if reply.get("type") != "reserved" or reply.get("relay") != self.relay_id:
            s.close()
            raise PermissionError(f"reservation refused: {reply.get('reason', reply.get('type'))}")
        s.settimeout(self.ping_interval)
        return s

    def _accept(self, token: str) -> None:
        try:
            s = _dial(self.host, self.port, self.timeout)
            s.settimeout(self.timeout)
            if (recv_msg(s, CONTROL_MAX_BYTES) or {}).get("type") != "challenge":
                s.close()
                return
            send_msg(s, {"type": "accept", "token": token})
            s.settimeout(None)
            self.server.adopt_socket(s)
        except (OSError, ConnectionError, ValueError) as exc:
            logger.warning("relayed circuit dial-back failed: %s", exc)

    def _run(self) -> None:
        backoff = 0.1
        while not self._stop.is_set():
            try:
                self._sock = self._reserve()
                self.ready.set()
                backoff = 0.1
                while not self._stop.is_set():
                    try:
                        m = recv_msg(self._sock, CONTROL_MAX_BYTES)
                    except socket.timeout:
                        send_msg(self._sock, {"type": "ping"})
                        continue
                    if m is None:
                        break
                    if m.get("type") == "incoming":
                        threading.Thread(target=self._accept, args=(str(m.get("token")),), daemon=True).start()
            except (OSError, ConnectionError, PermissionError, ValueError) as exc:
                if not self._stop.is_set():
                    logger.info("relay reservation on %s lost: %s", self.relay, exc)
            finally:
                self.ready.clear()
                if self._sock is not None:
                    self._sock.close()
                    self._sock = None
            self._stop.wait(backoff)
            backoff = min(5.0, backoff * 2)


def serve_via_relays(server, relays, identity: PeerIdentity, *, wait: float = 10.0) -> list[str]:
    """Reserve ``server`` on every relay multiaddr in ``relays``; returns the circuit
    addresses of the reservations that came up within ``wait`` seconds (the ones to
    advertise). The reservations stop with the server."""
    res = [RelayReservation(server, r, identity).start() for r in relays]
    server._observers.extend(_Stopper(r) for r in res)
    end = time.monotonic() + wait
    for r in res:
        r.ready.wait(max(0.0, end - time.monotonic()))
    return [r.addr for r in res if r.ready.is_set()]


class _Stopper:
    """Adapter so a server's shutdown also ends its relay reservations."""

    def __init__(self, reservation):
        self.reservation = reservation

    def stop(self) -> None:
        self.reservation.stop()


__all__ = ["RelayServer", "RelayReservation", "dial_circuit", "serve_via_relays", "circuit_addr", "relay_multiaddr",
           "parse_relay_multiaddr", "is_circuit"]
