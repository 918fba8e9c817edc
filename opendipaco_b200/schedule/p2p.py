"""libp2p transport seam (reference ``src/opendipaco/schedule/p2p.py``).

The reference's optional NAT tier runs its RPCs over libp2p streams (Noise-secured,
relay circuits, hole punching) with a trio thread behind a synchronous facade. The
``libp2p`` and ``trio`` packages are an optional extra there and are not installed
in this framework's image, so this module keeps the *interface*:

* ``parse_p2p_addr`` / ``parse_circuit_addr`` split ``/…/p2p/<id>`` and
  ``<relay>/p2p-circuit/p2p/<dest>`` multiaddrs (pure Python, always available);
* ``Libp2pTransport``, ``serve_over_libp2p`` and ``Libp2pLink`` (the worker-link
  seam: ``sch_rpc`` / ``sch_send`` / ``ps_rpc`` / ``close``) import libp2p lazily
  and raise ``Libp2pUnavailable`` with a clear message when it is missing.

Everything else in ``schedule`` runs over the TCP reactor (optionally TLS). ``nat``
peers are reached through this framework's own TCP circuit relay (``relay.py``):
reservations, circuit multiaddrs of the same form, end-to-end authenticated sessions,
without hole punching.
"""

from __future__ import annotations

RPC_PROTOCOL = "/opendipaco/rpc/1.0.0"
CIRCUIT_SEP = "/p2p-circuit"


class Libp2pUnavailable(ImportError):
    pass


def _require_libp2p():
    try:
        import libp2p  # noqa: F401
        import trio  # noqa: F401
    except ImportError as exc:
        raise Libp2pUnavailable(
            "the libp2p transport needs the optional 'libp2p' and 'trio' packages, which are not installed; "
            "use the TCP transport (public peers) instead") from exc


def parse_p2p_addr(addr: str) -> tuple[str, str]:
    """``/ip4/1.2.3.4/tcp/5/p2p/<id>`` -> (transport part, peer id)."""
    if "/p2p/" not in addr:
        raise ValueError(f"not a /p2p/ multiaddr: {addr!r}")
    head, pid = addr.rsplit("/p2p/", 1)
    if not pid or "/" in pid:
        raise ValueError(f"bad peer id in {addr!r}")
    return head, pid


def parse_circuit_addr(addr: str) -> tuple[str, str]:
    """``<relay multiaddr>/p2p-circuit/p2p/<dest>`` -> (relay multiaddr, dest peer id)."""
    i = addr.find(CIRCUIT_SEP)
    if i < 0:
        raise ValueError(f"not a circuit address: {addr!r}")
    relay, rest = addr[:i], addr[i + len(CIRCUIT_SEP):]
    if not rest.startswith("/p2p/"):
        raise ValueError(f"circuit address without destination: {addr!r}")
    parse_p2p_addr(relay)
    return relay, rest[len("/p2p/"):]


class Libp2pTransport:
    """Synchronous RPC facade over a libp2p host (needs the optional packages)."""

    def __init__(self, identity, *, handler=None, relay: bool = False, listen_addrs=("/ip4/127.0.0.1/tcp/0",),
                 dcutr: bool = True, max_msg_bytes: int | None = None):
        _require_libp2p()
        raise Libp2pUnavailable("libp2p transport is not built into this framework yet")


def serve_over_libp2p(server, *, identity=None, listen_addrs=("/ip4/127.0.0.1/tcp/0",),
                      require_identity: bool = True, dcutr: bool = True, max_msg_bytes: int | None = None):
    return Libp2pTransport(identity or getattr(server, "identity", None), listen_addrs=listen_addrs, dcutr=dcutr,
                           max_msg_bytes=max_msg_bytes)


class Libp2pLink:
    """Worker-link seam over a libp2p transport (same methods as the TCP link)."""

    def __init__(self, transport, sched_addr: str, *, rpc_timeout: float = 120.0, heartbeat_timeout: float = 15.0):
        self._t, self._sched = transport, sched_addr
        self._rpc_timeout, self._hb_timeout = rpc_timeout, heartbeat_timeout

    def sch_rpc(self, msg):
        return self._t.rpc(self._sched, msg, timeout=self._rpc_timeout)

    def sch_send(self, msg) -> None:
        try:
            self._t.rpc(self._sched, msg, timeout=self._hb_timeout)
        except Exception:
            pass

    def ps_rpc(self, addr, msg):
        return self._t.rpc(addr, msg, timeout=self._rpc_timeout)

    def close(self) -> None:
        self._t.close()
