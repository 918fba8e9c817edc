"""NAT peers through a TCP circuit relay (CPU, loopback): reservations, relayed RPC
round trips carrying tensors, end-to-end authentication (the server still sees the
client's identity; wrong keys are refused), the relay's own identity check, its
reservation allowlist, failover across several relays, a NAT parameter server serving
fetch and push, and a sharded generation whose owners are all behind the relay.

Behaviours of the reference's ``tests/test_p2p.py`` (libp2p circuit relay), on this
framework's relay (``schedule/relay.py``).
"""

import threading
import time

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.schedule import ParameterServer, PeerIdentity, Scheduler, make_grant, run_sharded_worker
from opendipaco_b200.schedule.reactor import ReactorServer
from opendipaco_b200.schedule.relay import (RelayServer, circuit_addr, dial_circuit, parse_relay_multiaddr,
                                            relay_multiaddr, serve_via_relays)
from opendipaco_b200.schedule.rpc import connect, one_shot, rpc

from helpers import rr_corpus, tiny_config


class _Echo(ReactorServer):
    def _handle(self, msg, nbytes, peer_id=None):
        if msg.get("type") == "boom":
            raise RuntimeError("handler failure")
        return {"type": "echo", "peer": peer_id, "x": msg.get("x")}


@pytest.fixture
def relay():
    r = RelayServer(host="127.0.0.1").start()
    yield r
    r.shutdown()


def _nat_echo(relay, **kw):
    ident = PeerIdentity.generate()
    srv = _Echo(host="127.0.0.1", **kw)
    srv.start()
    (addr,) = serve_via_relays(srv, [relay.multiaddr()], ident)
    return srv, ident, addr


def test_multiaddrs_round_trip():
    rid = PeerIdentity.generate().peer_id
    ma = relay_multiaddr("10.1.2.3", 4001, rid)
    assert ma == f"/ip4/10.1.2.3/tcp/4001/p2p/{rid}" and parse_relay_multiaddr(ma) == ("10.1.2.3", 4001, rid)
    assert relay_multiaddr("relay.example", 9, rid).startswith("/dns4/relay.example/tcp/9/")
    assert circuit_addr(ma, "dest").endswith("/p2p-circuit/p2p/dest")
    with pytest.raises(ValueError):
        parse_relay_multiaddr(f"/ip4/1.2.3.4/udp/1/p2p/{rid}")


def test_relayed_round_trip_carries_tensors(relay):
    srv, ident, addr = _nat_echo(relay)
    try:
        t = torch.arange(12, dtype=torch.float32).reshape(3, 4)
        reply = one_shot(addr, {"type": "x", "x": t})
        assert torch.equal(reply["x"], t) and reply["peer"] is None
        s = connect(addr)  # one circuit, several requests in order
        try:
            assert [rpc(s, {"type": "x", "x": i})["x"] for i in range(5)] == list(range(5))
        finally:
            s.close()
        assert relay.stats["circuits"] >= 2 and relay.stats["bytes"] > t.numel() * 4
    finally:
        srv.shutdown()


def test_authentication_is_end_to_end(relay):
    client = PeerIdentity.generate()
    srv, _, addr = _nat_echo(relay, auth_key="secret", admitted_peers=[client])
    try:
        assert one_shot(addr, {"type": "x"}, auth_key=client)["peer"] == client.peer_id
        assert one_shot(addr, {"type": "x"}, auth_key="secret")["peer"] is None
        with pytest.raises(PermissionError):
            one_shot(addr, {"type": "x"}, auth_key="wrong")
        with pytest.raises(PermissionError):
            one_shot(addr, {"type": "x"}, auth_key=PeerIdentity.generate())
    finally:
        srv.shutdown()


def test_relay_identity_and_missing_reservations(relay):
    srv, ident, addr = _nat_echo(relay)
    try:
        impostor = circuit_addr(relay_multiaddr("127.0.0.1", relay.port, PeerIdentity.generate().peer_id),
                                ident.peer_id)
        with pytest.raises(PermissionError):
            dial_circuit(impostor)
        with pytest.raises(ConnectionError):
            one_shot(circuit_addr(relay.multiaddr(), PeerIdentity.generate().peer_id), {"type": "x"})
    finally:
        srv.shutdown()
    deadline = time.monotonic() + 5  # the reservation ends with the server
    while time.monotonic() < deadline and ident.peer_id in relay.reserved_peers():
        time.sleep(0.05)
    assert ident.peer_id not in relay.reserved_peers()


def test_reservation_allowlist():
    member = PeerIdentity.generate()
    r = RelayServer(host="127.0.0.1", admitted=[member]).start()
    srv = _Echo(host="127.0.0.1")
    srv.start()
    try:
        assert serve_via_relays(srv, [r.multiaddr()], PeerIdentity.generate(), wait=1.0) == []
        assert len(serve_via_relays(srv, [r.multiaddr()], member)) == 1
        assert r.reserved_peers() == [member.peer_id] and r.stats["refused"] >= 1
    finally:
        srv.shutdown()
        r.shutdown()


def test_server_survives_a_raising_handler_over_a_circuit(relay):
    srv, _, addr = _nat_echo(relay)
    try:
        with pytest.raises((ConnectionError, OSError)):
            one_shot(addr, {"type": "boom"}, timeout=5.0)
        assert one_shot(addr, {"type": "x", "x": 1})["x"] == 1
    finally:
        srv.shutdown()


def test_failover_across_candidate_relays(relay):
    dead = RelayServer(host="127.0.0.1").start()
    ident = PeerIdentity.generate()
    srv = _Echo(host="127.0.0.1")
    srv.start()
    try:
        addrs = serve_via_relays(srv, [dead.multiaddr(), relay.multiaddr()], ident)
        assert len(addrs) == 2
        dead.shutdown()
        assert one_shot(addrs, {"type": "x", "x": 7})["x"] == 7  # the first relay is gone
    finally:
        srv.shutdown()


def test_nat_parameter_server_serves_fetch_and_push(relay):
    cfg = tiny_config()
    sched = PeerIdentity.generate()
    keys = cfg.build_topology().module_keys()
    ps = ParameterServer(cfg, keys, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), host="127.0.0.1", auth_key="k",
                         scheduler_pub=sched.public_key_hex)
    ps.start()
    try:
        (addr,) = serve_via_relays(ps, [relay.multiaddr()], PeerIdentity.generate())
        key = keys[0]
        got = one_shot(addr, {"type": "fetch", "keys": [key], "have": {}}, auth_key="k")
        assert key in got["weights"]
        grad = [torch.full(tuple(p.shape), 1e-3) for p in ps.bank[key].parameters()]
        ack = one_shot(addr, {"type": "push", "grant": make_grant((0, 0), [key], 1.0, "t", identity=sched),
                              "updates": {key: {"grad": grad}}, "private": {}}, auth_key="k")
        assert ack["applied"] and ps._versions[key][1] == 1
    finally:
        ps.shutdown()


def test_sharded_generation_with_owners_behind_the_relay(relay):
    """Static shards whose parameter servers are reachable only through the relay: the
    scheduler routes workers to circuit addresses and a generation completes."""
    cfg = tiny_config()
    dl = DiLoCoConfig(inner_steps=2, inner_lr=1e-3)
    keys = sorted(cfg.build_topology().module_keys())
    halves = [keys[0::2], keys[1::2]]
    owners, addrs = [], []
    for shard in halves:
        ps = ParameterServer(cfg, shard, dl, host="127.0.0.1", auth_key="k")
        ps.start()
        owners.append(ps)
        addrs += serve_via_relays(ps, [relay.multiaddr()], PeerIdentity.generate())
    sched = Scheduler(cfg, rr_corpus(cfg), [], dl, 2, host="127.0.0.1", auth_key="k")
    sched._static_routing = {k: addrs[0] if k in halves[0] else addrs[1] for k in keys}
    sched._routing = dict(sched._static_routing)
    sched.start()
    stop = threading.Event()
    w = threading.Thread(target=run_sharded_worker, args=(cfg, dl, ("127.0.0.1", sched.port)),
                         kwargs=dict(auth_key="k", stop_event=stop, heartbeat_interval=1.0), daemon=True)
    w.start()
    try:
        done = sched.fit(num_generations=1)
        assert all(v >= 1 for v in done.values())
        assert all(v[1] >= 1 for ps in owners for v in ps._versions.values())  # every key got its pushes
        assert relay.stats["circuits"] >= 2
    finally:
        stop.set()
        sched.shutdown()
        for ps in owners:
            ps.shutdown()
        w.join(timeout=15)


def test_relay_role_and_a_nat_owner_in_the_directory():
    """``run_relay`` stands up a relay; a NAT owner reserves on it, registers a ``nat``
    record with its circuit address, and an epoch built from the directory dials it
    through the relay."""
    from opendipaco_b200.launch.config import LaunchConfig
    from opendipaco_b200.launch.roles import run_relay
    from opendipaco_b200.schedule import Tracker, fetch_directory, make_epoch_record
    from opendipaco_b200.schedule.ownership import owner_addr

    cfg = LaunchConfig()
    cfg.transport.host = "127.0.0.1"
    box, stop = {}, threading.Event()
    th = threading.Thread(target=run_relay, args=(cfg,), kwargs=dict(on_start=lambda r: box.setdefault("r", r),
                                                                     stop_event=stop, port=0), daemon=True)
    th.start()
    deadline = time.monotonic() + 10
    while "r" not in box and time.monotonic() < deadline:
        time.sleep(0.05)
    relay = box["r"]
    tracker = Tracker(host="127.0.0.1", open_enrollment=True)
    tracker.start()
    mcfg = tiny_config()
    ident, sched = PeerIdentity.generate(), PeerIdentity.generate()
    ps = ParameterServer(mcfg, [], DiLoCoConfig(inner_steps=2), host="127.0.0.1", identity=ident, auth_key="k",
                         scheduler_pub=sched.public_key_hex)
    ps.start()
    try:
        circuits = serve_via_relays(ps, [relay.multiaddr()], ident)
        ps.start_tracker_heartbeat(("127.0.0.1", tracker.port), "unused", interval=0.2, circuit_addrs=circuits)
        deadline = time.monotonic() + 10
        recs = []
        while not recs and time.monotonic() < deadline:
            recs = fetch_directory(("127.0.0.1", tracker.port), roles=["owner"])
            time.sleep(0.05)
        (rec,) = recs
        assert rec["reachability"] == "nat" and rec["addr"] is None and rec["circuit_addrs"] == circuits
        epoch = make_epoch_record(sched, epoch=0, owner_records=recs, k=1, bootstrap=True)
        ps.apply_epoch(epoch)
        dial = owner_addr(epoch["owners"][0])
        assert dial == circuits[0]
        key = mcfg.build_topology().module_keys()[0]
        assert key in one_shot(dial, {"type": "fetch", "keys": [key], "have": {}}, auth_key="k")["weights"]
    finally:
        ps.shutdown()
        tracker.shutdown()
        stop.set()
        th.join(timeout=10)


def test_tls_runs_end_to_end_through_the_relay(relay, tmp_path):
    """With TLS the session is encrypted between client and NAT server: the relay only
    sees the handshake and ciphertext, never the frames' plaintext."""
    from opendipaco_b200.schedule.tls import client_context, generate_selfsigned_cert, server_context

    cert, key = generate_selfsigned_cert(str(tmp_path))
    srv, _, addr = _nat_echo(relay, tls=server_context(cert, key), auth_key="k")
    seen = []
    real_pipe = relay._pipe

    async def spy(src, dst):  # record what crosses the relay
        orig_write = dst.write

        def write(chunk):
            seen.append(bytes(chunk))
            orig_write(chunk)

        dst.write = write
        await real_pipe(src, dst)

    relay._pipe = spy
    try:
        s = connect(addr, auth_key="k", tls=client_context(cafile=cert, check_hostname=False))
        try:
            marker = "plaintext-marker-0123456789"
            assert rpc(s, {"type": "x", "x": marker})["x"] == marker
            assert s.version() in ("TLSv1.2", "TLSv1.3")
        finally:
            s.close()
        assert seen and not any(marker.encode() in c for c in seen)
    finally:
        srv.shutdown()


def test_a_circuit_proof_cannot_be_replayed_as_a_reservation(relay):
    """The relay signs the client's nonce to prove itself; that signature is made in the
    circuit context, so presenting it to another relay as a reservation fails."""
    import socket as _s

    from opendipaco_b200.schedule.wire import recv_msg, send_msg

    srv, _, addr = _nat_echo(relay)
    other = RelayServer(host="127.0.0.1").start()
    try:
        victim = _s.create_connection(("127.0.0.1", other.port), timeout=5)
        nonce = recv_msg(victim)["nonce"]              # the other relay's reservation challenge
        c = _s.create_connection(("127.0.0.1", relay.port), timeout=5)
        recv_msg(c)
        send_msg(c, {"type": "circuit", "target": addr.rsplit("/", 1)[1], "nonce": nonce})
        proof = recv_msg(c)
        assert proof["type"] == "connected"
        send_msg(victim, {"type": "reserve", "pub": proof["relay_pub"], "sig": proof["sig"]})
        assert recv_msg(victim)["type"] == "refused" and other.reserved_peers() == []
        c.close()
        victim.close()
    finally:
        other.shutdown()
        srv.shutdown()
