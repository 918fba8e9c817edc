"""The control-plane server core (schedule/reactor.py) on loopback TCP: framed
request / reply with and without TLS, shared-secret and identity authentication, the
frame-size cap, handler failures, the metrics exporter routes and an abrupt crash."""

import json
import socket
import struct
import time
import urllib.request

import pytest
import torch

from opendipaco_b200.schedule import wire
from opendipaco_b200.schedule.identity import PeerIdentity
from opendipaco_b200.schedule.reactor import ReactorServer, TransportMetrics
from opendipaco_b200.schedule.rpc import connect, rpc
from opendipaco_b200.schedule.tls import client_context, generate_selfsigned_cert, server_context


class Echo(ReactorServer):
    """Replies with the request's tensor doubled; "boom" raises inside the handler."""

    def _handle(self, msg, nbytes, peer_id=None):
        if msg.get("type") == "boom":
            raise RuntimeError("handler failure")
        if msg.get("type") == "quiet":
            return None
        return {"type": "echo", "x": msg["x"] * 2, "peer": peer_id, "n": nbytes}


@pytest.fixture
def server(request):
    kw = getattr(request, "param", {})
    srv = Echo(host="127.0.0.1", port=0, io_threads=2, **kw)
    srv.start()
    yield srv
    srv.shutdown()


def test_request_reply_and_ordering(server):
    s = connect(("127.0.0.1", server.port))
    for i in range(20):
        r = rpc(s, {"type": "q", "x": torch.full((3,), float(i))})
        assert r["type"] == "echo" and torch.equal(r["x"], torch.full((3,), 2.0 * i))
    s.close()
    assert server.metrics.bytes_control > 0 and server.metrics.bytes_opt == 0


@pytest.mark.parametrize("server", [{"auth_key": "new", "accept_keys": ["old"]}], indirect=True)
def test_shared_secret_rotation_and_rejection(server):
    for key in ("new", "old"):
        s = connect(("127.0.0.1", server.port), auth_key=key)
        assert rpc(s, {"type": "q", "x": torch.ones(1)})["type"] == "echo"
        s.close()
    with pytest.raises(PermissionError):
        connect(("127.0.0.1", server.port), auth_key="wrong", timeout=2.0)


def test_identity_admission():
    peer, stranger = PeerIdentity.generate(), PeerIdentity.generate()
    srv = Echo(host="127.0.0.1", port=0, admitted_peers=[peer.public_key_hex])
    srv.start()
    try:
        s = connect(("127.0.0.1", srv.port), auth_key=peer)
        assert rpc(s, {"type": "q", "x": torch.ones(1)})["peer"] == peer.peer_id
        s.close()
        with pytest.raises(PermissionError):
            connect(("127.0.0.1", srv.port), auth_key=stranger, timeout=2.0)
        srv.admit_peer(stranger)
        connect(("127.0.0.1", srv.port), auth_key=stranger).close()
        srv.revoke_peer(stranger)
        assert not srv.peer_admitted(stranger.public_key_hex)
    finally:
        srv.shutdown()


def test_tls_round_trip(tmp_path):
    cert, key = generate_selfsigned_cert(str(tmp_path))
    srv = Echo(host="127.0.0.1", port=0, tls=server_context(cert, key), auth_key="k")
    srv.start()
    try:
        s = connect(("127.0.0.1", srv.port), auth_key="k", tls=client_context(cafile=cert, check_hostname=True))
        assert torch.equal(rpc(s, {"type": "q", "x": torch.arange(4.0)})["x"], torch.arange(4.0) * 2)
        assert s.version() in ("TLSv1.2", "TLSv1.3")
        s.close()
    finally:
        srv.shutdown()


@pytest.mark.parametrize("server", [{"max_msg_bytes": 1024}], indirect=True)
def test_oversized_frame_and_handler_error_close_the_connection(server):
    s = connect(("127.0.0.1", server.port))
    s.sendall(struct.pack(">Q", 1 << 20))  # announces a frame above the cap
    s.settimeout(5.0)
    assert s.recv(1) == b""  # closed without reading the body
    s.close()
    s = connect(("127.0.0.1", server.port))
    wire.send_msg(s, {"type": "boom"})
    s.settimeout(5.0)
    assert wire.recv_msg(s) is None
    s.close()
    deadline = time.time() + 5
    while server.metrics.handler_errors == 0 and time.time() < deadline:
        time.sleep(0.02)
    assert server.metrics.handler_errors == 1
    # the server keeps serving other connections
    s = connect(("127.0.0.1", server.port))
    assert rpc(s, {"type": "q", "x": torch.ones(2)})["type"] == "echo"
    s.close()


def test_metrics_exporter_routes(server):
    server.metrics.record_update(3)
    server.metrics.record_worker("w1")
    ex = server.start_metrics_server(host="127.0.0.1", port=0)
    base = f"http://127.0.0.1:{ex.port}"
    prom = urllib.request.urlopen(base + "/metrics", timeout=5).read().decode()
    assert "opendipaco_transport_accepted_updates_total 1" in prom
    assert "# TYPE opendipaco_transport_max_staleness gauge" in prom
    assert "opendipaco_transport_active_workers 1" in prom
    assert urllib.request.urlopen(base + "/healthz", timeout=5).read() == b"ok\n"
    assert "accepted=1" in urllib.request.urlopen(base + "/", timeout=5).read().decode()
    snaps = []
    server.start_metrics_logging(interval=0.05, sink=snaps.append)
    time.sleep(0.3)
    assert snaps and json.dumps(snaps[-1])


def test_traffic_accounting_by_message_type():
    m = TransportMetrics()
    m.record_out({"type": "task", "shared_weights": {"w": torch.zeros(10)}, "shard": torch.zeros(4, dtype=torch.int32),
                  "private_weights": {}}, 1000)
    m.record_out({"type": "idle"}, 10)
    m.record_in({"type": "submit", "shared_grad": [torch.zeros(5)], "private_weights": {"p": torch.zeros(2)}}, 500)
    m.record_in({"type": "heartbeat"}, 7)
    s = m.summary()
    assert (s["tasks_sent"], s["bytes_down"], s["bytes_shared_weights"], s["bytes_shard"]) == (1, 1000, 40, 16)
    assert s["tasks_with_shard"] == 1 and s["tasks_with_private_down"] == 0
    assert (s["submits"], s["bytes_up"], s["bytes_shared_grad"], s["bytes_private_up"]) == (1, 500, 20, 8)
    assert (s["idle"], s["heartbeats"], s["bytes_control"]) == (1, 1, 17)
    m.reclaims += 2
    assert m.summary()["reclaims"] == 2


def test_simulate_crash_drops_connections_and_frees_the_port():
    srv = Echo(host="127.0.0.1", port=0)
    srv.start()
    port = srv.port
    s = connect(("127.0.0.1", port))
    assert rpc(s, {"type": "q", "x": torch.ones(1)})["type"] == "echo"
    srv.simulate_crash()
    s.settimeout(5.0)
    with pytest.raises((ConnectionError, OSError)):
        rpc(s, {"type": "q", "x": torch.ones(1)})
    with pytest.raises(ConnectionError):
        connect(("127.0.0.1", port), timeout=0.5)
    # a restarted server binds the same port
    again = Echo(host="127.0.0.1", port=port)
    again.start()
    try:
        c = connect(("127.0.0.1", port))
        assert rpc(c, {"type": "q", "x": torch.ones(1)})["type"] == "echo"
        c.close()
    finally:
        again.shutdown()
    assert isinstance(socket.gethostname(), str)
