"""Launcher: config schema + validation, run manifest, CLI, and whole clusters in one
process for every mode (coordinator, static sharded, rendezvous, decentralized), plus
a volunteer ``join`` from a signed manifest. All on CPU over loopback TCP."""

import json
import os
import threading

import pytest

from opendipaco_b200.launch import LaunchConfig, load_config, run_local
from opendipaco_b200.launch.cli import main as cli_main
from opendipaco_b200.launch.cli import starter_config
from opendipaco_b200.launch.manifest import build_manifest, manifest_fingerprint, manifest_to_config, verify_manifest
from opendipaco_b200.schedule import PeerIdentity


def _tiny(mode="coordinator", **sections):
    d = {"mode": mode,
         "model": {"vocab_size": 64, "hidden_size": 32, "num_attention_heads": 4, "intermediate_size": 64,
                   "max_position_embeddings": 64, "layers_per_level": [1, 1], "level_sizes": [2, 2],
                   "sequence_length": 16},
         "diloco": {"inner_steps": 2, "activation_checkpoint": False},
         "data": {"source": "synthetic", "num_documents": 32, "synthetic_doc_len": 40},
         "transport": {"host": "127.0.0.1", "port": 0, "auth_key": "s3cret", "heartbeat_timeout": 10.0},
         "run": {"generations": 1, "batch_size": 4, "local_workers": 2}}
    for k, v in sections.items():
        d.setdefault(k, {}).update(v)
    return LaunchConfig.from_dict(d)


# ------------------------------------------------------------------------ config
def test_defaults_and_unknown_keys():
    cfg = LaunchConfig.from_dict({})
    assert cfg.mode == "coordinator" and cfg.model.level_sizes == [4, 4] and cfg.diloco.activation_checkpoint
    with pytest.raises(ValueError, match="unknown top-level"):
        LaunchConfig.from_dict({"bogus": {}})
    with pytest.raises(ValueError, match="unknown keys"):
        LaunchConfig.from_dict({"model": {"hidden": 3}})


@pytest.mark.parametrize("d, msg", [
    ({"transport": {"down": "delta"}}, "requires mode: sharded"),
    ({"mode": "sharded", "schedule": {"mode": "decentralized"}}, "rendezvous"),
    ({"transport": {"up_density": 0.0}}, "up_density"),
    ({"transport": {"max_mbps": -1}}, "max_mbps"),
    ({"data": {"router_sample": 10}}, "ship: spec"),
    ({"tracker": {"seed_quorum": 2}}, "seed_quorum"),
    ({"tracker": {"seeds": [["h"]]}}, "must be \\[host, port\\]"),
    ({"mode": "ring"}, "mode must be one of"),
])
def test_validation_rejects(d, msg):
    with pytest.raises(ValueError, match=msg):
        LaunchConfig.from_dict(d)


def test_connect_addrs_default_to_loopback_for_wildcards():
    cfg = LaunchConfig.from_dict({"transport": {"host": "0.0.0.0", "port": 7}, "tracker": {"host": "10.0.0.2"}})
    assert cfg.connect_addr() == ("127.0.0.1", 7) and cfg.tracker_connect_addr() == ("10.0.0.2", 29600)


@pytest.mark.parametrize("fmt", ["yaml", "json"])
def test_init_config_round_trip(tmp_path, fmt, capsys):
    out = tmp_path / f"c.{fmt}"
    assert cli_main(["init-config", "--out", str(out), "--mode", "sharded"]) == 0
    assert load_config(out) == starter_config("sharded")


def test_toml_config(tmp_path):
    p = tmp_path / "c.toml"
    p.write_text('mode = "sharded"\n[model]\nhidden_size = 64\n[run]\ngenerations = 2\n')
    cfg = load_config(p)
    assert cfg.mode == "sharded" and cfg.model.hidden_size == 64 and cfg.run.generations == 2


def test_gen_identity(tmp_path, capsys):
    assert cli_main(["gen-identity", "--out", str(tmp_path / "peer.pem")]) == 0
    ident = PeerIdentity.load(tmp_path / "peer.pem")
    assert ident.peer_id in capsys.readouterr().out


# ------------------------------------------------------------------------ manifest
def test_manifest_strips_secrets_and_verifies():
    cfg = _tiny(transport={"grant_key": "g", "identity_key": "/secret/key.pem"}, data={"cache_path": "/x"})
    ident = PeerIdentity.generate()
    m = build_manifest(cfg, identity=ident)
    body = m["config"]
    assert body["transport"]["auth_key"] is None and body["transport"]["grant_key"] is None
    assert body["transport"]["identity_key"] is None and body["data"]["cache_path"] is None
    assert verify_manifest(m) and verify_manifest(m, server_pub=ident.public_key_hex)
    assert not verify_manifest(m, server_pub=PeerIdentity.generate().public_key_hex)
    tampered = json.loads(json.dumps(m))
    tampered["config"]["run"]["generations"] = 99
    assert not verify_manifest(tampered)
    unsigned = build_manifest(cfg)
    assert verify_manifest(unsigned) and not verify_manifest(unsigned, server_pub=ident.public_key_hex)
    assert manifest_fingerprint(m) == manifest_fingerprint(unsigned)
    back = manifest_to_config(m, overrides={"run": {"device": "cpu", "max_tasks": 3}, "transport": {"port": 5}})
    assert back.run.max_tasks == 3 and back.transport.port == 5 and back.model == cfg.model


# ------------------------------------------------------------------------ clusters
def _all_paths_done(completed, n=4):
    assert len(completed) == n and min(completed.values()) >= 1, completed


def test_run_local_coordinator():
    server, completed = run_local(_tiny())
    _all_paths_done(completed)
    assert server.metrics.accepted_updates >= 4


def test_run_local_sharded_static():
    cfg = _tiny("sharded", sharded={"num_shards": 2}, transport={"grant_key": "g"})
    sched, completed = run_local(cfg)
    _all_paths_done(completed)
    assert sched.metrics.accepted_updates >= 4


def test_run_local_rendezvous():
    cfg = _tiny("sharded", sharded={"num_shards": 3},
                ownership={"mode": "rendezvous", "k": 2, "epoch_poll_interval": 0.2, "min_epoch_interval": 0.0,
                           "owner_grace": 60.0, "replicate_interval": 0.5, "heartbeat_interval": 1.0},
                tracker={"ttl": 30.0})
    sched, completed = run_local(cfg)
    _all_paths_done(completed)
    assert sched._epoch_record is not None and len(sched._epoch_record["owners"]) == 3


def test_run_local_decentralized():
    cfg = _tiny("sharded", sharded={"num_shards": 2},
                ownership={"mode": "rendezvous", "k": 2, "heartbeat_interval": 1.0, "replicate_interval": 2.0},
                schedule={"mode": "decentralized", "read_quorum": 1, "lease_ttl": 5.0})
    cluster, completed = run_local(cfg)
    _all_paths_done(completed)
    bank = cluster.merged_bank()
    assert set(bank) == set(cfg_keys(cfg))


def cfg_keys(cfg):
    from opendipaco_b200.launch.config import dipaco_config

    return dipaco_config(cfg.model).build_topology().module_keys()


def test_join_from_signed_manifest(tmp_path):
    from opendipaco_b200.launch.client import run_join, resolve_device
    from opendipaco_b200.launch.roles import run_coordinator

    ident = PeerIdentity.generate()
    key = tmp_path / "server.pem"
    ident.save(key)
    cfg = _tiny(transport={"identity_key": str(key)})
    box, ready = {}, threading.Event()

    def on_start(s):
        box["s"] = s
        ready.set()

    th = threading.Thread(target=lambda: box.__setitem__("r", run_coordinator(cfg, on_start=on_start)), daemon=True)
    th.start()
    assert ready.wait(60)
    addr = f"127.0.0.1:{box['s'].port}"
    assert resolve_device(None, requested="cpu", batch_size=4, seq_len=16)[0] == "cpu"
    with pytest.raises(SystemExit, match="verification failed"):
        run_join(scheduler=addr, auth_key="s3cret", device="cpu", quiet=True,
                 server_pub=PeerIdentity.generate().public_key_hex)
    run_join(scheduler=addr, auth_key="s3cret", device="cpu", quiet=True, server_pub=ident.public_key_hex)
    th.join(timeout=120)
    _all_paths_done(box["r"][1])


def _train_cfg(tmp_path, **comm):
    from opendipaco_b200.launch.config import LaunchConfig

    return LaunchConfig.from_dict({
        "model": {"vocab_size": 256, "hidden_size": 64, "num_attention_heads": 2, "intermediate_size": 128,
                  "layers_per_level": [1, 1], "level_sizes": [2, 2], "sequence_length": 32,
                  "max_position_embeddings": 64},
        "diloco": {"inner_steps": 2, "activation_checkpoint": False},
        "data": {"num_documents": 64, "synthetic_doc_len": 48, "routing": "round_robin"},
        "run": {"generations": 2, "batch_size": 2, "checkpoint_dir": str(tmp_path / "ck")},
        "comm": comm, "kernels": {"fused": False}})


def test_train_command_single_process(tmp_path):
    from opendipaco_b200.launch.train import run_train

    hist = run_train(_train_cfg(tmp_path))
    assert len(hist) == 2 and all(m.inner_loss == m.inner_loss for m in hist)
    assert (tmp_path / "ck" / "round000002" / "rank0.pt").exists()


def test_comm_and_kernels_sections_validate():
    from opendipaco_b200.launch.config import LaunchConfig

    cfg = LaunchConfig.from_dict({"comm": {"backend": "nvlink", "outer_compress": "int4", "dp": 2},
                                  "kernels": {"attention": "mma", "peer_wait_ms": 50}})
    assert cfg.comm.dp == 2 and cfg.kernels.attention == "mma"
    for bad in ({"comm": {"backend": "gloo"}}, {"comm": {"outer_compress": "int4", "backend": "nccl"}},
                {"comm": {"outer_density": 0}}, {"kernels": {"attention": "triton"}}, {"kernels": {"peer": 1}}):
        with pytest.raises(ValueError):
            LaunchConfig.from_dict(bad)


def test_train_command_two_gloo_ranks(tmp_path):
    """``opendipaco train`` under torchrun: two CPU ranks (gloo) with the NCCL-style
    backend; both ranks end with identical shared modules."""
    import subprocess
    import sys

    import torch
    import yaml

    cfg = _train_cfg(tmp_path, backend="nccl").to_dict()
    path = tmp_path / "c.yaml"
    path.write_text(yaml.safe_dump(cfg))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29633", "-m", "opendipaco_b200.launch",
           "train", "--config", str(path)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ, OMP_NUM_THREADS="1"))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    a = torch.load(tmp_path / "ck" / "round000002" / "rank0.pt", weights_only=False)
    b = torch.load(tmp_path / "ck" / "round000002" / "rank1.pt", weights_only=False)
    shared = [k for k in a["bank"] if k in b["bank"] and ".p" not in k]
    assert shared
    for k in shared:
        for n in a["bank"][k]:
            assert torch.equal(a["bank"][k][n], b["bank"][k][n]), (k, n)
