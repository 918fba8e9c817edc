"""``opendipaco`` command line (reference ``src/opendipaco/launch/cli.py``).

    opendipaco run          --config c.yaml        all roles in one process
    opendipaco train        --config c.yaml        synchronous training on this node's GPUs
                                                   (under torchrun: one process per GPU)
    opendipaco coordinator  --config c.yaml        single-node async coordinator
    opendipaco scheduler    --config c.yaml        sharded scheduler (holds no weights)
    opendipaco ps           --config c.yaml --shard-id N
    opendipaco worker       --config c.yaml [--max-tasks N]
    opendipaco join         --scheduler HOST:PORT | --tracker HOST:PORT [--auth S]
    opendipaco ingest       --config c.yaml --shard-id N
    opendipaco tracker      --config c.yaml
    opendipaco relay        --config c.yaml        (circuit relay for peers behind NAT)
    opendipaco init-config  --out c.yaml [--mode sharded]
    opendipaco gen-cert     --out certs/
    opendipaco gen-identity --out peer.pem

Every host of a cluster runs one role from the same config file. Also runnable as
``python -m opendipaco_b200.launch``.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import sys
from pathlib import Path

from .config import DataCfg, DiLoCoCfg, LaunchConfig, ModelCfg, RunCfg, ShardedCfg, load_config


def _report(server, completed) -> None:
    print("per-path updates:", completed)
    print(server.metrics.report())


def cmd_run(a):
    from .roles import run_local

    _report(*run_local(load_config(a.config)))
    return 0


def cmd_train(a):
    from .train import run_train

    hist = run_train(load_config(a.config))
    if hist:
        print(f"final inner loss {hist[-1].inner_loss:.4f} after {len(hist)} rounds")
    return 0


def cmd_coordinator(a):
    from .roles import run_coordinator

    _report(*run_coordinator(load_config(a.config)))
    return 0


def cmd_scheduler(a):
    from .roles import run_scheduler

    _report(*run_scheduler(load_config(a.config)))
    return 0


def cmd_ps(a):
    from .roles import run_parameter_server

    cfg = load_config(a.config)
    print(f"parameter server shard {a.shard_id}/{cfg.sharded.num_shards} on {cfg.transport.host}; Ctrl-C to stop",
          flush=True)
    run_parameter_server(cfg, a.shard_id)
    return 0


def cmd_worker(a):
    from .roles import run_worker_role

    run_worker_role(load_config(a.config), max_tasks=a.max_tasks)
    return 0


def cmd_join(a):
    from .client import run_join

    run_join(scheduler=a.scheduler, tracker=a.tracker, auth_key=a.auth, identity_key=a.identity, device=a.device,
             max_tasks=a.max_tasks, server_pub=a.server_pub, data_dir=a.data_dir, max_mbps=a.max_mbps,
             max_shards=a.max_shards, verify_routing=a.verify_routing, quiet=a.quiet)
    return 0


def cmd_ingest(a):
    from .roles import run_ingest

    docs = run_ingest(load_config(a.config), a.shard_id)
    print(f"ingested {len(docs)} documents for shard {a.shard_id}")
    return 0


def cmd_tracker(a):
    from .roles import run_tracker

    cfg = load_config(a.config)
    print(f"tracker on {cfg.tracker.host}:{cfg.tracker.port} (ttl={cfg.tracker.ttl}s); Ctrl-C to stop", flush=True)
    run_tracker(cfg)
    return 0


def cmd_relay(a):
    from .roles import run_relay

    run_relay(load_config(a.config))
    return 0


def starter_config(mode: str = "coordinator") -> LaunchConfig:
    """A small config that runs end to end in seconds on CPU."""
    cfg = LaunchConfig(mode=mode,
                       model=ModelCfg(vocab_size=4096, hidden_size=128, num_attention_heads=4, intermediate_size=256,
                                      max_position_embeddings=128, layers_per_level=[1, 1], level_sizes=[2, 2],
                                      sequence_length=64),
                       diloco=DiLoCoCfg(inner_steps=10), data=DataCfg(source="synthetic", num_documents=512),
                       run=RunCfg(generations=3, batch_size=16, local_workers=2))
    if mode == "sharded":
        cfg.sharded = ShardedCfg(num_shards=2, parameter_servers=[["127.0.0.1", 29501], ["127.0.0.1", 29502]])
    return cfg


def cmd_init_config(a):
    data = dataclasses.asdict(starter_config(a.mode))
    out = Path(a.out)
    fmt = a.format or ("json" if out.suffix == ".json" else "yaml")
    if fmt == "json":
        out.write_text(json.dumps(data, indent=2) + "\n")
    else:
        import yaml

        out.write_text("# starter config: small and quick; scale model/data/generations and set run.device\n"
                       + yaml.safe_dump(data, sort_keys=False))
    print(f"wrote {a.mode} config to {out}")
    return 0


def cmd_gen_cert(a):
    from ..schedule import generate_selfsigned_cert

    cert, key = generate_selfsigned_cert(a.out, hosts=a.hosts.split(","))
    print(f"cert: {cert}\nkey:  {key}")
    return 0


def cmd_gen_identity(a):
    from ..schedule import PeerIdentity

    ident = PeerIdentity.generate()
    path = ident.save(a.out)
    print(f"key:     {path}\npeer id: {ident.peer_id}\npubkey:  {ident.public_key_hex}")
    print("set transport.identity_key to the key path; add the pubkey to transport.admitted_peers (servers) "
          "or tracker.enroll_peers (tracker)")
    return 0


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="opendipaco", description="DiPaCo cluster launcher")
    sub = p.add_subparsers(dest="command", required=True)

    def with_config(name, help_, func):
        s = sub.add_parser(name, help=help_)
        s.add_argument("--config", required=True, help="cluster config (.yaml/.toml/.json)")
        s.set_defaults(func=func)
        return s

    with_config("run", "stand up the whole cluster locally", cmd_run)
    with_config("train", "synchronous DiLoCo training on this node's GPUs (comm / kernels sections)", cmd_train)
    with_config("coordinator", "run a single-node coordinator", cmd_coordinator)
    with_config("scheduler", "run the sharded scheduler", cmd_scheduler)
    with_config("ps", "run one parameter-server shard", cmd_ps).add_argument("--shard-id", type=int, required=True)
    with_config("worker", "run a worker", cmd_worker).add_argument("--max-tasks", type=int, default=None)
    j = sub.add_parser("join", help="join a run as a volunteer worker (no config file)")
    src = j.add_mutually_exclusive_group(required=True)
    src.add_argument("--scheduler", help="scheduler host:port")
    src.add_argument("--tracker", help="tracker host:port (decentralized run)")
    j.add_argument("--auth", default=None, help="shared secret, if the run uses one")
    j.add_argument("--identity", default=None, help="Ed25519 key PEM (per-peer auth)")
    j.add_argument("--device", default=None, help="cuda / mps / cpu (default: autodetect)")
    j.add_argument("--max-mbps", type=float, default=None, help="bandwidth cap, megabits/s (send + receive)")
    j.add_argument("--max-tasks", type=int, default=None)
    j.add_argument("--max-shards", type=int, default=None, help="materialised shards kept resident")
    j.add_argument("--verify-routing", action="store_true", help="re-fit the shipped router before training")
    j.add_argument("--server-pub", default=None, help="pin the manifest signer's public key")
    j.add_argument("--data-dir", default=None, help="cache directory for spec-materialised shards")
    j.add_argument("--quiet", action="store_true", help="no health line")
    j.set_defaults(func=cmd_join)
    with_config("ingest", "resumably ingest a data shard", cmd_ingest).add_argument("--shard-id", type=int,
                                                                                      required=True)
    with_config("tracker", "run the rendezvous directory", cmd_tracker)
    with_config("relay", "run a circuit relay for peers behind NAT", cmd_relay)
    g = sub.add_parser("gen-identity", help="generate an Ed25519 peer identity")
    g.add_argument("--out", required=True, help="path of the private-key PEM")
    g.set_defaults(func=cmd_gen_identity)
    i = sub.add_parser("init-config", help="write a starter config")
    i.add_argument("--out", required=True)
    i.add_argument("--mode", choices=["coordinator", "sharded"], default="coordinator")
    i.add_argument("--format", choices=["yaml", "json"], default=None)
    i.set_defaults(func=cmd_init_config)
    c = sub.add_parser("gen-cert", help="generate a self-signed TLS certificate (development)")
    c.add_argument("--out", required=True, help="directory for cert.pem / key.pem")
    c.add_argument("--hosts", default="localhost,127.0.0.1")
    c.set_defaults(func=cmd_gen_cert)
    return p


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    return args.func(args)


if __name__ == "__main__":
    sys.exit(main())
