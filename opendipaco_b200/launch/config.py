"""Cluster launch configuration (reference ``src/opendipaco/launch/config.py``).

One file (``.yaml``/``.yml``, ``.toml`` or ``.json``) describes a run; every host of
the cluster reads the same file. Sections: ``model``, ``diloco``, ``data``,
``transport``, ``tls``, ``sharded``, ``tracker``, ``ownership``, ``robustness``,
``schedule``, ``run`` (plus top-level ``mode``) -- names, keys and defaults of the
reference's file format, so existing config files load unchanged -- and two sections of
this framework only: ``comm`` (the collective backend of synchronous multi-GPU training:
NVLink / NCCL, compressed outer payloads, intra-path data parallelism) and ``kernels``
(fused executor, CUDA graphs, attention kernels, cross-GPU wait bound). Neither enters
the model / DiLoCo fingerprint. Unknown keys and contradictory combinations are rejected
when the file is loaded.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field
from pathlib import Path

from ..config import BackboneConfig, DiLoCoConfig, DiPaCoConfig

_WILDCARD = ("0.0.0.0", "::")


@dataclass
class ModelCfg:
    vocab_size: int = 32000
    hidden_size: int = 512
    num_attention_heads: int = 8
    num_key_value_heads: int | None = None
    intermediate_size: int = 1024
    max_position_embeddings: int = 1024
    rope_theta: float = 10000.0
    layers_per_level: list[int] = field(default_factory=lambda: [2, 2])
    level_sizes: list[int] = field(default_factory=lambda: [4, 4])
    embedding: str = "shared"
    head: str = "shared"
    tie_word_embeddings: bool = False
    sequence_length: int = 256
    eval_sequence_length: int | None = None


@dataclass
class DiLoCoCfg:
    inner_steps: int = 50
    inner_lr: float = 4e-4
    inner_weight_decay: float = 0.1
    inner_grad_clip: float | None = 1.0
    inner_lr_schedule: str = "cosine"
    inner_warmup_steps: int = 0
    outer_lr: float = 0.7
    outer_momentum: float = 0.9
    outer_nesterov: bool = True
    rescale_by_sqrt_sharing: bool = True
    inner_autocast: bool = False
    activation_checkpoint: bool = True
    loss_chunks: int = 1
    optim_8bit: bool = False
    dedup_private: bool = False


@dataclass
class DataCfg:
    source: str = "synthetic"               # "synthetic" | "c4"
    num_documents: int = 2000
    max_doc_tokens: int | None = 256
    min_doc_tokens: int = 1
    tokenizer: str | None = None
    cache_path: str | None = None
    shard_cache_dir: str | None = None
    routing: str = "kmeans"                 # "kmeans" | "round_robin"
    router_seed: int = 0
    router_sample: int | None = None        # spec mode: fit the router on a streamed sample
    ship: str = "bytes"                     # "bytes" (packed shards) | "spec" (recipes)
    synthetic_topics: int = 4
    synthetic_doc_len: int = 80


@dataclass
class TLSCfg:
    enabled: bool = False
    certfile: str | None = None
    keyfile: str | None = None
    cafile: str | None = None
    insecure: bool = False
    require_client_cert: bool = False
    server_hostname: str | None = None


@dataclass
class TransportCfg:
    kind: str = "tcp"                       # "tcp" | "libp2p"
    libp2p_listen: list[str] = field(default_factory=lambda: ["/ip4/0.0.0.0/tcp/0"])
    relays: list[str] = field(default_factory=list)
    dcutr: bool = True
    connect_libp2p: str | None = None
    host: str = "0.0.0.0"
    connect_host: str | None = None
    port: int = 29500
    auth_key: str | None = None
    accept_keys: list[str] = field(default_factory=list)
    identity_key: str | None = None
    admitted_peers: list[str] = field(default_factory=list)
    scheduler_pub: str | None = None
    grant_key: str | None = None
    max_msg_bytes: int | None = None
    heartbeat_timeout: float = 20.0
    heartbeat_interval: float = 3.0
    staleness_bound: int | None = None
    staleness_weight: str = "inverse"
    max_update_norm: float | None = None
    compress: str = "none"
    down: str = "full"                      # "full" | "delta"
    up_density: float = 1.0
    max_mbps: float | None = None
    tailor_bandwidth: bool = False
    idle_backoff: float | None = None
    metrics_port: int | None = None
    metrics_host: str = "0.0.0.0"
    metrics_log_interval: float = 0.0


@dataclass
class ShardedCfg:
    num_shards: int = 2
    parameter_servers: list[list] = field(default_factory=list)


@dataclass
class TrackerCfg:
    host: str = "0.0.0.0"
    connect_host: str | None = None
    port: int = 29600
    ttl: float = 30.0
    open_enrollment: bool = False
    enroll_peers: list[str] = field(default_factory=list)
    seeds: list = field(default_factory=list)
    seed_quorum: int = 1


@dataclass
class OwnershipCfg:
    mode: str = "static"                    # "static" | "rendezvous"
    k: int = 3
    salt: str = ""
    bank_seed: int = 0
    replicate_interval: float = 10.0
    owner_grace: float = 60.0
    min_epoch_interval: float = 20.0
    epoch_poll_interval: float = 3.0
    heartbeat_interval: float = 10.0
    advertise_host: str | None = None


@dataclass
class RobustnessCfg:
    mode: str = "off"                       # "off" | "on"
    aggregate: str = "trimmed_mean"
    quorum_target: int = 3
    quorum_timeout: float = 30.0
    redundancy: int = 3
    redundancy_rate: float = 0.0
    audit_timeout: float = 60.0
    version_history: int = 1
    reputation_floor: float = 0.5
    reputation_credit: float = 0.02
    reputation_debit: float = 0.2
    reputation_halflife: float = 3600.0
    min_owner_reputation: float = 0.25
    rate_capacity: float = 8.0
    rate_refill_per_sec: float = 2.0
    private_policy: str = "overwrite"       # "overwrite" | "proposal"
    private_quorum: int = 2
    probe_docs: int = 0
    probe_quorum: int = 0
    probe_abs_margin: float = 0.05
    probe_rel_margin: float = 0.02
    probe_debit: bool = False


@dataclass
class ScheduleCfg:
    mode: str = "central"                   # "central" | "decentralized"
    lease_ttl: float = 20.0
    gossip_interval: float = 10.0
    read_quorum: int = 2


@dataclass
class RunCfg:
    generations: int = 10
    batch_size: int = 8
    seed: int = 0
    device: str = "cpu"
    checkpoint_dir: str | None = None
    checkpoint_every: int = 0
    resume: bool = False
    max_tasks: int | None = None
    local_workers: int = 2
    worker_max_batch: int | None = None
    worker_max_shards: int | None = None
    verify_routing: bool | None = None
    task_seconds: float | None = None
    park_factor: float = 3.0
    min_task_rate: float | None = None


@dataclass
class CommCfg:
    """Collectives of synchronous multi-GPU training (``opendipaco train`` on one node,
    one process per GPU). Not part of the model / DiLoCo fingerprint."""

    backend: str = "auto"                   # "auto" | "nvlink" | "nccl" | "local"
    outer_compress: str = "none"            # NVLink outer step payloads: "none" | "int4" | "topk"
    outer_density: float = 0.01             # top-k: kept fraction of each 4096-element block
    dp: int = 1                             # GPUs per path group (intra-path data parallelism)


@dataclass
class KernelsCfg:
    """B200 execution options of the engine (not part of any fingerprint)."""

    fused: bool | None = None               # None: fused executor on CUDA, module executor on CPU
    cuda_graphs: bool = True                # one CUDA graph per round of inner steps
    attention: str = "auto"                 # "auto" (tcgen05) | "mma" (older mma.sync kernels)
    peer_wait_ms: float = 2000.0            # bound of every wait on another GPU's flag


_SECTIONS = {"model": ModelCfg, "diloco": DiLoCoCfg, "data": DataCfg, "transport": TransportCfg, "tls": TLSCfg,
             "sharded": ShardedCfg, "tracker": TrackerCfg, "ownership": OwnershipCfg, "robustness": RobustnessCfg,
             "schedule": ScheduleCfg, "run": RunCfg, "comm": CommCfg, "kernels": KernelsCfg}


def _dial_host(host: str, connect_host: str | None) -> str:
    return connect_host or (host if host not in _WILDCARD else "127.0.0.1")


@dataclass
class LaunchConfig:
    mode: str = "coordinator"               # "coordinator" | "sharded"
    model: ModelCfg = field(default_factory=ModelCfg)
    diloco: DiLoCoCfg = field(default_factory=DiLoCoCfg)
    data: DataCfg = field(default_factory=DataCfg)
    transport: TransportCfg = field(default_factory=TransportCfg)
    tls: TLSCfg = field(default_factory=TLSCfg)
    sharded: ShardedCfg = field(default_factory=ShardedCfg)
    tracker: TrackerCfg = field(default_factory=TrackerCfg)
    ownership: OwnershipCfg = field(default_factory=OwnershipCfg)
    robustness: RobustnessCfg = field(default_factory=RobustnessCfg)
    schedule: ScheduleCfg = field(default_factory=ScheduleCfg)
    run: RunCfg = field(default_factory=RunCfg)
    comm: CommCfg = field(default_factory=CommCfg)
    kernels: KernelsCfg = field(default_factory=KernelsCfg)

    @classmethod
    def from_dict(cls, d: dict | None) -> "LaunchConfig":
        d = dict(d or {})
        kw = {"mode": d.pop("mode", "coordinator")}
        for name, dc in _SECTIONS.items():
            kw[name] = _section(dc, d.pop(name, None))
        if d:
            raise ValueError(f"unknown top-level config keys: {sorted(d)}")
        cfg = cls(**kw)
        cfg.validate()
        return cfg

    def validate(self) -> None:
        """Reject combinations that cannot work, with the reason."""
        t, r, dt, sch, own = self.transport, self.run, self.data, self.schedule, self.ownership
        sharded = self.mode == "sharded"
        _choice("mode", self.mode, ("coordinator", "sharded"))
        _choice("transport.kind", t.kind, ("tcp", "libp2p"))
        _choice("transport.down", t.down, ("full", "delta"))
        _choice("data.ship", dt.ship, ("bytes", "spec"))
        _choice("ownership.mode", own.mode, ("static", "rendezvous"))
        _choice("schedule.mode", sch.mode, ("central", "decentralized"))
        c, k = self.comm, self.kernels
        _choice("comm.backend", c.backend, ("auto", "nvlink", "nccl", "local"))
        _choice("comm.outer_compress", c.outer_compress, ("none", "int4", "topk"))
        _choice("kernels.attention", k.attention, ("auto", "mma"))
        if not 0.0 < c.outer_density <= 1.0:
            raise ValueError(f"comm.outer_density must be in (0, 1], got {c.outer_density!r}")
        if c.dp < 1:
            raise ValueError(f"comm.dp must be >= 1, got {c.dp}")
        if (c.outer_compress != "none" or c.dp > 1) and c.backend not in ("auto", "nvlink"):
            raise ValueError("comm.outer_compress and comm.dp > 1 need the NVLink backend (comm.backend: nvlink)")
        if k.peer_wait_ms <= 0:
            raise ValueError(f"kernels.peer_wait_ms must be positive, got {k.peer_wait_ms!r}")
        if t.down == "delta" and not sharded:
            raise ValueError("transport.down: delta requires mode: sharded (owners serve the deltas)")
        if not 0.0 < t.up_density <= 1.0:
            raise ValueError(f"transport.up_density must be in (0, 1], got {t.up_density!r}")
        if t.up_density < 1.0 and not sharded:
            raise ValueError("transport.up_density < 1.0 requires mode: sharded")
        m = t.max_mbps
        if m is not None and not (isinstance(m, (int, float)) and not isinstance(m, bool) and math.isfinite(m)
                                  and m > 0):
            raise ValueError(f"transport.max_mbps must be a positive number or null, got {m!r}")
        if t.tailor_bandwidth and not (sharded and sch.mode == "central"):
            raise ValueError("transport.tailor_bandwidth requires mode: sharded with schedule.mode: central")
        if r.task_seconds is not None and not sharded:
            raise ValueError("run.task_seconds requires mode: sharded")
        if r.worker_max_shards is not None and r.worker_max_shards < 1:
            raise ValueError(f"run.worker_max_shards must be >= 1, got {r.worker_max_shards}")
        if dt.router_sample is not None:
            if dt.router_sample < 1:
                raise ValueError(f"data.router_sample must be >= 1, got {dt.router_sample}")
            if dt.ship != "spec":
                raise ValueError("data.router_sample requires data.ship: spec")
            if dt.routing != "kmeans":
                raise ValueError("data.router_sample requires data.routing: kmeans")
        if sch.mode == "decentralized":
            if own.mode != "rendezvous":
                raise ValueError("schedule.mode: decentralized requires ownership.mode: rendezvous")
            if dt.ship == "spec":
                raise ValueError("schedule.mode: decentralized does not support data.ship: spec")
            if t.compress != "none":
                raise ValueError("schedule.mode: decentralized requires transport.compress: none "
                                 "(quorum reads compare replicas byte for byte)")
        for i, s in enumerate(self.tracker.seeds):
            try:
                host, _ = s[0], int(s[1])
            except (TypeError, ValueError, IndexError) as exc:
                raise ValueError(f"tracker.seeds[{i}]={s!r} must be [host, port]") from exc
            if not isinstance(host, str):
                raise ValueError(f"tracker.seeds[{i}] host must be a string, got {host!r}")
        from ..schedule.tracker import dedup_seeds

        n = len(dedup_seeds(self.tracker_connect_addr(), self.tracker.seeds))
        if not 1 <= self.tracker.seed_quorum <= n:
            raise ValueError(f"tracker.seed_quorum ({self.tracker.seed_quorum}) must be in [1, {n}] "
                             "(the number of distinct seeds)")

    def connect_addr(self) -> tuple[str, int]:
        """Where workers dial the coordinator / scheduler."""
        return _dial_host(self.transport.host, self.transport.connect_host), self.transport.port

    def tracker_connect_addr(self) -> tuple[str, int]:
        return _dial_host(self.tracker.host, self.tracker.connect_host), self.tracker.port

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


def _choice(name: str, value, allowed) -> None:
    if value not in allowed:
        raise ValueError(f"{name} must be one of {list(allowed)}, got {value!r}")


def _section(dc, data):
    data = dict(data or {})
    unknown = set(data) - {f.name for f in dataclasses.fields(dc)}
    if unknown:
        raise ValueError(f"unknown keys for [{dc.__name__}]: {sorted(unknown)}")
    return dc(**data)


def load_config(path) -> LaunchConfig:
    """Parse a ``.yaml``/``.yml``, ``.toml`` or ``.json`` cluster config."""
    path = Path(path)
    text = path.read_text()
    suffix = path.suffix.lower()
    if suffix in (".yaml", ".yml"):
        import yaml

        data = yaml.safe_load(text)
    elif suffix == ".toml":
        import tomllib

        data = tomllib.loads(text)
    elif suffix == ".json":
        import json

        data = json.loads(text)
    else:
        raise ValueError(f"unsupported config format {suffix!r}; use .yaml, .toml or .json")
    return LaunchConfig.from_dict(data)


def backbone_config(m: ModelCfg) -> BackboneConfig:
    return BackboneConfig(vocab_size=m.vocab_size, hidden_size=m.hidden_size,
                          num_attention_heads=m.num_attention_heads, num_key_value_heads=m.num_key_value_heads,
                          intermediate_size=m.intermediate_size, max_position_embeddings=m.max_position_embeddings,
                          rope_theta=m.rope_theta, layers_per_level=list(m.layers_per_level))


def dipaco_config(m: ModelCfg) -> DiPaCoConfig:
    return DiPaCoConfig(backbone=backbone_config(m), level_sizes=list(m.level_sizes), embedding=m.embedding,
                        head=m.head, tie_word_embeddings=m.tie_word_embeddings, sequence_length=m.sequence_length,
                        eval_sequence_length=m.eval_sequence_length)


def diloco_config(d: DiLoCoCfg) -> DiLoCoConfig:
    return DiLoCoConfig(inner_steps=d.inner_steps, inner_lr=d.inner_lr, inner_weight_decay=d.inner_weight_decay,
                        inner_grad_clip=d.inner_grad_clip, inner_lr_schedule=d.inner_lr_schedule,
                        inner_warmup_steps=d.inner_warmup_steps, outer_lr=d.outer_lr,
                        outer_momentum=d.outer_momentum, outer_nesterov=d.outer_nesterov,
                        rescale_by_sqrt_sharing=d.rescale_by_sqrt_sharing, inner_autocast=d.inner_autocast,
                        activation_checkpoint=d.activation_checkpoint, loss_chunks=d.loss_chunks,
                        optim_8bit=d.optim_8bit, dedup_private=d.dedup_private)
