"""Volunteer client: ``opendipaco join``.

A volunteer needs only a scheduler (or tracker) address and a credential. Joining runs
four steps, each a small function below:

1. fetch the run manifest from the address and verify it (against a pinned signer key,
   or trusting the signer on first use; an unsigned manifest is accepted with a
   warning, since then only the channel protects it);
2. choose a device -- the requested one, else CUDA, then Apple MPS, then the CPU -- and,
   on a GPU, the cheapest set of memory levers (bf16 inner loop, then activation
   checkpointing, then chunked logits) under which one path fits 90 % of the free
   memory; a GPU that cannot hold the path falls back to the CPU unless it was forced;
3. turn the manifest into a launch config with this volunteer's overrides;
4. run the ordinary worker role, with an optional bandwidth cap and a periodic health
   line that also notices when the machine was suspended (wall clock jumps).

Command-line surface and manifest handling follow the reference's
``src/opendipaco/launch/client.py``.
"""

from __future__ import annotations

import threading
import time
from dataclasses import dataclass, field

import torch

from ..schedule import PeerIdentity
from ..schedule.throttle import TokenBucket, rate_from_mbps
from ..schedule.tracker import tracker_rpc
from .config import dipaco_config
from .manifest import manifest_fingerprint, manifest_to_config, verify_manifest
from .roles import run_worker_role

# memory levers, cheapest first: (DiLoCo overrides, description)
MEMORY_LEVERS = (
    ({}, "no levers"),
    ({"inner_autocast": True}, "bf16 inner loop"),
    ({"inner_autocast": True, "activation_checkpoint": True}, "+ activation checkpoint"),
    ({"inner_autocast": True, "activation_checkpoint": True, "loss_chunks": 4}, "+ chunked logits"),
)
_USABLE_FRACTION = 0.9  # of the free device memory a path may plan for


def _split_addr(addr) -> tuple[str, int]:
    if isinstance(addr, (tuple, list)):
        return str(addr[0]), int(addr[1])
    host, sep, port = str(addr).rpartition(":")
    if not (sep and host and port):
        raise ValueError(f"address must be host:port, got {addr!r}")
    return host, int(port)


def _have_mps() -> bool:
    backend = getattr(torch.backends, "mps", None)
    return bool(backend is not None and backend.is_available())


@dataclass
class DeviceChoice:
    device: str
    overrides: dict = field(default_factory=dict)  # DiLoCo fields that make the path fit
    notes: list = field(default_factory=list)


def _check_forced(dev: str) -> None:
    kind = dev.split(":")[0]
    if kind not in ("cpu", "cuda", "mps"):
        raise SystemExit(f"--device {dev!r} not recognized (cpu, cuda[:N] or mps)")
    if kind == "cuda" and not torch.cuda.is_available():
        raise SystemExit("--device cuda requested but no CUDA device is available")
    if kind == "mps" and not _have_mps():
        raise SystemExit("--device mps requested but MPS is unavailable")


def choose_device(config, *, requested=None, batch_size: int, seq_len: int) -> DeviceChoice:
    forced = requested not in (None, "auto")
    if forced:
        _check_forced(requested)
        dev = requested
    else:
        dev = "cuda" if torch.cuda.is_available() else ("mps" if _have_mps() else "cpu")
    choice = DeviceChoice(dev, notes=[f"using {dev}" + ("" if forced or dev == "cpu" else " (autodetected)")])
    if not (dev.startswith("cuda") and torch.cuda.is_available()):
        return choice
    from ..train.memory import fits, vram_breakdown

    def need(levers: dict) -> dict:
        return vram_breakdown(config, batch_size=batch_size, seq_len=seq_len,
                              autocast=levers.get("inner_autocast", False),
                              checkpoint=levers.get("activation_checkpoint", False),
                              chunked_logits=levers.get("loss_chunks", 1) > 1)

    try:
        budget = int(torch.cuda.mem_get_info()[0] * _USABLE_FRACTION)
    except Exception as exc:
        if forced:
            raise SystemExit(f"--device {dev}: CUDA memory probe failed: {exc}") from exc
        return DeviceChoice("cpu", notes=choice.notes + [f"CUDA memory probe failed ({exc}); using cpu"])
    for levers, label in MEMORY_LEVERS:
        plan = need(levers)
        if fits(plan, budget):
            if levers:
                choice.notes.append(f"VRAM fit: enabled {label} (~{plan['total'] / 1e9:.1f} GB of "
                                    f"{budget / 1e9:.1f} GB)")
            choice.overrides = dict(levers)
            return choice
    most = need(MEMORY_LEVERS[-1][0])["total"]
    if forced:
        raise SystemExit(f"path does not fit {dev}: needs ~{most / 1e9:.1f} GB with every lever, "
                         f"~{budget / 1e9:.1f} GB usable")
    return DeviceChoice("cpu", notes=choice.notes + [f"VRAM too small (~{most / 1e9:.1f} GB needed); using cpu"])


def resolve_device(config, *, requested=None, batch_size: int, seq_len: int):
    """``(device, DiLoCo overrides, notes)`` (see :func:`choose_device`)."""
    c = choose_device(config, requested=requested, batch_size=batch_size, seq_len=seq_len)
    return c.device, c.overrides, c.notes


def fetch_manifest(addr, *, auth_key=None, tls=None, timeout: float = 10.0) -> dict:
    host, port = _split_addr(addr)
    reply = tracker_rpc((host, port), {"type": "manifest"}, auth_key=auth_key, tls=tls, timeout=timeout) or {}
    if reply.get("manifest") is None:
        raise SystemExit(f"{host}:{port} publishes no run manifest; join with a config file "
                         "(`opendipaco worker --config ...`) instead")
    return reply["manifest"]


def _trusted_manifest(source, cred, tls, server_pub) -> dict:
    manifest = fetch_manifest(source, auth_key=cred, tls=tls)
    if not verify_manifest(manifest, server_pub=server_pub):
        raise SystemExit("manifest verification failed (bad signature or --server-pub mismatch)")
    content = manifest_fingerprint(manifest)
    if server_pub is not None:
        print(f"[join] manifest verified against the pinned key (content {content})")
    elif "sig" in manifest:
        print(f"[join] trusting manifest signer {manifest.get('pub', '?')} on first use (content {content}); "
              "pin it with --server-pub")
    else:
        print(f"[join] accepting an UNSIGNED manifest (content {content}); only the channel protects it")
    return manifest


class HealthReporter:
    """Prints a status line every ``interval`` seconds. The loop waits on a monotonic
    clock, which stops while the machine is suspended, so a jump of the wall clock
    between two lines means the machine slept (its leases were fenced meanwhile)."""

    def __init__(self, *, target, device, interval: float = 10.0, quiet: bool = False, bucket=None,
                 cap_mbps=None):
        self.target, self.device, self.interval, self.quiet = target, device, interval, quiet
        self.bucket, self.cap_mbps = bucket, cap_mbps
        self._halt = threading.Event()
        self._thread = None

    def _bytes(self) -> int:
        return self.bucket.sent_bytes + self.bucket.recv_bytes if self.bucket else 0

    def _line(self, started: float, now: float, dt: float, moved: int) -> str:
        text = f"[join] training on {self.device} -> {self.target}  up {now - started:.0f}s"
        if self.bucket is not None and dt > 0:
            cap = f"/{self.cap_mbps:g}" if self.cap_mbps else ""
            text += f"  {moved * 8 / 1e6 / dt:.2f}{cap} Mbps  ({self._bytes() / 1e6:.1f} MB total)"
        return text

    def _run(self) -> None:
        started = last = time.time()
        seen = self._bytes()
        asleep_after = max(3 * self.interval, 30.0)
        while not self._halt.wait(self.interval):
            now = time.time()
            if now - last > asleep_after:
                print(f"[join] resumed after ~{now - last:.0f}s suspended; stale work is refused by the lease "
                      "fence", flush=True)
            total = self._bytes()
            print(self._line(started, now, now - last, total - seen), flush=True)
            last, seen = now, total

    def start(self) -> None:
        if not self.quiet:
            self._thread = threading.Thread(target=self._run, name="odp-join-health", daemon=True)
            self._thread.start()

    def stop(self) -> None:
        self._halt.set()
        if self._thread is not None:
            self._thread.join(timeout=1)


def run_join(*, scheduler=None, tracker=None, auth_key=None, identity_key=None, device=None, max_tasks=None,
             server_pub=None, data_dir=None, max_mbps=None, max_shards=None, verify_routing=False, quiet=False,
             tls=None, stop_event=None) -> None:
    if (scheduler is None) == (tracker is None):
        raise SystemExit("join needs exactly one of --scheduler / --tracker")
    source = scheduler if scheduler is not None else tracker
    try:
        cred = PeerIdentity.load(identity_key) if identity_key else auth_key
    except (OSError, ValueError) as exc:
        raise SystemExit(f"could not load --identity {identity_key!r}: {exc}") from exc
    manifest = _trusted_manifest(source, cred, tls, server_pub)
    base = manifest_to_config(manifest)
    if base.tls.enabled and tls is None:
        raise SystemExit("this run uses TLS; join with `opendipaco worker --config <file>` and its TLS settings")
    choice = choose_device(dipaco_config(base.model), requested=device, batch_size=base.run.batch_size,
                           seq_len=base.model.sequence_length)
    for note in choice.notes:
        print(f"[join] {note}")
    host, port = _split_addr(source)
    overrides = {"run": {"device": choice.device, "max_tasks": max_tasks, "worker_max_shards": max_shards,
                         "verify_routing": True if verify_routing else None},
                 "transport": {"auth_key": auth_key, "identity_key": identity_key},
                 "diloco": choice.overrides}
    if data_dir is not None:
        overrides["data"] = {"shard_cache_dir": data_dir}
    if scheduler is not None:
        overrides["transport"].update(connect_host=host, port=port)
    else:
        overrides["tracker"] = {"connect_host": host, "port": port}
    cfg = manifest_to_config(manifest, overrides=overrides)
    rate = rate_from_mbps(max_mbps)
    bucket = TokenBucket(rate) if rate else None
    if bucket is not None:
        print(f"[join] bandwidth cap: {max_mbps:g} Mbps (send + receive)")
    health = HealthReporter(target=f"{host}:{port}", device=choice.device, quiet=quiet, bucket=bucket,
                            cap_mbps=max_mbps)
    health.start()
    try:
        run_worker_role(cfg, max_tasks=max_tasks, stop_event=stop_event, bucket=bucket)
    finally:
        health.stop()
