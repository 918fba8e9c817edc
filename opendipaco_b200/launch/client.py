"""Volunteer client: ``opendipaco join`` (reference ``src/opendipaco/launch/client.py``).

With only a scheduler (or tracker) address and a credential, a volunteer fetches
the run manifest, verifies it (pinned key or trust-on-first-use), picks a device
(``cuda > mps > cpu``) and checks the path fits its memory -- switching on bf16,
activation checkpointing and chunked logits in that order before giving up on the
GPU -- then runs the ordinary worker role, printing a periodic health line that
also reports when the machine was suspended.
"""

from __future__ import annotations

import threading
import time

import torch

from ..schedule import PeerIdentity
from ..schedule.throttle import TokenBucket, rate_from_mbps
from ..schedule.tracker import tracker_rpc
from .config import dipaco_config
from .manifest import manifest_fingerprint, manifest_to_config, verify_manifest
from .roles import run_worker_role

# memory-saving switches, tried in this order until the path fits
_FIT_LADDER = (
    ({}, "no levers"),
    ({"inner_autocast": True}, "bf16 inner loop"),
    ({"inner_autocast": True, "activation_checkpoint": True}, "+ activation checkpoint"),
    ({"inner_autocast": True, "activation_checkpoint": True, "loss_chunks": 4}, "+ chunked logits"),
)


def _split_addr(addr) -> tuple[str, int]:
    if isinstance(addr, (tuple, list)):
        return str(addr[0]), int(addr[1])
    host, _, port = str(addr).rpartition(":")
    if not host or not port:
        raise ValueError(f"address must be host:port, got {addr!r}")
    return host, int(port)


def _mps() -> bool:
    m = getattr(torch.backends, "mps", None)
    return m is not None and m.is_available()


def resolve_device(config, *, requested=None, batch_size: int, seq_len: int):
    """``(device, diloco_overrides, notes)``; a forced device that cannot hold the path raises."""
    forced = requested not in (None, "auto")
    if forced:
        dev = requested
        if not (dev == "cpu" or dev.startswith("cuda") or dev.startswith("mps")):
            raise SystemExit(f"--device {dev!r} not recognized (cpu, cuda[:N] or mps)")
        if dev.startswith("cuda") and not torch.cuda.is_available():
            raise SystemExit("--device cuda requested but no CUDA device is available")
        if dev.startswith("mps") and not _mps():
            raise SystemExit("--device mps requested but MPS is unavailable")
    else:
        dev = "cuda" if torch.cuda.is_available() else "mps" if _mps() else "cpu"
    notes = [f"using {dev}" + ("" if forced or dev == "cpu" else " (autodetected)")]
    if not (dev.startswith("cuda") and torch.cuda.is_available()):
        return dev, {}, notes
    from ..train.memory import fits, vram_breakdown

    try:
        free = int(torch.cuda.mem_get_info()[0] * 0.9)
    except Exception as exc:
        if forced:
            raise SystemExit(f"--device {dev}: CUDA memory probe failed: {exc}") from exc
        return "cpu", {}, notes + [f"CUDA memory probe failed ({exc}); using cpu"]
    for over, label in _FIT_LADDER:
        bd = vram_breakdown(config, batch_size=batch_size, seq_len=seq_len, autocast=over.get("inner_autocast", False),
                            checkpoint=over.get("activation_checkpoint", False),
                            chunked_logits=over.get("loss_chunks", 1) > 1)
        if fits(bd, free):
            if over:
                notes.append(f"VRAM fit: enabled {label} (~{bd['total'] / 1e9:.1f} GB of {free / 1e9:.1f} GB)")
            return dev, dict(over), notes
    need = vram_breakdown(config, batch_size=batch_size, seq_len=seq_len, autocast=True, checkpoint=True,
                          chunked_logits=True)["total"]
    if forced:
        raise SystemExit(f"path does not fit {dev}: needs ~{need / 1e9:.1f} GB with every lever, "
                         f"~{free / 1e9:.1f} GB usable")
    return "cpu", {}, notes + [f"VRAM too small (~{need / 1e9:.1f} GB needed); using cpu"]


def fetch_manifest(addr, *, auth_key=None, tls=None, timeout: float = 10.0) -> dict:
    host, port = _split_addr(addr)
    m = (tracker_rpc((host, port), {"type": "manifest"}, auth_key=auth_key, tls=tls, timeout=timeout) or {}).get(
        "manifest")
    if m is None:
        raise SystemExit(f"{host}:{port} publishes no run manifest; join with a config file "
                         "(`opendipaco worker --config ...`) instead")
    return m


class HealthReporter:
    """One status line every ``interval`` s; a wall-clock gap (the monotonic clock stops
    during suspend on Linux) is reported as a resume from sleep."""

    def __init__(self, *, target, device, interval: float = 10.0, quiet: bool = False, bucket=None,
                 cap_mbps=None):
        self.target, self.device, self.interval, self.quiet = target, device, interval, quiet
        self.bucket, self.cap_mbps = bucket, cap_mbps
        self._stop = threading.Event()
        self._thread = None

    def start(self) -> None:
        if not self.quiet:
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()

    def _bandwidth(self, dt, prev):
        if self.bucket is None or dt <= 0:
            return "", prev
        cur = (self.bucket.sent_bytes, self.bucket.recv_bytes)
        mbps = (sum(cur) - sum(prev)) * 8 / 1e6 / dt
        cap = f"/{self.cap_mbps:g}" if self.cap_mbps else ""
        return f"  {mbps:.2f}{cap} Mbps  ({sum(cur) / 1e6:.1f} MB total)", cur

    def _loop(self) -> None:
        start = last = time.time()
        prev = (self.bucket.sent_bytes, self.bucket.recv_bytes) if self.bucket else (0, 0)
        gap = max(3 * self.interval, 30.0)
        while not self._stop.wait(self.interval):
            now = time.time()
            if now - last > gap:
                print(f"[join] resumed after ~{now - last:.0f}s suspended; stale work is refused by the lease "
                      "fence", flush=True)
            bw, prev = self._bandwidth(now - last, prev)
            last = now
            print(f"[join] training on {self.device} -> {self.target}  up {now - start:.0f}s{bw}", flush=True)

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=1)


def run_join(*, scheduler=None, tracker=None, auth_key=None, identity_key=None, device=None, max_tasks=None,
             server_pub=None, data_dir=None, max_mbps=None, max_shards=None, verify_routing=False, quiet=False,
             tls=None, stop_event=None) -> None:
    if (scheduler is None) == (tracker is None):
        raise SystemExit("join needs exactly one of --scheduler / --tracker")
    source = scheduler or tracker
    try:
        cred = PeerIdentity.load(identity_key) if identity_key else auth_key
    except (OSError, ValueError) as exc:
        raise SystemExit(f"could not load --identity {identity_key!r}: {exc}") from exc
    manifest = fetch_manifest(source, auth_key=cred, tls=tls)
    if not verify_manifest(manifest, server_pub=server_pub):
        raise SystemExit("manifest verification failed (bad signature or --server-pub mismatch)")
    fp = manifest_fingerprint(manifest)
    if server_pub is not None:
        print(f"[join] manifest verified against the pinned key (content {fp})")
    elif "sig" in manifest:
        print(f"[join] trusting manifest signer {manifest.get('pub', '?')} on first use (content {fp}); "
              "pin it with --server-pub")
    else:
        print(f"[join] accepting an UNSIGNED manifest (content {fp}); only the channel protects it")
    base = manifest_to_config(manifest)
    if base.tls.enabled and tls is None:
        raise SystemExit("this run uses TLS; join with `opendipaco worker --config <file>` and its TLS settings")
    dev, fit_over, notes = resolve_device(dipaco_config(base.model), requested=device,
                                          batch_size=base.run.batch_size, seq_len=base.model.sequence_length)
    for n in notes:
        print(f"[join] {n}")
    run_over = {"device": dev, "max_tasks": max_tasks, "worker_max_shards": max_shards,
                "verify_routing": True if verify_routing else None}
    over = {"run": run_over, "transport": {"auth_key": auth_key, "identity_key": identity_key}, "diloco": fit_over}
    if data_dir is not None:
        over["data"] = {"shard_cache_dir": data_dir}
    host, port = _split_addr(source)
    if scheduler is not None:
        over["transport"].update(connect_host=host, port=port)
    else:
        over["tracker"] = {"connect_host": host, "port": port}
    cfg = manifest_to_config(manifest, overrides=over)
    rate = rate_from_mbps(max_mbps)
    bucket = TokenBucket(rate) if rate else None
    if bucket is not None:
        print(f"[join] bandwidth cap: {max_mbps:g} Mbps (send + receive)")
    rep = HealthReporter(target=f"{host}:{port}", device=dev, quiet=quiet, bucket=bucket, cap_mbps=max_mbps)
    rep.start()
    try:
        run_worker_role(cfg, max_tasks=max_tasks, stop_event=stop_event, bucket=bucket)
    finally:
        rep.stop()
