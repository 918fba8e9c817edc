"""Run manifest (reference ``src/opendipaco/launch/manifest.py``).

A volunteer who joins with only a scheduler/tracker address has no model
description, so the operator's server publishes the launch config minus secrets
(credentials, TLS key material, operator-local paths and limits), signed with the
run's identity when it has one. The joiner verifies it -- pinned to a known key with
``server_pub``, or trust-on-first-use with a printed content fingerprint -- and
rebuilds a validated ``LaunchConfig`` with its own connection flags laid over it.
The manifest record layout is the reference's.
"""

from __future__ import annotations

import copy
import dataclasses
import hashlib
import json
import time

from ..schedule.identity import sign_record, verify_record
from .config import LaunchConfig

MANIFEST_KIND = "run_manifest"
# fields that must not leave the operator's host
_PRIVATE = {
    "transport": ("auth_key", "grant_key", "identity_key", "accept_keys", "admitted_peers", "max_mbps"),
    "run": ("worker_max_batch", "worker_max_shards", "verify_routing"),
    "tls": ("certfile", "keyfile", "cafile"),
    "data": ("cache_path", "shard_cache_dir"),
}


def build_manifest(cfg: LaunchConfig, *, identity=None) -> dict:
    body = dataclasses.asdict(cfg)
    for section, names in _PRIVATE.items():
        sec = body.get(section, {})
        for n in names:
            if n in sec:
                sec[n] = [] if isinstance(sec[n], list) else None
    rec = {"kind": MANIFEST_KIND, "config": body, "issued_at": time.time()}
    return sign_record(identity, rec) if identity is not None else rec


def manifest_fingerprint(manifest: dict) -> str:
    """16 hex chars over the config body only (re-signing does not change it)."""
    return hashlib.sha256(json.dumps(manifest.get("config", {}), sort_keys=True).encode()).hexdigest()[:16]


def verify_manifest(manifest, *, server_pub: str | None = None) -> bool:
    """A manifest; signed by ``server_pub`` when pinned; a present signature must be valid."""
    if not (isinstance(manifest, dict) and manifest.get("kind") == MANIFEST_KIND
            and isinstance(manifest.get("config"), dict)):
        return False
    signed = "sig" in manifest
    if server_pub is not None:
        return signed and verify_record(manifest) and str(manifest.get("pub", "")).lower() == server_pub.lower()
    return verify_record(manifest) if signed else True


def manifest_to_config(manifest: dict, *, overrides: dict | None = None) -> LaunchConfig:
    """The manifest's config with ``overrides`` (``{section: {key: value}}``, ``None``
    values ignored) laid over it, validated like a loaded file."""
    body = copy.deepcopy(manifest["config"])
    for section, vals in (overrides or {}).items():
        body.setdefault(section, {}).update({k: v for k, v in vals.items() if v is not None})
    return LaunchConfig.from_dict(body)
