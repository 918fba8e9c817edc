"""Ed25519 peer identities and self-certifying signed records
(reference ``src/opendipaco/schedule/identity.py``).

``peer_id = sha256(raw public key)``. Challenges are signed over
``b"opendipaco-peer-auth:" + nonce`` and records over
``b"opendipaco-peer-record:" + canonical JSON`` (sorted keys, compact separators,
every field except ``pub``/``sig``). Those byte strings are the wire contract with
other peers, so they are kept exactly.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

AUTH_CONTEXT = b"opendipaco-peer-auth:"
RECORD_CONTEXT = b"opendipaco-peer-record:"


def _ed25519():
    try:
        from cryptography.hazmat.primitives.asymmetric import ed25519
    except ImportError as exc:  # pragma: no cover
        raise RuntimeError("peer identity needs the 'cryptography' package") from exc
    return ed25519


def peer_id_of(public_key_hex: str) -> str:
    return hashlib.sha256(bytes.fromhex(public_key_hex)).hexdigest()


class PeerIdentity:
    def __init__(self, private_key):
        self._key = private_key
        self.public_key_hex = private_key.public_key().public_bytes_raw().hex()
        self.peer_id = peer_id_of(self.public_key_hex)

    @classmethod
    def generate(cls) -> "PeerIdentity":
        return cls(_ed25519().Ed25519PrivateKey.generate())

    @classmethod
    def load(cls, path) -> "PeerIdentity":
        from cryptography.hazmat.primitives import serialization

        key = serialization.load_pem_private_key(Path(path).read_bytes(), password=None)
        if not isinstance(key, _ed25519().Ed25519PrivateKey):
            raise ValueError(f"{path} is not an Ed25519 private key")
        return cls(key)

    def save(self, path) -> str:
        from cryptography.hazmat.primitives import serialization

        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        pem = self._key.private_bytes(serialization.Encoding.PEM, serialization.PrivateFormat.PKCS8,
                                      serialization.NoEncryption())
        fd = os.open(path, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
        with os.fdopen(fd, "wb") as f:
            os.fchmod(f.fileno(), 0o600)
            f.write(pem)
        return str(path)

    def auth_response(self, nonce: bytes) -> dict:
        return {"pub": self.public_key_hex, "sig": self._key.sign(AUTH_CONTEXT + nonce).hex()}

    def private_bytes_raw(self) -> bytes:
        return self._key.private_bytes_raw()

    def sign(self, data: bytes) -> bytes:
        return self._key.sign(data)


def _verify(pub_hex: str, sig: bytes, data: bytes) -> bool:
    try:
        _ed25519().Ed25519PublicKey.from_public_bytes(bytes.fromhex(pub_hex)).verify(sig, data)
        return True
    except Exception:
        return False


def verify_auth(pub: str, sig_hex: str, nonce: bytes) -> bool:
    try:
        return _verify(pub, bytes.fromhex(sig_hex), AUTH_CONTEXT + nonce)
    except (ValueError, TypeError):
        return False


def _canonical(record: dict) -> bytes:
    body = {k: v for k, v in record.items() if k not in ("pub", "sig")}
    return RECORD_CONTEXT + json.dumps(body, sort_keys=True, separators=(",", ":")).encode()


def sign_record(identity: PeerIdentity, record: dict) -> dict:
    out = dict(record, peer_id=identity.peer_id, pub=identity.public_key_hex)
    out["sig"] = identity.sign(_canonical(out)).hex()
    return out


def verify_record(record) -> bool:
    if not isinstance(record, dict):
        return False
    pub, sig = record.get("pub"), record.get("sig")
    if not isinstance(pub, str) or not isinstance(sig, str):
        return False
    try:
        return record.get("peer_id") == peer_id_of(pub) and _verify(pub, bytes.fromhex(sig), _canonical(record))
    except (ValueError, TypeError):
        return False
