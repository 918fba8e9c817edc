"""Ed25519 peer identities and self-certifying records.

A peer is known by ``peer_id = hex(sha256(raw 32-byte public key))``. It proves
possession of its key by signing a server's challenge nonce, and it publishes
directory records (tracker entries, epoch records) that anyone can check without a
certificate authority: the record carries the public key, and the peer id must hash
from it.

Byte contracts shared with the reference (``src/opendipaco/schedule/identity.py``), so
identities, signatures and records cross between the two frameworks unchanged:

* challenge signature over ``b"opendipaco-peer-auth:" + nonce``;
* record signature over ``b"opendipaco-peer-record:" + json.dumps(record without "pub"
  and "sig", sort_keys=True, separators=(",", ":"))``;
* identity files are PEM PKCS#8 Ed25519 private keys (created with mode 0600).
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

AUTH_CONTEXT = b"opendipaco-peer-auth:"
RECORD_CONTEXT = b"opendipaco-peer-record:"
_UNSIGNED = ("pub", "sig")  # record fields outside the signed body


def _crypto():
    """(ed25519 module, serialization module), imported on first use."""
    try:
        from cryptography.hazmat.primitives import serialization
        from cryptography.hazmat.primitives.asymmetric import ed25519
    except ImportError as exc:  # pragma: no cover - the package is an optional extra
        raise RuntimeError("peer identity needs the 'cryptography' package") from exc
    return ed25519, serialization


def peer_id_of(public_key_hex: str) -> str:
    return hashlib.sha256(bytes.fromhex(public_key_hex)).hexdigest()


def _signature_ok(public_key_hex: str, signature_hex: str, message: bytes) -> bool:
    """True when ``signature_hex`` is a valid Ed25519 signature of ``message`` by the key;
    any malformed input is simply a failed check."""
    ed25519, _ = _crypto()
    try:
        key = ed25519.Ed25519PublicKey.from_public_bytes(bytes.fromhex(public_key_hex))
        key.verify(bytes.fromhex(signature_hex), message)
    except Exception:
        return False
    return True


def verify_signature(public_key_hex, signature_hex, message: bytes) -> bool:
    """Ed25519 check of a signature over ``message`` exactly (callers add their own
    domain-separation prefix); malformed inputs fail."""
    if not isinstance(public_key_hex, str) or not isinstance(signature_hex, str):
        return False
    return _signature_ok(public_key_hex, signature_hex, message)


class PeerIdentity:
    """An Ed25519 key pair with its derived ``peer_id``."""

    __slots__ = ("_private", "public_key_hex", "peer_id")

    def __init__(self, private_key):
        self._private = private_key
        self.public_key_hex = private_key.public_key().public_bytes_raw().hex()
        self.peer_id = peer_id_of(self.public_key_hex)

    def __repr__(self) -> str:
        return f"PeerIdentity(peer_id={self.peer_id[:16]}...)"

    # -- creation / storage
    @classmethod
    def generate(cls) -> "PeerIdentity":
        ed25519, _ = _crypto()
        return cls(ed25519.Ed25519PrivateKey.generate())

    @classmethod
    def load(cls, path) -> "PeerIdentity":
        ed25519, serialization = _crypto()
        key = serialization.load_pem_private_key(Path(path).read_bytes(), password=None)
        if not isinstance(key, ed25519.Ed25519PrivateKey):
            raise ValueError(f"{path} is not an Ed25519 private key")
        return cls(key)

    def save(self, path) -> str:
        """Write the private key as PEM PKCS#8, readable by the owner only."""
        _, serialization = _crypto()
        pem = self._private.private_bytes(serialization.Encoding.PEM, serialization.PrivateFormat.PKCS8,
                                          serialization.NoEncryption())
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        fd = os.open(target, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
        try:
            os.fchmod(fd, 0o600)  # an existing file keeps its old mode otherwise
            os.write(fd, pem)
        finally:
            os.close(fd)
        return str(target)

    # -- signing
    def sign(self, data: bytes) -> bytes:
        return self._private.sign(data)

    def auth_response(self, nonce: bytes) -> dict:
        """Answer to a server challenge (the fields of the ``auth`` message)."""
        return {"pub": self.public_key_hex, "sig": self.sign(AUTH_CONTEXT + nonce).hex()}

    def private_bytes_raw(self) -> bytes:
        return self._private.private_bytes_raw()


def verify_auth(pub: str, sig_hex: str, nonce: bytes) -> bool:
    """Server side of the identity challenge."""
    if not isinstance(pub, str) or not isinstance(sig_hex, str):
        return False
    return _signature_ok(pub, sig_hex, AUTH_CONTEXT + nonce)


def _record_message(record: dict) -> bytes:
    body = {k: v for k, v in record.items() if k not in _UNSIGNED}
    return RECORD_CONTEXT + json.dumps(body, sort_keys=True, separators=(",", ":")).encode()


def sign_record(identity: PeerIdentity, record: dict) -> dict:
    """A copy of ``record`` stamped with the signer's ``peer_id``, public key and signature."""
    stamped = {**record, "peer_id": identity.peer_id, "pub": identity.public_key_hex}
    stamped["sig"] = identity.sign(_record_message(stamped)).hex()
    return stamped


def verify_record(record) -> bool:
    """True for a record whose signature checks out and whose ``peer_id`` hashes from its key."""
    if not isinstance(record, dict):
        return False
    pub, sig = record.get("pub"), record.get("sig")
    if not (isinstance(pub, str) and isinstance(sig, str)):
        return False
    try:
        if record.get("peer_id") != peer_id_of(pub):
            return False
    except ValueError:  # pub is not hex
        return False
    return _signature_ok(pub, sig, _record_message(record))
