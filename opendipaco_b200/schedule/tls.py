"""Encryption of the control-plane sockets.

The framed wire format and its HMAC handshake authenticate peers but send tensors in
the clear; these helpers build the ``ssl.SSLContext`` objects that the servers
(coordinator, scheduler, parameter servers, tracker) and the workers wrap their sockets
in. Both ends run this code, so the floor is TLS 1.2 everywhere. Public names and
arguments are those of the reference's ``src/opendipaco/schedule/tls.py`` (operators'
launch configs pass them through unchanged); the construction is this module's own.

``generate_selfsigned_cert`` writes a throwaway certificate for tests and single-host
development (an ECDSA P-256 key, the given hosts as subject alternative names).
"""

from __future__ import annotations

import datetime
import ipaddress
import os
import ssl

_FLOOR = ssl.TLSVersion.TLSv1_2


def _new(server: bool) -> ssl.SSLContext:
    ctx = ssl.SSLContext(ssl.PROTOCOL_TLS_SERVER if server else ssl.PROTOCOL_TLS_CLIENT)
    ctx.minimum_version = _FLOOR
    return ctx


def server_context(certfile: str, keyfile: str, *, cafile: str | None = None,
                   require_client_cert: bool = False, password: str | None = None) -> ssl.SSLContext:
    """Context for a listening server holding ``certfile`` / ``keyfile`` (PEM).

    ``cafile`` lets the server verify client certificates; with
    ``require_client_cert=True`` every client must present one (mutual TLS), which is
    meaningless without a CA to check it against.
    """
    if require_client_cert and cafile is None:
        raise ValueError("require_client_cert needs a cafile to verify the worker cert")
    ctx = _new(server=True)
    ctx.load_cert_chain(certfile, keyfile, password=password)
    if cafile is not None:
        ctx.load_verify_locations(cafile=cafile)
    ctx.verify_mode = ssl.CERT_REQUIRED if require_client_cert else ssl.CERT_NONE
    return ctx


def client_context(*, cafile: str | None = None, certfile: str | None = None, keyfile: str | None = None,
                   check_hostname: bool = False, insecure: bool = False) -> ssl.SSLContext:
    """Context for a connecting worker or tool.

    The server is verified against ``cafile`` (or the system store when none is given)
    unless ``insecure`` is set, which keeps the encryption but trusts any server (for a
    self-signed development server). ``check_hostname`` additionally matches the
    server's name against its certificate. ``certfile`` / ``keyfile`` present this
    client's own certificate (mutual TLS).
    """
    ctx = _new(server=False)
    verify = not insecure
    ctx.check_hostname = bool(check_hostname) and verify  # must be off before CERT_NONE
    ctx.verify_mode = ssl.CERT_REQUIRED if verify else ssl.CERT_NONE
    if verify:
        if cafile is not None:
            ctx.load_verify_locations(cafile=cafile)
        else:
            ctx.load_default_certs(ssl.Purpose.SERVER_AUTH)
    if certfile is not None:
        ctx.load_cert_chain(certfile, keyfile)
    return ctx


def _alt_names(hosts) -> list:
    from cryptography import x509

    names = []
    for h in hosts:
        try:
            names.append(x509.IPAddress(ipaddress.ip_address(h)))
        except ValueError:  # not an address literal: a DNS name
            names.append(x509.DNSName(str(h)))
    return names


def generate_selfsigned_cert(dirpath: str, *, common_name: str = "localhost",
                             hosts=("localhost", "127.0.0.1"), days: int = 365) -> tuple[str, str]:
    """Write ``cert.pem`` / ``key.pem`` (self-signed, valid ``days`` days, ``hosts`` as
    subject alternative names) into ``dirpath``; returns their paths. Development and
    tests only; needs the ``cryptography`` package."""
    try:
        from cryptography import x509
        from cryptography.hazmat.primitives import hashes, serialization
        from cryptography.hazmat.primitives.asymmetric import ec
        from cryptography.x509.oid import NameOID
    except ImportError as exc:  # pragma: no cover - the package is an optional extra
        raise RuntimeError("generate_selfsigned_cert needs the 'cryptography' package") from exc

    key = ec.generate_private_key(ec.SECP256R1())
    subject = x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, common_name)])
    start = datetime.datetime.now(datetime.timezone.utc) - datetime.timedelta(minutes=5)
    builder = x509.CertificateBuilder(
        issuer_name=subject, subject_name=subject, public_key=key.public_key(),
        serial_number=x509.random_serial_number(), not_valid_before=start,
        not_valid_after=start + datetime.timedelta(days=days),
        extensions=[],
    ).add_extension(x509.SubjectAlternativeName(_alt_names(hosts)), critical=False)
    cert = builder.sign(key, hashes.SHA256())
    os.makedirs(dirpath, exist_ok=True)
    out = {"cert.pem": cert.public_bytes(serialization.Encoding.PEM),
           "key.pem": key.private_bytes(serialization.Encoding.PEM, serialization.PrivateFormat.PKCS8,
                                        serialization.NoEncryption())}
    paths = []
    for name, data in out.items():
        path = os.path.join(dirpath, name)
        with open(path, "wb") as f:
            f.write(data)
        paths.append(path)
    return paths[0], paths[1]
