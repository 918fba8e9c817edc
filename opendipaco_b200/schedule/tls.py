"""Optional TLS for the transport (reference ``schedule/tls.py``): TLS >= 1.2 contexts
and a self-signed certificate generator for development."""

from __future__ import annotations

import datetime
import ipaddress
import os
import ssl


def server_context(certfile: str, keyfile: str, *, cafile: str | None = None,
                   require_client_cert: bool = False, password: str | None = None) -> ssl.SSLContext:
    ctx = ssl.SSLContext(ssl.PROTOCOL_TLS_SERVER)
    ctx.minimum_version = ssl.TLSVersion.TLSv1_2
    ctx.load_cert_chain(certfile, keyfile, password=password)
    if cafile:
        ctx.load_verify_locations(cafile)
    if require_client_cert:
        if not cafile:
            raise ValueError("require_client_cert needs a cafile to verify the worker cert")
        ctx.verify_mode = ssl.CERT_REQUIRED
    return ctx


def client_context(*, cafile: str | None = None, certfile: str | None = None, keyfile: str | None = None,
                   check_hostname: bool = False, insecure: bool = False) -> ssl.SSLContext:
    ctx = ssl.SSLContext(ssl.PROTOCOL_TLS_CLIENT)
    ctx.minimum_version = ssl.TLSVersion.TLSv1_2
    if insecure:
        ctx.check_hostname = False
        ctx.verify_mode = ssl.CERT_NONE
    else:
        ctx.check_hostname = check_hostname
        ctx.load_verify_locations(cafile) if cafile else ctx.load_default_certs()
    if certfile:
        ctx.load_cert_chain(certfile, keyfile)
    return ctx


def generate_selfsigned_cert(dirpath: str, *, common_name: str = "localhost",
                             hosts=("localhost", "127.0.0.1"), days: int = 365) -> tuple[str, str]:
    from cryptography import x509
    from cryptography.hazmat.primitives import hashes, serialization
    from cryptography.hazmat.primitives.asymmetric import rsa
    from cryptography.x509.oid import NameOID

    key = rsa.generate_private_key(public_exponent=65537, key_size=2048)
    name = x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, common_name)])
    sans = []
    for h in hosts:
        try:
            sans.append(x509.IPAddress(ipaddress.ip_address(h)))
        except ValueError:
            sans.append(x509.DNSName(h))
    now = datetime.datetime.now(datetime.timezone.utc)
    cert = (x509.CertificateBuilder().subject_name(name).issuer_name(name).public_key(key.public_key())
            .serial_number(x509.random_serial_number()).not_valid_before(now - datetime.timedelta(minutes=1))
            .not_valid_after(now + datetime.timedelta(days=days))
            .add_extension(x509.SubjectAlternativeName(sans), critical=False).sign(key, hashes.SHA256()))
    os.makedirs(dirpath, exist_ok=True)
    cf, kf = os.path.join(dirpath, "cert.pem"), os.path.join(dirpath, "key.pem")
    with open(cf, "wb") as f:
        f.write(cert.public_bytes(serialization.Encoding.PEM))
    with open(kf, "wb") as f:
        f.write(key.private_bytes(serialization.Encoding.PEM, serialization.PrivateFormat.TraditionalOpenSSL,
                                  serialization.NoEncryption()))
    return cf, kf
