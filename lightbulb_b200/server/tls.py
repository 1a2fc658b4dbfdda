"""TLS for the server (reference ``src/tls.rs``: existing PEM, cached self-signed certificate
valid 30 days; ACME is out of scope offline and falls back to self-signed as the reference
does).  Returns uvicorn ``ssl_*`` keyword arguments."""
from __future__ import annotations

import datetime
import os
import tempfile


def self_signed(dirpath: str, days: int = 30):
    from cryptography import x509
    from cryptography.hazmat.primitives import hashes, serialization
    from cryptography.hazmat.primitives.asymmetric import ec
    from cryptography.x509.oid import NameOID
    cert_p = os.path.join(dirpath, "cert.pem")
    key_p = os.path.join(dirpath, "key.pem")
    if os.path.exists(cert_p) and os.path.exists(key_p):
        with open(cert_p, "rb") as f:
            c = x509.load_pem_x509_certificate(f.read())
        if c.not_valid_after_utc > datetime.datetime.now(datetime.timezone.utc):
            return cert_p, key_p
    key = ec.generate_private_key(ec.SECP256R1())
    name = x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, "localhost")])
    now = datetime.datetime.now(datetime.timezone.utc)
    cert = (x509.CertificateBuilder().subject_name(name).issuer_name(name)
            .public_key(key.public_key()).serial_number(x509.random_serial_number())
            .not_valid_before(now).not_valid_after(now + datetime.timedelta(days=days))
            .add_extension(x509.SubjectAlternativeName([x509.DNSName("localhost")]), False)
            .sign(key, hashes.SHA256()))
    os.makedirs(dirpath, exist_ok=True)
    with open(key_p, "wb") as f:
        f.write(key.private_bytes(serialization.Encoding.PEM,
                                  serialization.PrivateFormat.PKCS8,
                                  serialization.NoEncryption()))
    with open(cert_p, "wb") as f:
        f.write(cert.public_bytes(serialization.Encoding.PEM))
    return cert_p, key_p


def ssl_kwargs(sc) -> dict:
    if sc.tls_cert and sc.tls_key:
        return {"ssl_certfile": sc.tls_cert, "ssl_keyfile": sc.tls_key}
    if sc.tls_self_signed:
        c, k = self_signed(os.path.join(tempfile.gettempdir(), "lightbulb_tls"))
        return {"ssl_certfile": c, "ssl_keyfile": k}
    return {}
