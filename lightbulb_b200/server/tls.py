"""TLS for the server (reference ``src/tls.rs``): an existing PEM pair, a cached self-signed
certificate valid 30 days, or ACME.  Returns uvicorn ``ssl_*`` keyword arguments.

ACME follows the reference's behaviour (``src/tls.rs:252-300,387-450``): the configuration
(directory URL, domains, contact e-mail, certificate and cache directories) is accepted, a
cached ``acme_cert.pem`` / ``acme_key.pem`` pair that is still valid is used, the HTTP-01
challenge responses live in :class:`AcmeChallenges` (served at
``/.well-known/acme-challenge/<token>`` by the app), and without a valid cached certificate the
server falls back to a self-signed certificate for the first domain.  Talking to the ACME
directory itself needs network access, which this framework's deployments do not assume."""
from __future__ import annotations

import datetime
import logging
import os
import tempfile
import threading
from dataclasses import dataclass, field
from typing import Dict, List, Optional

log = logging.getLogger("lightbulb_b200.tls")


@dataclass
class AcmeConfig:
    directory_url: str = "https://acme-v02.api.letsencrypt.org/directory"
    domains: List[str] = field(default_factory=list)
    contact_email: str = ""
    cert_dir: str = ""
    cache_dir: str = ""

    @classmethod
    def from_env(cls) -> Optional["AcmeConfig"]:
        """``LIGHTBULB_TLS_ACME_DOMAINS`` (comma-separated) enables ACME; ``..._DIRECTORY``,
        ``..._EMAIL``, ``..._CERT_DIR`` and ``..._CACHE_DIR`` refine it."""
        doms = [d.strip() for d in os.environ.get("LIGHTBULB_TLS_ACME_DOMAINS", "").split(",")
                if d.strip()]
        if not doms:
            return None
        c = cls(domains=doms)
        c.directory_url = os.environ.get("LIGHTBULB_TLS_ACME_DIRECTORY", c.directory_url)
        c.contact_email = os.environ.get("LIGHTBULB_TLS_ACME_EMAIL", "")
        base = os.path.join(tempfile.gettempdir(), "lightbulb_tls")
        c.cert_dir = os.environ.get("LIGHTBULB_TLS_ACME_CERT_DIR", os.path.join(base, "acme"))
        c.cache_dir = os.environ.get("LIGHTBULB_TLS_ACME_CACHE_DIR", os.path.join(base, "cache"))
        return c


class AcmeChallenges:
    """HTTP-01 challenge store: token -> key authorisation, shared with the HTTP app."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._m: Dict[str, str] = {}

    def add(self, token: str, key_authorization: str) -> None:
        with self._lock:
            self._m[token] = key_authorization

    def remove(self, token: str) -> None:
        with self._lock:
            self._m.pop(token, None)

    def get(self, token: str) -> Optional[str]:
        with self._lock:
            return self._m.get(token)


CHALLENGES = AcmeChallenges()


def _valid_pair(cert_p: str, key_p: str) -> bool:
    from cryptography import x509
    if not (os.path.exists(cert_p) and os.path.exists(key_p)):
        return False
    try:
        with open(cert_p, "rb") as f:
            c = x509.load_pem_x509_certificate(f.read())
    except ValueError:
        return False
    return c.not_valid_after_utc > datetime.datetime.now(datetime.timezone.utc)


def acme_certificate(cfg: AcmeConfig):
    """(cert, key) paths: the cached ACME pair when still valid, else a self-signed pair for
    the first domain (the reference's fallback)."""
    cert_p = os.path.join(cfg.cert_dir, "acme_cert.pem")
    key_p = os.path.join(cfg.cert_dir, "acme_key.pem")
    if _valid_pair(cert_p, key_p):
        log.info("using the cached ACME certificate for %s", cfg.domains)
        return cert_p, key_p
    log.warning("ACME issuance for %s needs the HTTP-01 exchange with %s; falling back to a "
                "self-signed certificate", cfg.domains, cfg.directory_url)
    return self_signed(os.path.join(cfg.cert_dir, "fallback"),
                       common_name=cfg.domains[0] if cfg.domains else "localhost")


def self_signed(dirpath: str, days: int = 30, common_name: str = "localhost"):
    from cryptography import x509
    from cryptography.hazmat.primitives import hashes, serialization
    from cryptography.hazmat.primitives.asymmetric import ec
    from cryptography.x509.oid import NameOID
    cert_p = os.path.join(dirpath, "cert.pem")
    key_p = os.path.join(dirpath, "key.pem")
    if _valid_pair(cert_p, key_p):
        with open(cert_p, "rb") as f:
            c = x509.load_pem_x509_certificate(f.read())
        if c.subject.get_attributes_for_oid(NameOID.COMMON_NAME)[0].value == common_name:
            return cert_p, key_p
    key = ec.generate_private_key(ec.SECP256R1())
    name = x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, common_name)])
    now = datetime.datetime.now(datetime.timezone.utc)
    cert = (x509.CertificateBuilder().subject_name(name).issuer_name(name)
            .public_key(key.public_key()).serial_number(x509.random_serial_number())
            .not_valid_before(now).not_valid_after(now + datetime.timedelta(days=days))
            .add_extension(x509.SubjectAlternativeName([x509.DNSName(common_name)]), False)
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
    acme = getattr(sc, "tls_acme", None)
    if acme is not None:
        c, k = acme_certificate(acme)
        return {"ssl_certfile": c, "ssl_keyfile": k}
    if sc.tls_self_signed:
        c, k = self_signed(os.path.join(tempfile.gettempdir(), "lightbulb_tls"))
        return {"ssl_certfile": c, "ssl_keyfile": k}
    return {}
