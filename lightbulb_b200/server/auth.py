"""Optional API-key auth, fixed-window rate limiting and audit log.

Reference: ``src/api/auth_middleware.rs:33-272`` + ``migrations/V1..V4`` (Postgres): bearer key
-> SHA-256 -> ``api_keys`` lookup, per-minute fixed-window usage counter, ``audit_logs`` insert,
admin role check; everything is a no-op without a database.  Here the database is sqlite
(``DATABASE_URL=sqlite:///path``, stdlib driver); other URLs disable auth with a warning.
"""
from __future__ import annotations

import hashlib
import logging
import secrets
import sqlite3
import threading
import time
from typing import Optional, Tuple

log = logging.getLogger("lightbulb_b200.auth")

SCHEMA = """
CREATE TABLE IF NOT EXISTS api_keys (
  key_hash TEXT PRIMARY KEY, name TEXT, role TEXT DEFAULT 'user',
  rate_limit_per_minute INTEGER DEFAULT 60, created_at REAL, revoked INTEGER DEFAULT 0);
CREATE TABLE IF NOT EXISTS api_key_usage (
  key_hash TEXT, window_start INTEGER, count INTEGER, PRIMARY KEY (key_hash, window_start));
CREATE TABLE IF NOT EXISTS audit_logs (
  ts REAL, key_hash TEXT, method TEXT, path TEXT, status INTEGER, latency_ms REAL);
"""


def hash_key(key: str) -> str:
    return hashlib.sha256(key.encode()).hexdigest()


class AuthStore:
    def __init__(self, database_url: Optional[str]):
        self.conn = None
        self._lock = threading.Lock()
        if not database_url:
            return
        if database_url.startswith("sqlite:///") or database_url == "sqlite://:memory:":
            path = ":memory:" if database_url.endswith(":memory:") else database_url[len("sqlite:///"):]
            self.conn = sqlite3.connect(path, check_same_thread=False)
            self.conn.executescript(SCHEMA)
            self.conn.commit()
        else:
            log.warning("DATABASE_URL %s: only sqlite is supported here; auth disabled",
                        database_url.split(":")[0])

    @property
    def enabled(self) -> bool:
        return self.conn is not None

    def create_key(self, name: str, role: str = "user", rate_limit: int = 60) -> str:
        key = "lb-" + secrets.token_urlsafe(24)
        with self._lock:
            self.conn.execute("INSERT INTO api_keys VALUES (?,?,?,?,?,0)",
                              (hash_key(key), name, role, rate_limit, time.time()))
            self.conn.commit()
        return key

    def lookup(self, key: str) -> Optional[Tuple[str, str, int]]:
        with self._lock:
            r = self.conn.execute("SELECT key_hash, role, rate_limit_per_minute FROM api_keys "
                                  "WHERE key_hash=? AND revoked=0", (hash_key(key),)).fetchone()
        return r

    def hit(self, key_hash: str, limit: int) -> bool:
        """Count one request in the current minute window; False if over the limit."""
        w = int(time.time() // 60)
        with self._lock:
            self.conn.execute("INSERT INTO api_key_usage VALUES (?,?,1) ON CONFLICT(key_hash, "
                              "window_start) DO UPDATE SET count=count+1", (key_hash, w))
            c = self.conn.execute("SELECT count FROM api_key_usage WHERE key_hash=? AND "
                                  "window_start=?", (key_hash, w)).fetchone()[0]
            self.conn.commit()
        return c <= limit

    def audit(self, key_hash: Optional[str], method: str, path: str, status: int, ms: float):
        with self._lock:
            self.conn.execute("INSERT INTO audit_logs VALUES (?,?,?,?,?,?)",
                              (time.time(), key_hash, method, path, status, ms))
            self.conn.commit()
