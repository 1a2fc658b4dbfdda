"""Tracing: NVTX ranges for profiler timelines and per-category debug logging.

Reference: ``src/debug.rs:16-84`` -- feature-gated ``debug_prefill!`` ... ``debug_engine!``
eprintln macros (``Cargo.toml:65-75``).  Here the categories are runtime switches:

* ``LB_DEBUG=prefill,decode,engine,scheduler,kv,spec,tp`` (or ``all``) turns on DEBUG logging for
  ``lightbulb_b200.<category>`` loggers; :func:`debug` is a no-op for disabled categories.
* ``LB_NVTX=1`` wraps engine steps, scheduling, runner execution and sampling in NVTX ranges
  (``torch.cuda.nvtx``) so a timeline profiler shows them; off, :func:`nvtx_range` costs one
  boolean check.
"""
from __future__ import annotations

import contextlib
import logging
import os
from typing import Iterator

CATEGORIES = ("prefill", "decode", "engine", "scheduler", "kv", "spec", "tp", "server")

_enabled = set()
_nvtx = False


def configure(debug: str = None, nvtx: bool = None) -> None:
    global _enabled, _nvtx
    debug = os.environ.get("LB_DEBUG", "") if debug is None else debug
    cats = {c.strip() for c in debug.split(",") if c.strip()}
    if "all" in cats:
        cats = set(CATEGORIES)
    _enabled = cats
    for c in CATEGORIES:
        lg = logging.getLogger(f"lightbulb_b200.{c}")
        if c in cats:
            lg.setLevel(logging.DEBUG)
            if not lg.handlers and not logging.getLogger().handlers:
                h = logging.StreamHandler()
                h.setFormatter(logging.Formatter("[%(name)s] %(message)s"))
                lg.addHandler(h)
    _nvtx = (os.environ.get("LB_NVTX", "0") not in ("", "0")) if nvtx is None else bool(nvtx)


def enabled(category: str) -> bool:
    return category in _enabled


def debug(category: str, msg: str, *args) -> None:
    if category in _enabled:
        logging.getLogger(f"lightbulb_b200.{category}").debug(msg, *args)


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if not _nvtx:
        yield
        return
    import torch
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


configure()
