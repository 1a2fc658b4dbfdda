"""Checkpoint manager behind ``/v1/lightbulb/state/*`` (reference
``src/engine/state_persistence.rs:32-500``: JSON checkpoints, max-N eviction, branch, list).

A checkpoint stores a JSON payload (the engine's request table: prompts, generated ids,
sampling params, plus any knowledge-base facts); ``restore`` re-submits the requests so their
KV is rebuilt (prefix-cache hits reuse whatever KV is still resident)."""
from __future__ import annotations

import json
import os
import threading
import time
from typing import List, Optional


class CheckpointManager:
    def __init__(self, directory: str, max_checkpoints: int = 16):
        self.dir = directory
        self.max = max_checkpoints
        self._lock = threading.Lock()
        os.makedirs(directory, exist_ok=True)

    def _path(self, name: str) -> str:
        safe = "".join(ch for ch in name if ch.isalnum() or ch in "-_.")
        if not safe:
            raise ValueError("invalid checkpoint name")
        return os.path.join(self.dir, safe + ".json")

    def save(self, name: str, payload: dict, parent: Optional[str] = None) -> dict:
        meta = {"name": name, "created": time.time(), "parent": parent, "payload": payload}
        with self._lock:
            with open(self._path(name), "w") as f:
                json.dump(meta, f)
            self._evict()
        return {k: meta[k] for k in ("name", "created", "parent")}

    def restore(self, name: str) -> dict:
        with open(self._path(name)) as f:
            return json.load(f)

    def branch(self, source: str, new_name: str) -> dict:
        src = self.restore(source)
        return self.save(new_name, src["payload"], parent=source)

    def list(self) -> List[dict]:
        out = []
        for fn in sorted(os.listdir(self.dir)):
            if fn.endswith(".json"):
                try:
                    with open(os.path.join(self.dir, fn)) as f:
                        m = json.load(f)
                    out.append({k: m.get(k) for k in ("name", "created", "parent")})
                except Exception:
                    continue
        return sorted(out, key=lambda m: m["created"] or 0)

    def _evict(self):
        items = self.list()
        for m in items[:max(0, len(items) - self.max)]:
            try:
                os.remove(self._path(m["name"]))
            except OSError:
                pass


def engine_snapshot(engine) -> dict:
    """The request table of an engine as JSON-able data."""
    reqs = []
    for rid, s in engine.seqs.items():
        reqs.append({"request_id": rid, "prompt_token_ids": s.prompt_token_ids,
                     "output_token_ids": list(s.output_token_ids),
                     "finished": s.finished, "finish_reason": s.finish_reason,
                     "params": {"temperature": s.params.temperature, "top_k": s.params.top_k,
                                "top_p": s.params.top_p, "max_tokens": s.params.max_tokens}})
    return {"requests": reqs, "model": engine.cfg.model.name}
