"""Checkpoint manager behind ``/v1/lightbulb/state/*`` (reference
``src/engine/state_persistence.rs:32-500``: JSON checkpoints, max-N eviction, branch, list).

A checkpoint stores a JSON payload (the engine's request table: prompts, generated ids,
sampling params, plus any knowledge-base facts); ``restore`` re-submits the requests so their
KV is rebuilt (prefix-cache hits reuse whatever KV is still resident).

:func:`save_engine_state` / :func:`restore_engine_state` go further than the reference (whose
KV snapshot is metadata only): the KV rows of every cached position are saved with the
requests, and a restore places them in fresh blocks so decoding resumes without recomputing
the prompt or the generated tokens."""
from __future__ import annotations

import json
import os
import tempfile
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

    def kv_path(self, name: str) -> str:
        """File of the KV snapshot that accompanies checkpoint ``name``."""
        return self._path(name)[:-len(".json")] + ".lbkv"

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


# ---------------------------------------------------------------------------------------
# engine state with KV: save and resume without recomputation
# ---------------------------------------------------------------------------------------
def _kv_rows(engine, seq, n: int):
    """[n, layers, 2, Hkv, D] KV rows of the first n cached positions of ``seq``."""
    import torch
    bm, st = engine.blocks, engine.kv.storage
    bs = st.shape[4]
    table = bm.block_table(seq.seq_id)
    pos = torch.arange(n)
    slots = torch.tensor(table, dtype=torch.long)[pos // bs] * bs + pos % bs
    s = slots.to(st.device)
    return st[:, :, s // bs, :, s % bs].to("cpu").contiguous()


def save_engine_state(engine, path: str, request_ids=None, include_kv: bool = True) -> dict:
    """Write the engine's unfinished requests (token lists, sampling parameters, progress) and,
    with ``include_kv``, the KV rows of their cached positions, to one file (LBKV tensor codec,
    CRC-checked).  An overlapped decode step in flight is completed first; its outputs are
    returned in ``["drained"]`` so the caller can still deliver them."""
    import dataclasses
    from ..kv.tiers import encode_tensors
    drained = engine.drain()
    reqs, tensors = [], {}
    for rid, s in engine.seqs.items():
        if s.finished or (request_ids is not None and rid not in request_ids):
            continue
        n = s.num_computed_tokens if (include_kv and not s.evicted and
                                      engine.blocks.has_seq(s.seq_id)) else 0
        if n:
            tensors[f"kv/{rid}"] = _kv_rows(engine, s, n)
        reqs.append({"request_id": rid, "prompt_token_ids": list(s.prompt_token_ids),
                     "output_token_ids": list(s.output_token_ids),
                     "output_text": s.output_text, "params": dataclasses.asdict(s.params),
                     "max_new_tokens": s.max_new_tokens, "priority": s.priority,
                     "num_cached": n})
    st = engine.kv.storage
    meta = {"model": engine.cfg.model.name, "layers": st.shape[0], "kv_heads": st.shape[3],
            "head_dim": st.shape[5], "dtype": str(st.dtype), "requests": reqs}
    blob = encode_tensors(tensors, meta)
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=d)
    with os.fdopen(fd, "wb") as f:
        f.write(blob)
    os.replace(tmp, path)
    return {"path": path, "requests": len(reqs), "kv_tensors": len(tensors),
            "bytes": len(blob), "drained": drained}


def restore_engine_state(engine, path: str) -> List[str]:
    """Re-admit the requests saved by :func:`save_engine_state` into ``engine`` (same model
    shape).  Requests saved with KV get fresh blocks holding those rows and resume decoding
    where they stopped; the others are recomputed from their token lists.  Returns the
    request ids."""
    import torch
    from ..engine.sampling import SamplingParams
    from ..engine.sequence import Sequence, SeqStatus
    from ..engine.tokenizer import IncrementalDetokenizer
    from ..kv.tiers import decode_tensors
    with open(path, "rb") as f:
        tensors, meta = decode_tensors(f.read())
    st = engine.kv.storage
    if (meta["layers"], meta["kv_heads"], meta["head_dim"]) != (st.shape[0], st.shape[3],
                                                                 st.shape[5]):
        raise ValueError(f"snapshot of a different model shape: {meta['layers']} layers, "
                         f"{meta['kv_heads']} KV heads, head dim {meta['head_dim']}")
    engine.drain()
    bm, sch = engine.blocks, engine.scheduler
    bs = st.shape[4]
    out = []
    for r in meta["requests"]:
        rid = r["request_id"]
        if rid in engine.seqs and not engine.seqs[rid].finished:
            raise ValueError(f"request {rid} is already running")
        seq = Sequence(rid, list(r["prompt_token_ids"]), SamplingParams(**r["params"]),
                       output_token_ids=list(r["output_token_ids"]), priority=r["priority"])
        seq.max_new_tokens = r["max_new_tokens"]
        seq.output_text = r["output_text"]
        det = IncrementalDetokenizer(engine.tokenizer)
        for t in seq.output_token_ids:
            det.push(t)
        n = int(r["num_cached"])
        rows = tensors.get(f"kv/{rid}")
        fits = n > 0 and rows is not None and (n + bs - 1) // bs <= bm.num_free_blocks()
        if fits:
            bm.add_sequence(seq.seq_id)
            slots, _ = bm.append_slots(seq.seq_id, n, seq.all_token_ids[:n])
            s = torch.tensor(slots, dtype=torch.long, device=st.device)
            st[:, :, s // bs, :, s % bs] = rows.to(st.device, st.dtype)
            seq.num_computed_tokens = n
            seq.status = SeqStatus.RUNNING
            sch.running.append(seq)
        else:
            sch.add(seq)                         # no KV (or no room): recompute from tokens
        engine.seqs[rid] = seq
        engine.detok[rid] = det
        out.append(rid)
    return out
