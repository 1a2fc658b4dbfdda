"""Tiered KV storage: demote a sequence's tokens from device KV to host RAM and on to disk,
promote them back on request.

Reference: ``src/cache/tiered_storage.rs:32-545`` (VRAM -> RAM -> disk demotion of KV spans with
a knowledge-base summary, promotion on ``<RETRIEVE:key>``), ``src/cache/tensor_codec.rs:24-290``
(tensor serialisation for the disk tier) and ``BlockTierMover`` in
``src/model_fuel/policies.rs:1244-1490`` (demote / promote paged blocks to a ``DiskStore``, with
rollback on failure).

Here a demoted entry holds the K/V rows of the chosen token positions for every layer (one
gather from the paged pool, ``[tokens, layers, 2, Hkv, D]``), their positions and token ids.  Promotion allocates fresh blocks, writes the rows back (keys keep their rotary positions,
since keys are stored after RoPE) and appends them to the sequence's block table; the sequence's
``evicted`` count drops accordingly.  Any failure during promotion returns the blocks and leaves
the sequence unchanged.
"""
from __future__ import annotations

import collections
import hashlib
import json
import os
import re
import struct
import tempfile
import zlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

_MAGIC = b"LBKV"
_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.int32: 3,
           torch.int64: 4, torch.uint8: 5, torch.int8: 6}
_RDTYPES = {v: k for k, v in _DTYPES.items()}


# ---------------------------------------------------------------------------------------
# tensor codec
# ---------------------------------------------------------------------------------------
def encode_tensors(tensors: Dict[str, torch.Tensor], meta: Optional[dict] = None) -> bytes:
    """``LBKV`` | u32 header length | JSON header (names, dtypes, shapes, offsets, meta) |
    raw little-endian payloads | u32 CRC-32 of everything before it."""
    entries, blobs, off = [], [], 0
    for name, t in tensors.items():
        t = t.detach().to("cpu").contiguous()
        raw = t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.uint8 else \
            t.numpy().tobytes()
        entries.append({"name": name, "dtype": _DTYPES[t.dtype], "shape": list(t.shape),
                        "offset": off, "nbytes": len(raw)})
        blobs.append(raw)
        off += len(raw)
    hdr = json.dumps({"tensors": entries, "meta": meta or {}}).encode()
    body = _MAGIC + struct.pack("<I", len(hdr)) + hdr + b"".join(blobs)
    return body + struct.pack("<I", zlib.crc32(body) & 0xFFFFFFFF)


def decode_tensors(buf: bytes):
    if len(buf) < 12 or buf[:4] != _MAGIC:
        raise ValueError("not an LBKV blob")
    body, crc = buf[:-4], struct.unpack("<I", buf[-4:])[0]
    if zlib.crc32(body) & 0xFFFFFFFF != crc:
        raise ValueError("LBKV checksum mismatch")
    n = struct.unpack("<I", body[4:8])[0]
    hdr = json.loads(body[8:8 + n])
    base = 8 + n
    out = {}
    for e in hdr["tensors"]:
        raw = bytearray(body[base + e["offset"]: base + e["offset"] + e["nbytes"]])
        u8 = torch.frombuffer(raw, dtype=torch.uint8) if raw else torch.empty(0, dtype=torch.uint8)
        dt = _RDTYPES[e["dtype"]]
        out[e["name"]] = (u8 if dt == torch.uint8 else u8.view(dt)).reshape(e["shape"]).clone()
    return out, hdr.get("meta", {})


# ---------------------------------------------------------------------------------------
# stores
# ---------------------------------------------------------------------------------------
class DiskStore:
    def put(self, key: str, data: bytes) -> None:
        raise NotImplementedError

    def get(self, key: str) -> Optional[bytes]:
        raise NotImplementedError

    def delete(self, key: str) -> None:
        raise NotImplementedError

    def keys(self) -> List[str]:
        raise NotImplementedError


class FileDiskStore(DiskStore):
    """One file per key (hashed file name), written atomically (temp file + rename)."""

    def __init__(self, root: str):
        self.root = root
        os.makedirs(root, exist_ok=True)
        self._index_path = os.path.join(root, "index.json")
        self._index: Dict[str, str] = {}
        if os.path.exists(self._index_path):
            with open(self._index_path) as f:
                self._index = json.load(f)

    def _path(self, key: str) -> str:
        return os.path.join(self.root, hashlib.sha256(key.encode()).hexdigest()[:32] + ".lbkv")

    def _save_index(self) -> None:
        fd, tmp = tempfile.mkstemp(dir=self.root)
        with os.fdopen(fd, "w") as f:
            json.dump(self._index, f)
        os.replace(tmp, self._index_path)

    def put(self, key: str, data: bytes) -> None:
        p = self._path(key)
        fd, tmp = tempfile.mkstemp(dir=self.root)
        with os.fdopen(fd, "wb") as f:
            f.write(data)
        os.replace(tmp, p)
        self._index[key] = os.path.basename(p)
        self._save_index()

    def get(self, key: str) -> Optional[bytes]:
        if key not in self._index:
            return None
        with open(os.path.join(self.root, self._index[key]), "rb") as f:
            return f.read()

    def delete(self, key: str) -> None:
        name = self._index.pop(key, None)
        if name:
            try:
                os.remove(os.path.join(self.root, name))
            except FileNotFoundError:
                pass
            self._save_index()

    def keys(self) -> List[str]:
        return list(self._index)


class MemoryDiskStore(DiskStore):
    def __init__(self):
        self.d: Dict[str, bytes] = {}

    def put(self, key, data):
        self.d[key] = bytes(data)

    def get(self, key):
        return self.d.get(key)

    def delete(self, key):
        self.d.pop(key, None)

    def keys(self):
        return list(self.d)


# ---------------------------------------------------------------------------------------
# mover
# ---------------------------------------------------------------------------------------
@dataclass
class TierEntry:
    key: str
    seq_id: int
    positions: List[int]
    token_ids: List[int]
    kv: Optional[torch.Tensor] = None     # [n, layers, 2, Hkv, D] on the host (RAM tier)
    summary: str = ""
    tier: str = "ram"


RETRIEVE_RE = re.compile(r"<RETRIEVE:([^>]+)>")


def find_retrieve_requests(text: str) -> List[str]:
    """Keys of ``<RETRIEVE:key>`` markers in generated text."""
    return RETRIEVE_RE.findall(text)


class BlockTierMover:
    """Demotes token KV of running sequences to RAM (bounded, LRU) and disk, promotes it back."""

    def __init__(self, engine, disk: Optional[DiskStore] = None, max_ram_entries: int = 64,
                 knowledge_base=None, summarize=None):
        self.eng = engine
        self.disk = disk
        self.max_ram = max_ram_entries
        self.kb = knowledge_base
        self.summarize = summarize   # (token_ids) -> str
        self.entries: "collections.OrderedDict[str, TierEntry]" = collections.OrderedDict()
        self.stats = {"demoted": 0, "promoted": 0, "to_disk": 0, "rollbacks": 0}

    # -- helpers ------------------------------------------------------------------------
    def _slots(self, seq, positions: List[int]) -> torch.Tensor:
        bm, bs = self.eng.blocks, self.eng.kv.block_size
        table = bm.block_table(seq.seq_id)
        return torch.tensor([table[p // bs] * bs + p % bs for p in positions], dtype=torch.long)

    def _gather(self, slots: torch.Tensor) -> torch.Tensor:
        st = self.eng.kv.storage                      # [L, 2, NB, Hkv, BS, D]
        bs = st.shape[4]
        s = slots.to(st.device)
        rows = st[:, :, s // bs, :, s % bs]           # [n, L, 2, Hkv, D]
        return rows.to("cpu", non_blocking=False).contiguous()

    def _scatter(self, slots: torch.Tensor, rows: torch.Tensor) -> None:
        st = self.eng.kv.storage
        bs = st.shape[4]
        s = slots.to(st.device)
        st[:, :, s // bs, :, s % bs] = rows.to(st.device, st.dtype)

    def _spill(self) -> None:
        while len([e for e in self.entries.values() if e.tier == "ram"]) > self.max_ram:
            for k, e in self.entries.items():
                if e.tier == "ram":
                    break
            if self.disk is not None:
                self.disk.put(k, encode_tensors({"kv": e.kv}, {
                    "seq_id": e.seq_id, "positions": e.positions, "token_ids": e.token_ids,
                    "summary": e.summary}))
                e.tier, e.kv = "disk", None
                self.stats["to_disk"] += 1
            else:
                del self.entries[k]          # no disk tier: the oldest RAM entry is dropped

    # -- API ----------------------------------------------------------------------------
    def demote(self, seq, positions: List[int], key: Optional[str] = None) -> str:
        """Copy the KV rows of ``positions`` (KV positions of ``seq``) to the RAM tier.  The
        caller removes them from the device (e.g. by compaction)."""
        key = key or f"seq{seq.seq_id}-{positions[0]}-{positions[-1]}"
        rows = self._gather(self._slots(seq, positions))
        toks = seq.all_token_ids
        base = getattr(seq, "evicted", 0)
        ids = [toks[p + base] if 0 <= p + base < len(toks) else -1 for p in positions]
        summary = self.summarize(ids) if self.summarize else ""
        if self.kb is not None and summary:
            self.kb.add(summary, source=f"tier:{key}")
        self.entries[key] = TierEntry(key, seq.seq_id, list(positions), ids, rows, summary)
        self.entries.move_to_end(key)
        self.stats["demoted"] += 1
        self._spill()
        return key

    def load(self, key: str) -> TierEntry:
        e = self.entries.get(key)
        if e is None:
            raise KeyError(key)
        if e.tier == "disk":
            blob = self.disk.get(key) if self.disk is not None else None
            if blob is None:
                raise KeyError(f"{key}: missing from the disk tier")
            t, _ = decode_tensors(blob)
            e.kv, e.tier = t["kv"], "ram"
            self.disk.delete(key)
            self.entries.move_to_end(key)
            self._spill()
        return e

    def promote(self, seq, key: str) -> int:
        """Append the entry's KV to ``seq``'s cache; returns the number of tokens restored."""
        e = self.load(key)
        eng = self.eng
        bm, bs = eng.blocks, eng.kv.block_size
        n = len(e.positions)
        kvlen = seq.num_computed_tokens
        table = list(bm.block_table(seq.seq_id))
        tail_free = (len(table) * bs) - kvlen
        new_blocks = []
        try:
            need = max(0, n - tail_free)
            new_blocks = bm.alloc_blocks((need + bs - 1) // bs) if need else []
            full = table + list(new_blocks)
            slots = torch.tensor([full[(kvlen + i) // bs] * bs + (kvlen + i) % bs
                                  for i in range(n)], dtype=torch.long)
            self._scatter(slots, e.kv)
            bm.set_blocks(seq.seq_id, full, kvlen + n)
        except Exception:
            if new_blocks:
                bm.free_blocks(new_blocks)
            self.stats["rollbacks"] += 1
            raise
        seq.num_computed_tokens = kvlen + n
        seq.evicted = max(0, seq.evicted - n)
        del self.entries[key]
        self.stats["promoted"] += 1
        return n

    def handle_retrieve(self, seq, text: str) -> int:
        """Promote every entry named by ``<RETRIEVE:key>`` markers in ``text``."""
        restored = 0
        for k in find_retrieve_requests(text):
            if k in self.entries:
                restored += self.promote(seq, k)
        return restored
