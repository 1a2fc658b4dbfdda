"""Sampling parameters, per-token seeds and the CPU sampling oracle.

Semantics follow ``src/sampling.rs:9-102`` (temperature scaling, top-k threshold with ties
kept, top-p nucleus as the smallest descending prefix whose mass reaches p, seeded draw)
and ``src/model_fuel/engine_model.rs:25-52`` (temperature <= 0 is greedy argmax, first max
wins; the seed of a token is derived from (request id, token index) so one request's samples
never depend on other traffic).  ``sample_row_reference`` restates the GPU kernel's exact
rule (fixed-point masses, SplitMix64 draw) for tests.
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

MASK64 = (1 << 64) - 1


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_k: int = 0          # 0 = disabled
    top_p: float = 1.0      # 1.0 = disabled
    max_tokens: int = 100   # reference default (src/api/openai/chat.rs:467)
    stop: List[str] = field(default_factory=list)
    stop_token_ids: List[int] = field(default_factory=list)
    ignore_eos: bool = False
    seed: Optional[int] = None
    logprobs: bool = False
    detokenize: bool = True  # False: token-id clients, no incremental text

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0


def splitmix64(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def token_seed(request_id: str, token_index: int, base_seed: Optional[int] = None) -> int:
    """Seed of one sampled token: a hash of (request id, token index[, user seed])."""
    h = hashlib.blake2b(f"{request_id}\x00{token_index}\x00{base_seed}".encode(),
                        digest_size=8).digest()
    return int.from_bytes(h, "little") & ((1 << 63) - 1)


def _f2key(x: np.ndarray) -> np.ndarray:
    b = x.astype(np.float32).view(np.uint32)
    return np.where(b & 0x80000000, ~b, b | 0x80000000).astype(np.uint32)


def sample_row_reference(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                         seed: int) -> int:
    """CPU restatement of the sampling kernel (same thresholds, same draw)."""
    x = logits.detach().float().cpu().numpy().astype(np.float32)
    if not temperature > 0.0:
        return int(np.argmax(x))  # numpy argmax returns the first maximum
    v = (x * np.float32(1.0 / temperature)).astype(np.float32)
    smx = np.float32(x.max() * np.float32(1.0 / temperature))
    keys = _f2key(v)
    thr = np.uint32(0)
    n = v.shape[0]
    if 0 < top_k < n:
        thr = np.sort(keys)[::-1][top_k - 1]
    mass = np.floor(np.exp((v - smx).astype(np.float64)) * 4294967296.0).astype(np.uint64)
    kept = keys >= thr
    total = int(mass[kept].sum())
    if 0.0 < top_p < 1.0:
        target = int(float(top_p) * float(total))
        order = np.argsort(-keys.astype(np.int64), kind="stable")
        order = order[kept[order]]
        ks = keys[order]
        # group equal keys, accumulate until target reached
        acc = 0
        i = 0
        while i < len(order):
            j = i
            while j < len(order) and ks[j] == ks[i]:
                j += 1
            grp = int(mass[order[i:j]].sum())
            if acc + grp >= target:
                if ks[i] > thr:
                    thr = ks[i]
                break
            acc += grp
            i = j
        kept = keys >= thr
        total = int(mass[kept].sum())
    r = splitmix64(int(seed) & MASK64)
    u = (r >> 11) * (1.0 / 9007199254740992.0)
    target = int(u * float(total))
    acc = 0
    for i in np.nonzero(kept)[0]:
        acc += int(mass[i])
        if acc > target:
            return int(i)
    return int(np.argmax(x))


def apply_penalties_reference(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    if temperature <= 0 or abs(temperature - 1.0) < 1e-7:
        return logits
    return logits / temperature
