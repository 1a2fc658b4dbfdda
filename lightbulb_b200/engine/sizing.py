"""Hardware profile, memory estimates, batch sizing and model recommendation.

Reference: ``src/hardware/mod.rs:27-280`` (``HardwareProfile::detect``),
``src/hardware/batch_sizing.rs:28-310`` (initial batch size from memory, and
``RuntimeBatchAdjuster``: shrink x3/4 above 80 % memory use, grow x5/4 below 50 % while the queue
is longer than the batch), ``src/hardware/model_selection.rs`` (largest model that fits),
``src/init.rs:32-320`` (``SystemConfig::auto_detect``) and the memory estimators in
``src/memory/*.rs`` (weights / KV / activations, speculative pair).

The estimates here are exact for this engine's layouts: packed bf16 or quantized weights
(``models/weights.py``), a paged KV pool of ``[layers, 2, blocks, Hkv, 16, head_dim_padded]``
bf16 and the per-step activation workspace of the largest batched-token budget.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

from ..config import ModelConfig, get_preset


# ---------------------------------------------------------------------------------------
# memory estimates
# ---------------------------------------------------------------------------------------
def weight_bytes(cfg: ModelConfig, dtype_bytes: float = 2.0, quant_bits: int = 0,
                 group: int = 128, tp: int = 1) -> int:
    """Per-GPU bytes of the packed weights (embeddings and norms stay bf16)."""
    h, f, L = cfg.hidden_size, cfg.intermediate_size, cfg.num_layers
    dp = cfg.head_dim_padded
    q_rows = cfg.num_heads * dp // tp
    kv_rows = max(1, cfg.num_kv_heads // tp) * dp
    lin = [((q_rows + 2 * kv_rows), h), (h, cfg.num_heads * dp // tp), (2 * f // tp, h),
           (h, f // tp)]
    per_layer = 0.0
    for n, k in lin:
        if quant_bits:
            per_layer += n * k * quant_bits / 8 + 2 * 2 * n * (k // group)
        else:
            per_layer += n * k * dtype_bytes
    per_layer += 2 * h * 2  # two norms
    emb = cfg.vocab_size * h * 2
    head = 0 if cfg.tie_word_embeddings else (cfg.vocab_size + tp - 1) // tp * h * 2
    return int(L * per_layer + emb + head + h * 2)


def kv_bytes_per_token(cfg: ModelConfig, tp: int = 1, dtype_bytes: int = 2) -> int:
    return cfg.num_layers * 2 * max(1, cfg.num_kv_heads // tp) * cfg.head_dim_padded * dtype_bytes


def activation_bytes(cfg: ModelConfig, max_batched_tokens: int, tp: int = 1) -> int:
    """Peak per-step activations: residual + QKV + attention out + gate/up + logits rows."""
    h = cfg.hidden_size
    dp = cfg.head_dim_padded
    qkv = (cfg.num_heads + 2 * cfg.num_kv_heads) * dp // tp
    t = max_batched_tokens
    bf = 2
    return int(t * (3 * h + qkv + cfg.num_heads * dp // tp + 2 * cfg.intermediate_size // tp) * bf
               + min(t, 1024) * (cfg.vocab_size // tp) * 4)


@dataclass
class MemoryPlan:
    weights: int
    activations: int
    kv_per_token: int
    kv_budget: int
    num_blocks: int
    max_tokens: int
    max_seqs_at_len: int
    fits: bool


def plan_memory(cfg: ModelConfig, free_bytes: int, block_size: int = 16,
                max_batched_tokens: int = 8192, max_model_len: int = 4096, tp: int = 1,
                quant_bits: int = 0, utilization: float = 0.92,
                reserve_bytes: int = 2 << 30) -> MemoryPlan:
    w = weight_bytes(cfg, quant_bits=quant_bits, tp=tp)
    act = activation_bytes(cfg, max_batched_tokens, tp)
    per_tok = kv_bytes_per_token(cfg, tp)
    budget = int(free_bytes * utilization) - w - act - reserve_bytes
    blocks = max(0, budget // (per_tok * block_size))
    tokens = blocks * block_size
    return MemoryPlan(w, act, per_tok, max(0, budget), int(blocks), int(tokens),
                      int(tokens // max(1, max_model_len)), blocks > 0)


def speculative_bytes(target: ModelConfig, draft: ModelConfig, batch: int, seq_len: int,
                      k: int = 4, tp: int = 1) -> int:
    """Target + draft weights and both KV pools for ``batch`` sequences of ``seq_len`` + k."""
    toks = batch * (seq_len + k + 1)
    return (weight_bytes(target, tp=tp) + weight_bytes(draft, tp=tp) +
            toks * (kv_bytes_per_token(target, tp) + kv_bytes_per_token(draft, tp)))


# ---------------------------------------------------------------------------------------
# hardware profile
# ---------------------------------------------------------------------------------------
@dataclass
class HardwareProfile:
    cpu_cores: int
    ram_bytes: int
    gpus: List[Tuple[str, int, int]] = field(default_factory=list)  # (name, total, free)
    nvswitch: bool = False

    @property
    def gpu_free_min(self) -> int:
        return min((g[2] for g in self.gpus), default=0)

    @classmethod
    def detect(cls, topology=None) -> "HardwareProfile":
        try:
            import psutil
            ram = int(psutil.virtual_memory().total)
        except Exception:
            ram = 0
        cores = os.cpu_count() or 1
        gpus = []
        nvs = False
        if topology is None:
            try:
                from ..parallel.topology import discover
                topology = discover()
            except Exception:
                topology = None
        if topology is not None:
            gpus = [(g.name, g.total_bytes, g.free_bytes) for g in topology.gpus]
            nvs = topology.nvswitch
        return cls(cores, ram, gpus, nvs)


def initial_batch_size(profile: HardwareProfile, cfg: ModelConfig, seq_len: int,
                       min_batch: int = 1, max_batch: int = 512, tp: int = 1,
                       quant_bits: int = 0) -> int:
    """Largest batch whose KV for ``seq_len`` tokens per sequence fits next to the weights."""
    if not profile.gpus:
        return min_batch
    plan = plan_memory(cfg, profile.gpu_free_min, max_model_len=seq_len, tp=tp,
                       quant_bits=quant_bits)
    return max(min_batch, min(max_batch, plan.max_seqs_at_len))


def recommend_model(profile: HardwareProfile, candidates=("llama3-70b", "llama3-8b", "phi3-mini",
                                                          "llama3.2-1b", "tinyllama"),
                    seq_len: int = 4096, min_batch: int = 8, tp: int = 1) -> Optional[str]:
    """First (largest) preset that serves ``min_batch`` sequences of ``seq_len`` tokens."""
    for name in candidates:
        cfg = get_preset(name)
        plan = plan_memory(cfg, profile.gpu_free_min * tp, max_model_len=seq_len, tp=tp)
        if plan.fits and plan.max_seqs_at_len >= min_batch:
            return name
    return None


# ---------------------------------------------------------------------------------------
# runtime batch adjuster
# ---------------------------------------------------------------------------------------
@dataclass
class BatchSizeConfig:
    min_batch_size: int = 1
    max_batch_size: int = 512
    shrink_above: float = 0.8
    grow_below: float = 0.5
    cooldown_s: float = 0.0


class RuntimeBatchAdjuster:
    """Adjusts the scheduler's ``max_num_seqs`` from observed memory pressure: x3/4 above
    ``shrink_above`` utilisation, x5/4 below ``grow_below`` while the queue is longer than the
    batch (the reference's rule), at most once per ``cooldown_s``."""

    def __init__(self, initial: int, config: Optional[BatchSizeConfig] = None,
                 clock=time.monotonic):
        self.current = initial
        self.cfg = config or BatchSizeConfig()
        self.peak_per_request: Optional[int] = None
        self.history: List[Tuple[float, int, str]] = []
        self._clock = clock
        self._last = -1e18

    def record_batch_memory(self, total_used: int, batch: int) -> None:
        if batch > 0:
            per = total_used // batch
            self.peak_per_request = per if self.peak_per_request is None else max(
                self.peak_per_request, per)

    def check(self, used: int, available: int, queue_length: int) -> Optional[int]:
        now = self._clock()
        if now - self._last < self.cfg.cooldown_s:
            return None
        u = used / max(1, available)
        c = self.cfg
        if u > c.shrink_above and self.current > c.min_batch_size:
            new = max(c.min_batch_size, self.current * 3 // 4)
            why = f"reduced: memory pressure {100 * u:.1f}%"
        elif u < c.grow_below and queue_length > self.current and self.current < c.max_batch_size:
            new = min(c.max_batch_size, max(self.current + 1, self.current * 5 // 4))
            why = f"increased: utilisation {100 * u:.1f}%, queue {queue_length}"
        else:
            return None
        self.current = new
        self._last = now
        self.history.append((now, new, why))
        return new

    def apply(self, engine, used: int, available: int) -> Optional[int]:
        """Check against the engine's queue and resize its scheduler's admission limit."""
        new = self.check(used, available, len(engine.scheduler.waiting))
        if new is not None:
            engine.scheduler.cfg.max_num_seqs = new
        return new


@dataclass
class SystemConfig:
    """``SystemConfig::auto_detect``: hardware, a model that fits, batch size and KV plan."""
    profile: HardwareProfile
    model: Optional[str]
    batch_size: int
    plan: Optional[MemoryPlan]

    @classmethod
    def auto_detect(cls, seq_len: int = 4096, model: Optional[str] = None,
                    topology=None) -> "SystemConfig":
        prof = HardwareProfile.detect(topology)
        name = model or recommend_model(prof, seq_len=seq_len)
        if name is None or not prof.gpus:
            return cls(prof, name, 1, None)
        cfg = get_preset(name)
        plan = plan_memory(cfg, prof.gpu_free_min, max_model_len=seq_len)
        return cls(prof, name, initial_batch_size(prof, cfg, seq_len), plan)
