"""Mixed-precision profiler: per-layer activation statistics, a recommended precision per layer,
and run-time adjustment from observed accuracy.

Reference: ``src/engine/mixed_precision.rs:33-460``.  Recommendation rules follow it: dynamic
range > 1e6 -> fp32; range < 10 with standard deviation < 1 -> int8; range < 1e4 -> bf16; else
fp16.  Layer overrides win; sensitive layers (names containing lm_head / embed / norm) never
go below bf16.  With dynamic adjustment, after ``profiling_window`` batches a layer whose
accuracy falls below the threshold steps up one precision (int8 -> fp16 -> bf16 -> fp32), and
one above 0.99 steps down one every 10 batches.

Differences: statistics are exact running moments (Welford) over tensors rather than the
reference's per-batch spread around the mean magnitude, and :meth:`PrecisionProfiler.plan`
maps the result onto what this engine can deploy (bf16 weights, Q8_0 int8, AWQ int4).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch


class Precision(str, enum.Enum):
    FP32 = "fp32"
    FP16 = "fp16"
    BF16 = "bf16"
    INT8 = "int8"

    @property
    def bits(self) -> int:
        return {"fp32": 32, "fp16": 16, "bf16": 16, "int8": 8}[self.value]

    @property
    def memory_ratio(self) -> float:
        return self.bits / 32.0


_UP = {Precision.INT8: Precision.FP16, Precision.FP16: Precision.BF16,
       Precision.BF16: Precision.FP32, Precision.FP32: Precision.FP32}
_DOWN = {Precision.FP32: Precision.BF16, Precision.BF16: Precision.FP16,
         Precision.FP16: Precision.INT8, Precision.INT8: Precision.INT8}
# deployable weight format of this engine for each precision
DEPLOY_FORMAT = {Precision.FP32: "bf16", Precision.FP16: "bf16", Precision.BF16: "bf16",
                 Precision.INT8: "q8_0"}


@dataclass
class ActivationStats:
    n: int = 0
    mean: float = 0.0
    m2: float = 0.0
    mean_abs: float = 0.0
    min: float = float("inf")
    max: float = float("-inf")

    def update(self, values) -> None:
        x = torch.as_tensor(values).detach().float().reshape(-1)
        if x.numel() == 0:
            return
        k = x.numel()
        bm, bv = float(x.mean()), float(x.var(unbiased=False))
        delta = bm - self.mean
        tot = self.n + k
        self.mean += delta * k / tot
        self.m2 += bv * k + delta * delta * self.n * k / tot
        self.mean_abs += (float(x.abs().mean()) - self.mean_abs) * k / tot
        self.min = min(self.min, float(x.min()))
        self.max = max(self.max, float(x.max()))
        self.n = tot

    @property
    def std(self) -> float:
        return (self.m2 / self.n) ** 0.5 if self.n else 0.0

    @property
    def dynamic_range(self) -> float:
        return self.max - self.min if self.n else 0.0

    def recommend(self) -> Precision:
        r = self.dynamic_range
        if r > 1e6:
            return Precision.FP32
        if r < 10.0 and self.std < 1.0:
            return Precision.INT8
        if r < 1e4:
            return Precision.BF16
        return Precision.FP16


@dataclass
class MixedPrecisionConfig:
    default_precision: Precision = Precision.BF16
    accuracy_threshold: float = 0.95
    dynamic_adjustment: bool = True
    profiling_window: int = 10
    overrides: Dict[str, Precision] = field(default_factory=dict)
    sensitive_patterns: Sequence[str] = ("lm_head", "embed", "norm")

    def is_sensitive(self, name: str) -> bool:
        low = name.lower()
        return any(p in low for p in self.sensitive_patterns)


class PrecisionProfiler:
    def __init__(self, config: Optional[MixedPrecisionConfig] = None):
        self.config = config or MixedPrecisionConfig()
        self.stats: Dict[str, ActivationStats] = {}
        self.chosen: Dict[str, Precision] = {}
        self.accuracy: Dict[str, float] = {}
        self.latency: Dict[str, List[float]] = {}
        self.batches = 0

    def record_activation(self, layer: str, values) -> None:
        self.stats.setdefault(layer, ActivationStats()).update(values)

    def record_latency(self, layer: str, us: float) -> None:
        w = self.latency.setdefault(layer, [])
        w.append(float(us))
        del w[:-self.config.profiling_window]

    def record_accuracy(self, layer: str, acc: float) -> None:
        self.accuracy[layer] = float(acc)

    def end_batch(self) -> None:
        self.batches += 1

    def _floor(self, layer: str, p: Precision) -> Precision:
        if self.config.is_sensitive(layer) and p in (Precision.INT8, Precision.FP16):
            return Precision.BF16
        return p

    def select(self, layer: str) -> Precision:
        c = self.config
        if layer in c.overrides:
            return c.overrides[layer]
        cur = self.chosen.get(layer)
        if cur is None:
            st = self.stats.get(layer)
            cur = self._floor(layer, st.recommend() if st and st.n else c.default_precision)
            self.chosen[layer] = cur
            return cur
        if c.dynamic_adjustment and self.batches > c.profiling_window:
            acc = self.accuracy.get(layer, 1.0)
            if acc < c.accuracy_threshold:
                cur = _UP[cur]
            elif acc > 0.99 and self.batches % 10 == 0:
                cur = self._floor(layer, _DOWN[cur])
            self.chosen[layer] = cur
        return cur

    def avg_latency(self, layer: str) -> Optional[float]:
        w = self.latency.get(layer)
        return sum(w) / len(w) if w else None

    def plan(self, layers: Sequence[str]) -> Dict[str, dict]:
        """Per layer: chosen precision, deployable weight format, memory ratio vs fp32."""
        out = {}
        for name in layers:
            p = self.select(name)
            out[name] = {"precision": p.value, "format": DEPLOY_FORMAT[p],
                         "memory_ratio": p.memory_ratio}
        return out
