"""Segmented KV cache: tagged spans of a sequence's context, scored by the attention they keep
receiving, evicted (or demoted to the tiered store) as whole spans under context pressure.

Reference: ``src/cache/cache_span.rs:55-395`` (``CacheTag``, spans with Active / PartiallyEvicted
states, registry), ``src/cache/segmented_cache_config.rs:42-240`` (defaults: attention power 2.0,
base decay 0.02 per pass, pressure threshold 0.80, pressure EMA alpha 0.3, shadow mode on,
tiered demotion on, at most 64 RAM-demoted segments) and
``src/cache/segmented_eviction_policy.rs:34-530`` (scores: relevance decays by
``base_decay * modifier`` each pass, modifier 1 below the pressure threshold rising linearly to 3
at full context; a span whose tokens received attention gains ``max_attention ** power`` times
a 0.9-per-repeat diminishing factor times its tag weight; system-prompt spans are never ranked;
hybrid per-token tracking inside the lowest span).

The attention statistics come from this engine's H2O score pool (cumulative decayed attention
mass per KV slot, accumulated on the device), so spans are scored without copying attention
probabilities to the host every step (the reference copies them every ``h2o_update_interval``
steps).
"""
from __future__ import annotations

import enum
import itertools
import logging
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Tuple

log = logging.getLogger("lightbulb_b200.spans")


class CacheTag(enum.Enum):
    SYSTEM_PROMPT = "system_prompt"
    USER_INPUT = "user_input"
    TOOL_OUTPUT = "tool_output"
    LONG_TERM_MEMORY = "long_term_memory"
    MODEL_GENERATION = "model_generation"
    CUSTOM = "custom"


# how hard a span of each tag is to evict (reference tag_importance)
TAG_IMPORTANCE = {
    CacheTag.SYSTEM_PROMPT: 1.0,
    CacheTag.TOOL_OUTPUT: 0.8,
    CacheTag.LONG_TERM_MEMORY: 0.75,
    CacheTag.USER_INPUT: 0.7,
    CacheTag.MODEL_GENERATION: 0.5,
    CacheTag.CUSTOM: 0.6,
}


@dataclass
class SegmentedCacheConfig:
    enabled: bool = False
    attention_power: float = 2.0
    base_decay_rate: float = 0.02
    eviction_pressure_threshold: float = 0.80
    pressure_ema_alpha: float = 0.3
    tiered_demotion: bool = True
    per_token_eviction: bool = False
    shadow_mode: bool = True
    log_span_attention: bool = False
    max_ram_demoted_segments: int = 64
    disk_storage_path: Optional[str] = None

    @classmethod
    def observation(cls) -> "SegmentedCacheConfig":
        return cls(enabled=True, shadow_mode=True, log_span_attention=True)

    @classmethod
    def live(cls) -> "SegmentedCacheConfig":
        return cls(enabled=True, shadow_mode=False)


@dataclass
class Span:
    span_id: int
    start: int                      # first position (inclusive)
    end: int                        # last position (exclusive); grows while open
    tag: CacheTag
    name: str = ""
    open: bool = True
    evicted: bool = False
    removed: List[Tuple[int, int]] = field(default_factory=list)  # evicted sub-ranges

    @property
    def active(self) -> bool:
        return not self.evicted

    def remaining_ranges(self) -> List[Tuple[int, int]]:
        if self.evicted:
            return []
        out, cur = [], self.start
        for a, b in sorted(self.removed):
            if a > cur:
                out.append((cur, a))
            cur = max(cur, b)
        if cur < self.end:
            out.append((cur, self.end))
        return out

    def positions(self) -> Iterable[int]:
        for a, b in self.remaining_ranges():
            yield from range(a, b)


class SpanRegistry:
    """Spans of one sequence's context (positions are KV positions of that sequence)."""

    def __init__(self):
        self._spans: Dict[int, Span] = {}
        self._ids = itertools.count(1)

    def begin(self, start: int, tag: CacheTag, name: str = "") -> int:
        sid = next(self._ids)
        self._spans[sid] = Span(sid, start, start, tag, name)
        return sid

    def extend(self, span_id: int, end: int) -> None:
        s = self._spans[span_id]
        s.end = max(s.end, end)

    def end(self, span_id: int, end: int) -> None:
        self.extend(span_id, end)
        self._spans[span_id].open = False

    def tag_range(self, start: int, end: int, tag: CacheTag, name: str = "") -> int:
        sid = self.begin(start, tag, name)
        self.end(sid, end)
        return sid

    def get(self, span_id: int) -> Optional[Span]:
        return self._spans.get(span_id)

    def spans(self) -> List[Span]:
        return sorted(self._spans.values(), key=lambda s: s.start)

    def span_at(self, pos: int) -> Optional[Span]:
        for s in self._spans.values():
            if s.start <= pos < s.end and not s.evicted:
                return s
        return None

    def evict(self, span_id: int) -> List[int]:
        s = self._spans[span_id]
        pos = list(s.positions())
        s.evicted = True
        return pos

    def evict_partial(self, span_id: int, positions: Iterable[int]) -> None:
        s = self._spans[span_id]
        for p in sorted(set(positions)):
            s.removed.append((p, p + 1))
        if not s.remaining_ranges():
            s.evicted = True

    def insert_context_at(self, at: int, length: int) -> None:
        """Positions >= ``at`` move ``length`` later (context inserted at ``at``)."""
        for s in self._spans.values():
            if s.start >= at:
                s.start += length
                s.end += length
                s.removed = [(a + length, b + length) for a, b in s.removed]
            elif s.end > at:
                s.end += length

    def remove(self, span_id: int) -> None:
        self._spans.pop(span_id, None)


@dataclass
class SpanScore:
    relevance: float = 1.0
    hits_this_pass: int = 0
    passes_without_attention: int = 0


class SegmentedEvictionPolicy:
    def __init__(self, config: Optional[SegmentedCacheConfig] = None):
        self.cfg = config or SegmentedCacheConfig(enabled=True)
        self.smoothed_pressure = 0.0
        self.scores: Dict[int, SpanScore] = {}
        self.passes = 0

    def update_pressure(self, utilization: float) -> None:
        a = self.cfg.pressure_ema_alpha
        self.smoothed_pressure = a * utilization + (1 - a) * self.smoothed_pressure

    def pressure_decay_modifier(self) -> float:
        thr = self.cfg.eviction_pressure_threshold
        if self.smoothed_pressure <= thr:
            return 1.0
        return 1.0 + 2.0 * (self.smoothed_pressure - thr) / max(1.0 - thr, 0.01)

    def update_scores(self, registry: SpanRegistry, attention: Callable[[int], float],
                      utilization: float) -> None:
        """One pass: ``attention(pos)`` is the cumulative attention mass at a position."""
        self.passes += 1
        self.update_pressure(utilization)
        decay = self.cfg.base_decay_rate * self.pressure_decay_modifier()
        seen = set()
        for s in registry.spans():
            if not s.active:
                continue
            seen.add(s.span_id)
            sc = self.scores.setdefault(s.span_id, SpanScore())
            sc.hits_this_pass = 0
            sc.relevance = max(0.0, sc.relevance - decay)
            mx = 0.0
            for p in s.positions():
                mx = max(mx, attention(p))
            if mx > 0.0:
                boost = (mx ** self.cfg.attention_power) * (0.9 ** sc.hits_this_pass)
                sc.relevance += boost * TAG_IMPORTANCE[s.tag]
                sc.hits_this_pass += 1
                sc.passes_without_attention = 0
            else:
                sc.passes_without_attention += 1
            if self.cfg.log_span_attention:
                log.info("span %d %s [%d,%d) max_att %.4f relevance %.4f", s.span_id,
                         s.tag.value, s.start, s.end, mx, sc.relevance)
        for k in list(self.scores):
            if k not in seen:
                del self.scores[k]

    def rank_spans_for_eviction(self, registry: SpanRegistry) -> List[Tuple[int, float]]:
        out = []
        for sid, sc in self.scores.items():
            s = registry.get(sid)
            if s is None or not s.active or s.tag == CacheTag.SYSTEM_PROMPT or s.open:
                continue
            out.append((sid, sc.relevance))
        return sorted(out, key=lambda x: (x[1], x[0]))

    def plan(self, registry: SpanRegistry, tokens_to_free: int) -> List[int]:
        """Lowest-relevance closed spans until ``tokens_to_free`` positions are covered."""
        chosen, freed = [], 0
        for sid, _ in self.rank_spans_for_eviction(registry):
            if freed >= tokens_to_free:
                break
            chosen.append(sid)
            freed += sum(1 for _ in registry.get(sid).positions())
        return chosen


class PerTokenTracker:
    """Hybrid eviction inside one span: per-token relevance with the same decay / superlinear
    boost, culling individual low-value tokens of the lowest-scoring span."""

    def __init__(self, span: Span, power: float = 2.0, decay_rate: float = 0.02):
        self.span_id = span.span_id
        self.power, self.decay = power, decay_rate
        self.scores: Dict[int, float] = {p: 1.0 for p in span.positions()}
        self.evicted: set = set()

    def update(self, attention: Callable[[int], float], modifier: float = 1.0) -> None:
        d = self.decay * modifier
        for p in self.scores:
            if p in self.evicted:
                continue
            self.scores[p] = max(0.0, self.scores[p] - d) + attention(p) ** self.power

    def select_evictions(self, max_evictions: int, threshold: float) -> List[int]:
        cand = sorted((s, p) for p, s in self.scores.items()
                      if p not in self.evicted and s < threshold)
        return [p for _, p in cand[:max_evictions]]

    def mark_evicted(self, positions: Iterable[int]) -> None:
        self.evicted.update(positions)


class SegmentedKV:
    """Drives span scoring and eviction for the sequences of an engine.

    ``attention_of(seq, pos)`` reads the H2O score pool (the engine must have H2O enabled for
    attention statistics; without it every span looks unattended and only decay applies).
    In shadow mode the chosen spans are only logged; otherwise their tokens are removed with the
    same compaction path as H2O (``kv_compact``), optionally demoted to a tier store first."""

    def __init__(self, engine, config: Optional[SegmentedCacheConfig] = None, tiers=None):
        self.eng = engine
        self.cfg = config or SegmentedCacheConfig.live()
        self.policy = SegmentedEvictionPolicy(self.cfg)
        self.registries: Dict[int, SpanRegistry] = {}
        self.tiers = tiers
        self.shadow_log: List[Tuple[int, List[int]]] = []
        self.evicted_spans = 0

    def registry(self, seq) -> SpanRegistry:
        return self.registries.setdefault(seq.seq_id, SpanRegistry())

    def attention_of(self, seq, pos: int) -> float:
        h2o = getattr(self.eng.model, "h2o", None)
        if h2o is None:
            return 0.0
        bm, bs = self.eng.blocks, self.eng.kv.block_size
        table = bm.block_table(seq.seq_id)
        if pos // bs >= len(table):
            return 0.0
        return float(h2o.score[table[pos // bs] * bs + pos % bs])

    def step(self, seq, context_limit: int) -> List[int]:
        reg = self.registry(seq)
        used = seq.num_computed_tokens
        self.policy.update_scores(reg, lambda p: self.attention_of(seq, p),
                                  used / max(1, context_limit))
        if self.policy.smoothed_pressure <= self.cfg.eviction_pressure_threshold:
            return []
        target = int(context_limit * self.cfg.eviction_pressure_threshold)
        spans = self.policy.plan(reg, used - target)
        if not spans:
            return []
        if self.cfg.shadow_mode:
            self.shadow_log.append((seq.seq_id, spans))
            log.info("shadow: would evict spans %s of seq %d", spans, seq.seq_id)
            return spans
        self.evict_spans(seq, spans)
        return spans

    def evict_spans(self, seq, span_ids: List[int]) -> None:
        from .. import ops
        import torch
        reg = self.registry(seq)
        drop = set()
        for sid in span_ids:
            if self.tiers is not None and self.cfg.tiered_demotion:
                pos = list(reg.get(sid).positions())
                self.tiers.demote(seq, pos, key=f"seq{seq.seq_id}-span{sid}")
            drop.update(reg.evict(sid))
        eng = self.eng
        bm, bs = eng.blocks, eng.kv.block_size
        kvlen = seq.num_computed_tokens
        keep = [p for p in range(kvlen) if p not in drop]
        table = bm.block_table(seq.seq_id)
        src = torch.tensor([table[p // bs] * bs + p % bs for p in keep], dtype=torch.int32)
        fresh = bm.alloc_blocks((len(keep) + bs - 1) // bs)
        dst = torch.tensor([fresh[i // bs] * bs + i % bs for i in range(len(keep))],
                           dtype=torch.int32)
        st = eng.kv.storage
        if st.is_cuda:
            h2o = getattr(eng.model, "h2o", None)
            ops._need_c().kv_compact(st, src.to(st.device), dst.to(st.device),
                                     h2o.score if h2o is not None else None)
            ops.launch_counter_add(1)
        else:
            sb, so = src.long() // bs, src.long() % bs
            db, do = dst.long() // bs, dst.long() % bs
            st[:, :, db, :, do] = st[:, :, sb, :, so]
        bm.set_blocks(seq.seq_id, fresh, len(keep))
        seq.evicted += kvlen - len(keep)
        seq.num_computed_tokens = len(keep)
        # later spans move left by the number of evicted positions before them
        for s in reg.spans():
            if s.evicted:
                continue
            shift_s = sum(1 for p in drop if p < s.start)
            shift_e = sum(1 for p in drop if p < s.end)
            s.start -= shift_s
            s.end -= shift_e
        self.evicted_spans += len(span_ids)
