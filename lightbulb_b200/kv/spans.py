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
import time
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

    def plan(self, registry: SpanRegistry, tokens_to_free: int,
             protected: Iterable[int] = ()) -> List[int]:
        """Lowest-relevance closed spans until ``tokens_to_free`` positions are covered
        (spans in ``protected`` are skipped)."""
        chosen, freed = [], 0
        skip = set(protected)
        for sid, _ in self.rank_spans_for_eviction(registry):
            if freed >= tokens_to_free:
                break
            if sid in skip:
                continue
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

    def step(self, seq, context_limit: int, protected: Iterable[int] = ()) -> List[int]:
        reg = self.registry(seq)
        used = seq.num_computed_tokens
        self.policy.update_scores(reg, lambda p: self.attention_of(seq, p),
                                  used / max(1, context_limit))
        if self.policy.smoothed_pressure <= self.cfg.eviction_pressure_threshold:
            return []
        target = int(context_limit * self.cfg.eviction_pressure_threshold)
        spans = self.policy.plan(reg, used - target, protected)
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


class SegmentedPolicy:
    """Segmented spans and tiered storage driven by the engine's step loop (reference
    ``src/model/parallel_model_manager.rs:626-660`` enable_segmented_cache and ``:689-853``
    eviction-pressure handling with demotion).  Installed as the engine's KV policy:

    * spans are created automatically: the prompt as one ``USER_INPUT`` span once prefilled,
      the generated KV in ``MODEL_GENERATION`` segments of ``segment_tokens``;
    * attention statistics come from the H2O score pool that the model accumulates on the device
      in every decode step (the H2O policy's compaction is not used);
    * after every step, each running sequence's spans are scored and, when the context
      utilisation (KV length / ``context_limit``) stays above the pressure threshold, the
      lowest-scoring spans are evicted (compaction kernel), demoted first to the RAM tier
      (spilling to disk past ``max_ram_demoted_segments``) with a knowledge-base fact whose
      ``[KB:key] summary`` placeholder names the tier key;
    * new tokens of each sequence (generated or injected as context) are scanned for
      ``<RETRIEVE:key>``; a named span is promoted back into the sequence's KV (appended at the
      end, keys keep their rotary positions) and registered as a ``LONG_TERM_MEMORY`` span.
    """

    def __init__(self, engine, config: Optional[SegmentedCacheConfig] = None,
                 context_limit: Optional[int] = None, segment_tokens: int = 64,
                 knowledge_base=None, summarize=None):
        from .compression import H2OPolicy
        from .tiers import BlockTierMover, FileDiskStore, MemoryDiskStore
        self.eng = engine
        self.cfg = config or SegmentedCacheConfig.live()
        self.h2o = H2OPolicy(engine, budget=1 << 30, sinks=0)     # score accumulation only
        disk = (FileDiskStore(self.cfg.disk_storage_path) if self.cfg.disk_storage_path
                else MemoryDiskStore())
        self.kb = knowledge_base
        self.summarize = summarize or self._summary
        self.tiers = BlockTierMover(engine, disk=disk,
                                    max_ram_entries=self.cfg.max_ram_demoted_segments,
                                    knowledge_base=None, summarize=self.summarize)
        self.seg = SegmentedKV(engine, self.cfg, self.tiers)
        self.context_limit = context_limit or engine.cfg.scheduler.max_model_len
        self.segment_tokens = int(segment_tokens)
        self._end: Dict[int, int] = {}        # KV end covered by spans, per sequence
        self._scanned: Dict[int, int] = {}    # tokens already scanned for RETRIEVE markers
        self._tail: Dict[int, str] = {}       # undecoded text tail (a marker split by a step)
        # spans that may not be evicted yet: span id -> steps of grace left.  A promoted span
        # was asked for by the model and has no attention history yet; it gets
        # ``segment_tokens`` decode steps to earn a score before it can be evicted again.
        self._grace: Dict[int, Dict[int, int]] = {}
        self.stats = {"spans": 0, "evicted_spans": 0, "demoted": 0, "promoted": 0}

    def _summary(self, token_ids: List[int]) -> str:
        ids = [t for t in token_ids if t >= 0]
        try:
            text = self.eng.tokenizer.decode(ids)
        except Exception:
            text = ""
        text = " ".join(text.split())
        return (text[:77] + "...") if len(text) > 80 else (text or f"{len(ids)} tokens")

    def before_step(self, so) -> None:
        self.h2o.before_step(so)

    # -- span bookkeeping ---------------------------------------------------------------
    def _register(self, seq) -> None:
        reg = self.seg.registry(seq)
        sid, kvlen = seq.seq_id, seq.num_computed_tokens
        end = self._end.get(sid)
        if end is None:
            if kvlen < seq.prompt_len or kvlen == 0:
                return                                      # prompt not yet in the KV
            reg.tag_range(0, seq.prompt_len, CacheTag.USER_INPUT, "prompt")
            self.stats["spans"] += 1
            end = seq.prompt_len
        while kvlen - end >= self.segment_tokens:
            reg.tag_range(end, end + self.segment_tokens, CacheTag.MODEL_GENERATION)
            self.stats["spans"] += 1
            end += self.segment_tokens
        self._end[sid] = end

    def _retrieve(self, seq) -> None:
        from .tiers import find_retrieve_requests
        toks = seq.all_token_ids
        start = self._scanned.get(seq.seq_id, len(seq.prompt_token_ids))
        if start >= len(toks):
            return
        new = [t for t in toks[start:] if t >= 0]
        self._scanned[seq.seq_id] = len(toks)
        try:
            text = self._tail.get(seq.seq_id, "") + self.eng.tokenizer.decode(new)
        except Exception:
            return
        keys = find_retrieve_requests(text)
        cut = text.rfind("<RETRIEVE:")
        self._tail[seq.seq_id] = text[cut:] if cut >= 0 and ">" not in text[cut:] else ""
        for key in keys:
            if key not in self.tiers.entries:
                continue
            reg = self.seg.registry(seq)
            end = self._end.get(seq.seq_id, 0)
            kvlen = seq.num_computed_tokens
            if kvlen > end:                      # cover the uncovered tail first
                reg.tag_range(end, kvlen, CacheTag.MODEL_GENERATION)
                self.stats["spans"] += 1
            n = self.tiers.promote(seq, key)
            span = reg.tag_range(kvlen, kvlen + n, CacheTag.LONG_TERM_MEMORY, key)
            self._grace.setdefault(seq.seq_id, {})[span] = self.segment_tokens
            self._end[seq.seq_id] = kvlen + n
            self.stats["promoted"] += 1

    def after_step(self, engine) -> None:
        for seq in list(engine.scheduler.running):
            if seq.num_uncomputed != 1:            # still prefilling: nothing settled yet
                continue
            self._retrieve(seq)
            self._register(seq)
            before_kv = seq.num_computed_tokens
            grace = self._grace.get(seq.seq_id, {})
            spans = self.seg.step(seq, self.context_limit, protected=list(grace))
            for sid in list(grace):
                grace[sid] -= 1
                if grace[sid] <= 0:
                    del grace[sid]
            if spans and not self.cfg.shadow_mode:
                self.stats["evicted_spans"] += len(spans)
                # every evicted position lay below the covered end: it moves left as much
                self._end[seq.seq_id] = self._end.get(seq.seq_id, 0) - \
                    (before_kv - seq.num_computed_tokens)
                self._record_facts(seq, spans)

    def _record_facts(self, seq, span_ids: List[int]) -> None:
        """A knowledge-base fact per demoted span, keyed by its tier key (what a
        ``<RETRIEVE:key>`` names)."""
        self.stats["demoted"] = self.tiers.stats["demoted"]
        if self.kb is None:
            return
        from ..extras.knowledge import EvictionRecord, Fact
        for sid in span_ids:
            key = f"seq{seq.seq_id}-span{sid}"
            e = self.tiers.entries.get(key)
            if e is None or self.kb.peek_fact(key) is not None:
                continue
            lo, hi = (e.positions[0], e.positions[-1] + 1) if e.positions else (0, 0)
            self.kb.add_fact(Fact(self.summarize(e.token_ids), source=f"evicted_{lo}_{hi}",
                                  key=key, summary=e.summary or self.summarize(e.token_ids),
                                  source_tokens=list(e.token_ids)))
            self.kb.evictions.append(EvictionRecord(key, (lo, hi), f"[KB:{key}] {e.summary}",
                                                    time.time()))

    def placeholders(self, seq) -> List[str]:
        """``[KB:key] summary`` lines of the spans demoted from ``seq``."""
        return [f"[KB:{k}] {e.summary}" for k, e in self.tiers.entries.items()
                if e.seq_id == seq.seq_id]

