"""Request metadata, routing to pipelines, adaptive context-provider selection and a context
cache.

Reference: ``src/engine/metadata_scheduling.rs:37-560`` (priority, tags derived from the query
intent, ethical flags, routing rules of required tags ordered by rule priority, confidence
0.5 + 0.5 x matched / all tags, default pipeline otherwise),
``src/engine/adaptive_selection.rs:15-340`` (providers scored per query, adjusted by their
observed success rate, selected all / top-N / by threshold; latency as an EMA with weight 0.1;
fallback providers tried when one fails) and ``src/engine/performance_optimization.rs:71-260``
(TTL + LRU cache of provider contexts keyed by the normalised query and its intent).
"""
from __future__ import annotations

import collections
import enum
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Set, Tuple

from .context import ContextInjection, ContextManager, ContextProvider, ProviderResult
from .query import AnalyzedQuery, Intent


class Priority(enum.IntEnum):
    LOW = 0
    NORMAL = 1
    HIGH = 2
    CRITICAL = 3


# tags implied by each intent (reference table)
INTENT_TAGS: Dict[Intent, Tuple[str, ...]] = {
    Intent.DEFINITION: ("factual",),
    Intent.PROCEDURE: ("procedural", "factual"),
    Intent.COMPARISON: ("comparison", "reasoning"),
    Intent.TROUBLESHOOTING: ("troubleshooting", "reasoning"),
    Intent.EXPLANATION: ("reasoning", "factual"),
    Intent.ANALYSIS: ("reasoning", "comparison"),
    Intent.SYNTHESIS: ("reasoning", "creative"),
    Intent.FACTUAL: ("factual",),
    Intent.UNKNOWN: (),
}


@dataclass
class RequestMetadata:
    request_id: str
    priority: Priority = Priority.NORMAL
    tags: Set[str] = field(default_factory=set)
    context_hints: List[str] = field(default_factory=list)
    ethical_flags: Set[str] = field(default_factory=set)
    episode_id: Optional[str] = None

    @classmethod
    def from_query(cls, request_id: str, q: AnalyzedQuery) -> "RequestMetadata":
        m = cls(request_id, tags=set(INTENT_TAGS.get(q.intent, ())))
        low = q.original.lower()
        if any(k in low for k in ("code", "function", "compile", "rust", "python", "```")):
            m.tags.add("code")
        if any(ch.isdigit() for ch in low) and any(op in low for op in ("+", "*", "/", "=",
                                                                        "sum", "integral")):
            m.tags.add("math")
        m.context_hints = [e.text for e in q.entities]
        return m


@dataclass
class RoutingDecision:
    pipeline: str
    confidence: float
    reason: str
    matched_tags: Set[str] = field(default_factory=set)


@dataclass
class _Rule:
    required: Set[str]
    target: str
    priority: int
    min_priority: Priority = Priority.LOW


class RoutingPolicy:
    def __init__(self, name: str, default_pipeline: str):
        self.name, self.default = name, default_pipeline
        self.rules: List[_Rule] = []

    def add_rule(self, required_tags: Sequence[str], target: str, priority: int = 0,
                 min_priority: Priority = Priority.LOW) -> "RoutingPolicy":
        self.rules.append(_Rule(set(required_tags), target, priority, min_priority))
        self.rules.sort(key=lambda r: -r.priority)        # stable: ties keep insertion order
        return self

    def route(self, m: RequestMetadata) -> RoutingDecision:
        for r in self.rules:
            if r.required <= m.tags and m.priority >= r.min_priority:
                conf = 0.5 + 0.5 * (len(r.required) / len(m.tags)) if m.tags else 0.5
                return RoutingDecision(r.target, conf, f"matched tags {sorted(r.required)}",
                                       set(r.required))
        return RoutingDecision(self.default, 0.5, "no rule matched: default pipeline")


class ConstraintValidator:
    """Blocks requests carrying a forbidden ethical flag and caps per-priority concurrency."""

    def __init__(self, blocked_flags: Sequence[str] = (),
                 max_inflight: Optional[Dict[Priority, int]] = None):
        self.blocked = set(blocked_flags)
        self.max_inflight = max_inflight or {}
        self.inflight: Dict[Priority, int] = collections.Counter()

    def admit(self, m: RequestMetadata) -> Tuple[bool, str]:
        bad = m.ethical_flags & self.blocked
        if bad:
            return False, f"blocked by ethical flags {sorted(bad)}"
        cap = self.max_inflight.get(m.priority)
        if cap is not None and self.inflight[m.priority] >= cap:
            return False, f"{m.priority.name.lower()} priority at its limit ({cap})"
        self.inflight[m.priority] += 1
        return True, "ok"

    def release(self, m: RequestMetadata) -> None:
        self.inflight[m.priority] = max(0, self.inflight[m.priority] - 1)


# ---------------------------------------------------------------------------------------
# adaptive provider selection
# ---------------------------------------------------------------------------------------
class SelectionStrategy(str, enum.Enum):
    ALL = "all"
    TOP_N = "top_n"
    THRESHOLD = "threshold"
    PERFORMANCE_WEIGHTED = "performance_weighted"


@dataclass
class SelectionConfig:
    strategy: SelectionStrategy = SelectionStrategy.TOP_N
    top_n: int = 3
    confidence_threshold: float = 0.6
    max_providers: int = 5
    track_performance: bool = True
    fallbacks: bool = True


@dataclass
class ProviderMetrics:
    total_calls: int = 0
    successful_calls: int = 0
    avg_latency_ms: float = 0.0

    @property
    def success_rate(self) -> float:
        return self.successful_calls / self.total_calls if self.total_calls else 1.0

    def update(self, ok: bool, latency_ms: float) -> None:
        self.total_calls += 1
        self.successful_calls += ok
        self.avg_latency_ms = latency_ms if self.total_calls == 1 else \
            0.9 * self.avg_latency_ms + 0.1 * latency_ms


class ProviderSelector:
    def __init__(self, config: Optional[SelectionConfig] = None):
        self.config = config or SelectionConfig()
        self.providers: Dict[str, Tuple[ContextProvider, Callable[[AnalyzedQuery], float],
                                        Tuple[Intent, ...]]] = {}
        self.metrics: Dict[str, ProviderMetrics] = {}
        self.fallbacks: Dict[str, List[str]] = {}

    def register(self, p: ContextProvider, scorer: Callable[[AnalyzedQuery], float] = None,
                 intents: Sequence[Intent] = ()) -> None:
        self.providers[p.id] = (p, scorer or (lambda q: 1.0), tuple(intents))
        self.metrics[p.id] = ProviderMetrics()

    def set_fallbacks(self, provider_id: str, fallbacks: Sequence[str]) -> None:
        self.fallbacks[provider_id] = list(fallbacks)

    def _adjusted(self, pid: str, base: float) -> float:
        if not self.config.track_performance:
            return base
        m = self.metrics[pid]
        # reliability scales the score; the weighted strategy also prefers fast providers
        s = base * (0.5 + 0.5 * m.success_rate)
        if self.config.strategy == SelectionStrategy.PERFORMANCE_WEIGHTED and m.total_calls:
            s *= 1.0 / (1.0 + m.avg_latency_ms / 1000.0)
        return s

    def select(self, q: AnalyzedQuery) -> List[Tuple[str, float]]:
        c = self.config
        scored = []
        for pid, (p, scorer, intents) in self.providers.items():
            if intents and q.intent not in intents:
                continue
            s = self._adjusted(pid, float(scorer(q)))
            if c.strategy == SelectionStrategy.ALL or s >= c.confidence_threshold:
                scored.append((pid, s))
        scored.sort(key=lambda x: -x[1])
        n = min(c.top_n, c.max_providers) if c.strategy == SelectionStrategy.TOP_N else \
            c.max_providers
        return scored[:n]

    def _call(self, pid: str, q: AnalyzedQuery, prompt: str) -> ProviderResult:
        t = time.perf_counter()
        try:
            inj = self.providers[pid][0].provide(q, prompt)
            r = ProviderResult(pid, True, list(inj))
        except Exception as e:
            r = ProviderResult(pid, False, error=str(e))
        r.elapsed_ms = (time.perf_counter() - t) * 1e3
        if self.config.track_performance:
            self.metrics[pid].update(r.success, r.elapsed_ms)
        return r

    def execute(self, q: AnalyzedQuery, prompt: str) -> List[ProviderResult]:
        out = []
        for pid, _ in self.select(q):
            r = self._call(pid, q, prompt)
            if not r.success and self.config.fallbacks:
                for fb in self.fallbacks.get(pid, []):
                    if fb in self.providers:
                        r2 = self._call(fb, q, prompt)
                        if r2.success:
                            r = r2
                            break
            out.append(r)
        return out


# ---------------------------------------------------------------------------------------
# context cache
# ---------------------------------------------------------------------------------------
@dataclass
class CacheConfig:
    max_entries: int = 1000
    ttl_s: float = 300.0


class ContextCache:
    """Provider contexts keyed by (normalised query, intent); entries expire after ``ttl_s``
    and the least recently used one is evicted beyond ``max_entries``."""

    def __init__(self, config: Optional[CacheConfig] = None, clock=time.monotonic):
        self.config = config or CacheConfig()
        self.clock = clock
        self._d: "collections.OrderedDict[tuple, tuple]" = collections.OrderedDict()
        self._lock = threading.Lock()
        self.hits = self.misses = self.evictions = 0

    @staticmethod
    def key(text: str, q: AnalyzedQuery) -> tuple:
        return (" ".join(text.lower().split()), q.intent)

    def get(self, text: str, q: AnalyzedQuery) -> Optional[List[ContextInjection]]:
        k = self.key(text, q)
        with self._lock:
            v = self._d.get(k)
            if v is None or self.clock() - v[0] > self.config.ttl_s:
                if v is not None:
                    del self._d[k]
                self.misses += 1
                return None
            self._d.move_to_end(k)
            self.hits += 1
            return list(v[1])

    def put(self, text: str, q: AnalyzedQuery, contexts: Sequence[ContextInjection]) -> None:
        with self._lock:
            self._d[self.key(text, q)] = (self.clock(), list(contexts))
            self._d.move_to_end(self.key(text, q))
            while len(self._d) > self.config.max_entries:
                self._d.popitem(last=False)
                self.evictions += 1

    def stats(self) -> dict:
        n = self.hits + self.misses
        return {"entries": len(self._d), "hits": self.hits, "misses": self.misses,
                "evictions": self.evictions, "hit_rate": self.hits / n if n else 0.0}


def provide_cached(manager: ContextManager, cache: ContextCache, q: AnalyzedQuery,
                   prompt: str) -> List[ProviderResult]:
    """:meth:`ContextManager.provide` through the cache (successful results only are kept)."""
    hit = cache.get(prompt, q)
    if hit is not None:
        return [ProviderResult("cache", True, hit)]
    res = manager.provide(q, prompt)
    cache.put(prompt, q, [i for r in res if r.success for i in r.injections])
    return res
