"""Knowledge base behind ``/v1/lightbulb/knowledge/*`` (reference ``src/engine/knowledge_base.rs``,
routes ``src/api/lightbulb.rs:18-24``): facts with source, confidence and category,
keyword-overlap retrieval, claim validation, and the eviction side of the reference's design:
content evicted from a sequence's KV cache becomes a fact with a generated key, an eviction
record keeps the evicted position range and the ``[KB:key] summary`` placeholder left in its
place, and ``<RETRIEVE:key>`` brings the full content back (``knowledge_base.rs:63-200,
446-520``).  A convergence detector stops iterative fact-gathering loops at saturation
(``knowledge_base.rs:523-600``).  Host-side logic, no tensors."""
from __future__ import annotations

import copy
import re
import threading
import time
import uuid
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional, Tuple

_WORD = re.compile(r"[a-z0-9]+")

# Fact categories of the reference (``FactCategory``): factual, numerical, temporal, relational,
# procedural, general.
CATEGORIES = ("factual", "numerical", "temporal", "relational", "procedural", "general")

SYSTEM_INSTRUCTIONS = (
    "KNOWLEDGE BASE SYSTEM:\n"
    "Some earlier content was moved out of your context to save memory. A line\n"
    "  [KB:key] summary\n"
    "stands for such content; the summary is a short overview. To get the full text back,\n"
    "output <RETRIEVE:key> and it will be inserted. Keep these instructions in context.")


def _toks(s: str) -> set:
    return set(_WORD.findall(s.lower()))


class KnowledgeBaseError(KeyError):
    pass


@dataclass
class Fact:
    content: str                        # full content (the reference's full_content)
    source: str = "user"
    confidence: float = 1.0
    key: Optional[str] = None          # optional name for exact lookup (e.g. "gdp_2023")
    id: str = field(default_factory=lambda: uuid.uuid4().hex[:12])
    created: float = field(default_factory=time.time)
    summary: str = ""                   # one-line summary shown in the placeholder
    category: str = "general"
    retrieval_count: int = 0
    source_tokens: Optional[List[int]] = None

    def __post_init__(self):
        if self.category not in CATEGORIES:
            raise ValueError(f"category must be one of {CATEGORIES}")
        self.confidence = min(1.0, max(0.0, float(self.confidence)))
        if not self.summary:
            self.summary = self.content if len(self.content) <= 120 else self.content[:117] + "..."

    def as_placeholder(self) -> str:
        return f"[KB:{self.key}] {self.summary}"


@dataclass
class EvictionRecord:
    fact_key: str
    position_range: Tuple[int, int]
    placeholder_text: str
    timestamp: float


@dataclass
class KnowledgeBaseConfig:
    max_facts: int = 0              # 0: unlimited; when full, new facts are rejected
    auto_generate_keys: bool = True  # fact_1, fact_2, ... (else time-based)
    track_evictions: bool = True
    enable_stats: bool = True


class ConvergenceDetector:
    """Stop an iterative fact-gathering loop after ``max_iterations`` or when an iteration adds
    fewer than ``min_new_facts`` facts (saturation)."""

    def __init__(self, max_iterations: int, min_new_facts: int):
        self.max_iterations = max_iterations
        self.min_new_facts = min_new_facts
        self.facts_per_iteration: List[int] = []
        self.converged = False
        self.reason: Optional[str] = None

    @property
    def current_iteration(self) -> int:
        return len(self.facts_per_iteration)

    def record_iteration(self, new_facts: int) -> None:
        self.facts_per_iteration.append(int(new_facts))
        if self.current_iteration >= self.max_iterations:
            self.converged = True
            self.reason = f"Max iterations ({self.max_iterations}) reached"
        elif new_facts < self.min_new_facts:
            self.converged = True
            self.reason = (f"Fact saturation detected (only {new_facts} new facts, "
                           f"threshold: {self.min_new_facts})")

    def has_converged(self) -> bool:
        return self.converged

    def total_facts(self) -> int:
        return sum(self.facts_per_iteration)


class KnowledgeBase:
    def __init__(self, config: Optional[KnowledgeBaseConfig] = None):
        self.config = config or KnowledgeBaseConfig()
        self.facts: List[Fact] = []
        self.evictions: List[EvictionRecord] = []
        self.retrievals = 0
        self._key_counter = 0
        self._lock = threading.Lock()

    def add(self, content: str, source: str = "user", confidence: float = 1.0,
            key: Optional[str] = None, summary: str = "", category: str = "general") -> Fact:
        f = Fact(content, source, float(confidence), key, summary=summary, category=category)
        return self.add_fact(f, allow_duplicate_key=True)

    def add_fact(self, f: Fact, allow_duplicate_key: bool = False) -> Fact:
        """Store ``f``.  Rejects a key already present (unless allowed: then the newest fact
        wins lookups) and, with ``max_facts``, a full base."""
        with self._lock:
            if f.key is not None and not allow_duplicate_key and \
                    any(g.key == f.key for g in self.facts):
                raise KnowledgeBaseError(f"Fact with key {f.key} already exists")
            if self.config.max_facts and len(self.facts) >= self.config.max_facts:
                raise KnowledgeBaseError("Knowledge base is full")
            self.facts.append(f)
        return f

    def _new_key(self) -> str:
        if self.config.auto_generate_keys:
            self._key_counter += 1
            return f"fact_{self._key_counter}"
        return f"fact_{time.time_ns()}"

    def create_fact_from_eviction(self, summary: str, full_content: str,
                                  position_range: Tuple[int, int],
                                  tokens: Optional[List[int]] = None,
                                  category: str = "general") -> str:
        """Content evicted from positions ``position_range`` of a KV cache becomes a fact; the
        returned key is what a ``[KB:key]`` placeholder and ``<RETRIEVE:key>`` name."""
        with self._lock:
            key = self._new_key()
        f = Fact(full_content, f"evicted_{position_range[0]}_{position_range[1]}", 1.0, key,
                 summary=summary, category=category,
                 source_tokens=list(tokens) if tokens is not None else None)
        self.add_fact(f)
        if self.config.track_evictions:
            with self._lock:
                self.evictions.append(EvictionRecord(key, tuple(position_range),
                                                     f.as_placeholder(), f.created))
        return key

    def get_fact(self, key: str) -> Fact:
        """Retrieval by key (counts as a retrieval)."""
        f = self.get(key)
        if f is None:
            raise KnowledgeBaseError(f"Fact with key {key} not found")
        with self._lock:
            f.retrieval_count += 1
            self.retrievals += 1
        return f

    def peek_fact(self, key: str) -> Optional[Fact]:
        return self.get(key)

    def facts_by_category(self, category: str) -> List[Fact]:
        with self._lock:
            return [f for f in self.facts if f.category == category]

    def eviction_history(self) -> List[EvictionRecord]:
        with self._lock:
            return list(self.evictions)

    def to_context_string(self) -> str:
        with self._lock:
            if not self.facts:
                return ""
            lines = [f"[{f.key or f.id}] {f.summary} (confidence: {f.confidence:.2f})"
                     for f in self.facts]
        return "=== Knowledge Base ===\n" + "\n".join(lines) + "\n======================\n"

    @staticmethod
    def system_instructions() -> str:
        return SYSTEM_INSTRUCTIONS

    def stats(self) -> dict:
        with self._lock:
            by_cat: Dict[str, int] = {}
            for f in self.facts:
                by_cat[f.category] = by_cat.get(f.category, 0) + 1
            top = max(self.facts, key=lambda f: f.retrieval_count, default=None)
            return {"fact_count": len(self.facts), "eviction_count": len(self.evictions),
                    "retrieval_count": self.retrievals, "facts_by_category": by_cat,
                    "avg_confidence": (sum(f.confidence for f in self.facts) / len(self.facts)
                                       if self.facts else 0.0),
                    "most_retrieved_key": (top.key if top is not None and top.retrieval_count
                                           else None)}

    def clear(self) -> None:
        with self._lock:
            self.facts.clear()
            self.evictions.clear()
            self.retrievals = 0
            self._key_counter = 0

    def __len__(self) -> int:
        return len(self.facts)

    def __deepcopy__(self, memo):
        """Independent copy (facts cloned, fresh lock): used to explore branches of a plan."""
        kb = KnowledgeBase(copy.copy(self.config))
        with self._lock:
            kb.facts = [copy.copy(f) for f in self.facts]
            kb.evictions = list(self.evictions)
            kb.retrievals, kb._key_counter = self.retrievals, self._key_counter
        return kb

    def get(self, key: str) -> Optional[Fact]:
        """The newest fact stored under ``key`` (exact name), if any."""
        with self._lock:
            for f in reversed(self.facts):
                if f.key == key:
                    return f
        return None

    def query(self, text: str, top_k: int = 5, min_score: float = 0.0) -> List[dict]:
        q = _toks(text)
        scored = []
        with self._lock:
            for f in self.facts:
                t = _toks(f.content)
                if not q or not t:
                    continue
                s = len(q & t) / len(q | t) * f.confidence
                if s > min_score:
                    scored.append((s, f))
        scored.sort(key=lambda x: -x[0])
        return [dict(asdict(f), score=round(s, 4)) for s, f in scored[:top_k]]

    def validate(self, claim: str, threshold: float = 0.5) -> dict:
        hits = self.query(claim, top_k=3)
        best = hits[0]["score"] if hits else 0.0
        return {"claim": claim, "supported": best >= threshold, "score": best, "evidence": hits}
