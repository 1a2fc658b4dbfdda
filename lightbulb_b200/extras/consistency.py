"""Consistency checking of a new fact against stored facts before it enters the knowledge base.

Reference: ``src/engine/consistency_checking.rs:45-460``.  Conflict kinds and confidences
follow it: "X is Y" vs "X is not Y" is a direct contradiction (0.95), two different "X is ..."
predicates a semantic conflict (0.75), mutually exclusive states of the same subject
(alive/dead, true/false, open/closed, started/stopped, on/off) a logical inconsistency (0.85),
and different years for the same subject a temporal conflict.  A fact is rejected when its
most confident conflict reaches ``rejection_threshold`` (0.8); coherence is
1 - conflicts / facts.

Differences: words are matched whole (the reference's substring tests make "London" contain
"on"); the subject is the text before the first verb; an optional ``nli(premise, hypothesis)``
callable (probability of contradiction, e.g. from a classifier model) is consulted when the
rules find nothing.
"""
from __future__ import annotations

import enum
import re
import time
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence, Tuple

_WORD = re.compile(r"[a-z0-9']+")
_VERBS = {"is", "are", "was", "were", "has", "have", "had", "happened", "occurred", "became",
          "will", "did", "does"}
_STOP = {"the", "a", "an", "this", "that", "these", "those", "of", "in", "on", "at"}
EXCLUSIVE_STATES = (("alive", "dead"), ("true", "false"), ("open", "closed"),
                    ("started", "stopped"), ("on", "off"))
_YEAR = re.compile(r"\b(1[5-9]\d\d|2\d\d\d)\b")


class ConsistencyError(ValueError):
    pass


class ConflictType(str, enum.Enum):
    DIRECT_CONTRADICTION = "direct_contradiction"
    LOGICAL_INCONSISTENCY = "logical_inconsistency"
    TEMPORAL_CONFLICT = "temporal_conflict"
    SEMANTIC_CONFLICT = "semantic_conflict"


@dataclass
class Conflict:
    kind: ConflictType
    existing_fact: str
    explanation: str
    confidence: float


@dataclass
class ValidationResult:
    valid: bool
    conflicts: List[Conflict]
    confidence: float
    coherence_score: float
    latency_us: float


@dataclass
class CheckerConfig:
    detect_contradictions: bool = True
    detect_logical: bool = True
    detect_temporal: bool = True
    rejection_threshold: float = 0.8
    nli: Optional[Callable[[str, str], float]] = None


@dataclass
class CheckerStats:
    total_validations: int = 0
    contradictions_detected: int = 0
    logical_conflicts: int = 0
    temporal_conflicts: int = 0
    avg_latency_us: float = 0.0


def _words(s: str) -> List[str]:
    return _WORD.findall(s.lower())


def subject(s: str) -> Tuple[str, ...]:
    w = _words(s)
    for i, t in enumerate(w):
        if t in _VERBS:
            return tuple(x for x in w[:i] if x not in _STOP)
    return tuple(x for x in w[:2] if x not in _STOP)


def is_statement(s: str) -> Optional[Tuple[Tuple[str, ...], Tuple[str, ...]]]:
    w = _words(s)
    for i, t in enumerate(w):
        if t in ("is", "are", "was", "were"):
            subj = tuple(x for x in w[:i] if x not in _STOP)
            pred = tuple(x for x in w[i + 1:] if x not in ("a", "an", "the"))
            return (subj, pred) if subj and pred else None
    return None


class ConsistencyChecker:
    def __init__(self, config: Optional[CheckerConfig] = None):
        self.config = config or CheckerConfig()
        self.stats = CheckerStats()

    def validate(self, new_fact: str, existing: Sequence[str]) -> ValidationResult:
        if not new_fact.strip():
            raise ConsistencyError("empty fact")
        t0 = time.perf_counter()
        c = self.config
        conflicts: List[Conflict] = []
        if c.detect_contradictions:
            conflicts += self._contradictions(new_fact, existing)
        if c.detect_logical:
            conflicts += self._exclusive_states(new_fact, existing)
        if c.detect_temporal:
            conflicts += self._temporal(new_fact, existing)
        if not conflicts and c.nli is not None:
            for e in existing:
                p = float(c.nli(e, new_fact))
                if p >= 0.5:
                    conflicts.append(Conflict(ConflictType.SEMANTIC_CONFLICT, e,
                                              "entailment model: contradiction", p))
        us = (time.perf_counter() - t0) * 1e6
        s = self.stats
        s.total_validations += 1
        s.contradictions_detected += sum(x.kind == ConflictType.DIRECT_CONTRADICTION
                                         for x in conflicts)
        s.logical_conflicts += sum(x.kind == ConflictType.LOGICAL_INCONSISTENCY for x in conflicts)
        s.temporal_conflicts += sum(x.kind == ConflictType.TEMPORAL_CONFLICT for x in conflicts)
        s.avg_latency_us += (us - s.avg_latency_us) / s.total_validations
        coherence = 1.0 if not conflicts else 1.0 - min(1.0, len(conflicts) / max(1, len(existing)))
        top = max((x.confidence for x in conflicts), default=0.0)
        valid = top < c.rejection_threshold
        conf = 1.0 if valid and not conflicts else (
            sum(x.confidence for x in conflicts) / len(conflicts))
        return ValidationResult(valid, conflicts, conf, coherence, us)

    @staticmethod
    def _contradictions(new: str, existing: Sequence[str]) -> List[Conflict]:
        a = is_statement(new)
        out = []
        if a is None:
            return out
        for e in existing:
            b = is_statement(e)
            if b is None or a[0] != b[0] or a[1] == b[1]:
                continue
            pa = tuple(x for x in a[1] if x != "not")
            pb = tuple(x for x in b[1] if x != "not")
            if ("not" in a[1]) != ("not" in b[1]) and pa == pb:
                out.append(Conflict(ConflictType.DIRECT_CONTRADICTION, e,
                                    f"contradicts the stored fact about {' '.join(a[0])}", 0.95))
            else:
                out.append(Conflict(ConflictType.SEMANTIC_CONFLICT, e,
                                    f"different claims about {' '.join(a[0])}: "
                                    f"'{' '.join(a[1])}' vs '{' '.join(b[1])}'", 0.75))
        return out

    @staticmethod
    def _exclusive_states(new: str, existing: Sequence[str]) -> List[Conflict]:
        nw, ns = set(_words(new)), subject(new)
        out = []
        for e in existing:
            ew = set(_words(e))
            if not ns or subject(e) != ns:
                continue
            for t1, t2 in EXCLUSIVE_STATES:
                if (t1 in nw and t2 in ew) or (t2 in nw and t1 in ew):
                    out.append(Conflict(ConflictType.LOGICAL_INCONSISTENCY, e,
                                        f"mutually exclusive states: {t1} vs {t2}", 0.85))
        return out

    @staticmethod
    def _temporal(new: str, existing: Sequence[str]) -> List[Conflict]:
        ny, ns = set(_YEAR.findall(new)), subject(new)
        out = []
        if not ny:
            return out
        for e in existing:
            ey = set(_YEAR.findall(e))
            if ey and ns and subject(e) == ns and ey != ny:
                out.append(Conflict(ConflictType.TEMPORAL_CONFLICT, e,
                                    f"different times: {sorted(ny)} vs {sorted(ey)}", 0.85))
        return out
