"""Query analysis: intent, entities, constraints, ambiguities and sub-queries of a user query.

Reference: ``src/engine/query_analysis.rs:59-700``.  Intent comes from trigger phrases (the
phrase table is the reference's; a match at the start of the query and a longer phrase score
higher: confidence = (0.7 + 0.3 * len / 20) x (1.0 at the start, else 0.8)); candidates are
tried in a fixed order so ties resolve the same way every run.  Entities are capitalised
words (paths when they contain "." or "/"), constraints are temporal / category cues, and
ambiguities are vague pronouns or several questions.  A compound query is split at question
marks (or at " and " when long); later parts that compare, evaluate or follow ("then",
"next", "after") depend on earlier ones.
"""
from __future__ import annotations

import enum
import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple


class QueryAnalysisError(ValueError):
    pass


class Intent(str, enum.Enum):
    DEFINITION = "definition"
    PROCEDURE = "procedure"
    COMPARISON = "comparison"
    TROUBLESHOOTING = "troubleshooting"
    EXPLANATION = "explanation"
    ANALYSIS = "analysis"
    SYNTHESIS = "synthesis"
    FACTUAL = "factual"
    UNKNOWN = "unknown"


# trigger phrases per intent (observable behaviour of the reference's classifier)
INTENT_PHRASES: Dict[Intent, Tuple[str, ...]] = {
    Intent.DEFINITION: ("what is", "what are", "define", "definition of", "meaning of",
                        "what does", "what's"),
    Intent.PROCEDURE: ("how to", "how do i", "how can i", "steps to", "guide to", "tutorial",
                       "instructions for"),
    Intent.COMPARISON: (" vs ", " versus ", "difference between", "compare", "comparison of",
                        "better than", "worse than"),
    Intent.TROUBLESHOOTING: ("why doesn't", "why won't", "how to fix", "not working", "error",
                             "problem with", "issue with", "troubleshoot"),
    Intent.EXPLANATION: ("why does", "why is", "how does", "how is", "explain",
                         "explanation of", "reason for"),
    Intent.ANALYSIS: ("should i", "is it", "evaluate", "assess", "pros and cons",
                      "advantages of", "disadvantages of"),
    Intent.SYNTHESIS: ("summarize", "summary of", "key points", "main ideas", "overview of",
                       "what are the"),
    Intent.FACTUAL: ("when was", "when did", "who is", "who was", "where is", "where was",
                     "which"),
}

_QUESTION_WORDS = {"what", "when", "where", "who", "why", "how", "the", "and", "or"}
_PRONOUNS = ("it", "this", "that", "they", "them")


@dataclass
class Entity:
    text: str
    kind: str              # path | concept | other
    position: int          # word index
    confidence: float = 0.6


@dataclass
class Constraint:
    kind: str              # temporal | category
    value: str
    operator: str          # gt | lt | eq | ne


@dataclass
class SubQuery:
    text: str
    intent: Intent
    depends_on: List[int] = field(default_factory=list)
    priority: int = 0


@dataclass
class AnalyzedQuery:
    original: str
    intent: Intent
    confidence: float
    entities: List[Entity] = field(default_factory=list)
    constraints: List[Constraint] = field(default_factory=list)
    ambiguities: List[str] = field(default_factory=list)
    sub_queries: List[SubQuery] = field(default_factory=list)
    metadata: Dict[str, str] = field(default_factory=dict)


def _has_word(text: str, word: str) -> bool:
    return re.search(rf"\b{re.escape(word)}\b", text) is not None


class QueryAnalyzer:
    def __init__(self, max_query_length: int = 10000,
                 phrases: Optional[Dict[Intent, Tuple[str, ...]]] = None):
        self.max_query_length = max_query_length
        self.phrases = phrases or INTENT_PHRASES

    def classify(self, text: str) -> Tuple[Intent, float]:
        q = text.lower()
        if "compare" in q and ("how does" in q or "how do" in q):
            return Intent.COMPARISON, 0.85
        best, conf = Intent.UNKNOWN, 0.0
        for intent, phrases in self.phrases.items():
            for ph in phrases:
                if ph in q:
                    c = (0.7 + 0.3 * len(ph) / 20.0) * (1.0 if q.startswith(ph) else 0.8)
                    if c > conf:
                        best, conf = intent, c
        return best, (min(conf, 1.0) if conf > 0 else 0.3)

    def analyze(self, query: str) -> AnalyzedQuery:
        if not query.strip():
            raise QueryAnalysisError("empty query")
        if len(query) > self.max_query_length:
            raise QueryAnalysisError(f"query of {len(query)} characters exceeds "
                                     f"{self.max_query_length}")
        intent, conf = self.classify(query)
        q = query.lower()
        return AnalyzedQuery(query, intent, conf, self._entities(query), self._constraints(q),
                             self._ambiguities(q))

    @staticmethod
    def _entities(query: str) -> List[Entity]:
        out = []
        for i, w in enumerate(query.split()):
            clean = "".join(c for c in w if c.isalnum() or c == "-")
            if len(clean) > 1 and clean[0].isupper() and clean.lower() not in _QUESTION_WORDS:
                kind = "path" if ("." in w.rstrip(".?!,") or "/" in w) else "concept"
                out.append(Entity(clean, kind, i))
        return out

    @staticmethod
    def _constraints(q: str) -> List[Constraint]:
        out = []
        if _has_word(q, "after") or _has_word(q, "since"):
            out.append(Constraint("temporal", "recent", "gt"))
        if _has_word(q, "before") or _has_word(q, "until"):
            out.append(Constraint("temporal", "past", "lt"))
        if _has_word(q, "only") or _has_word(q, "just"):
            out.append(Constraint("category", "exclusive", "eq"))
        if _has_word(q, "exclude") or _has_word(q, "without"):
            out.append(Constraint("category", "exclusive", "ne"))
        return out

    @staticmethod
    def _ambiguities(q: str) -> List[str]:
        out = [f"pronoun '{p}' may be unclear" for p in _PRONOUNS if _has_word(q, p)]
        n = q.count("?")
        if n > 1:
            out.append(f"multiple questions detected ({n})")
        return out

    # -------------------------------------------------------------------------------
    def decompose(self, aq: AnalyzedQuery) -> AnalyzedQuery:
        """Fill ``aq.sub_queries`` for compound queries (no-op for simple ones)."""
        text = aq.original
        if text.count("?") <= 1 and " and " not in text and " or " not in text:
            return aq
        if text.count("?") > 1:
            parts = [p.strip() + "?" for p in text.split("?") if p.strip()]
        elif " and " in text and len(text) > 100:
            parts = [p.strip() for p in text.split(" and ") if len(p.strip()) > 20]
        else:
            parts = []
        parts = parts or [text]
        subs: List[SubQuery] = []
        for i, part in enumerate(parts):
            low = part.lower()
            deps: List[int] = []
            if i > 0:
                if "compare" in low or "difference" in low or " vs " in low:
                    deps = list(range(i))
                elif any(_has_word(low, w) for w in ("evaluate", "assess", "should", "then",
                                                      "next", "after")):
                    deps = [i - 1]
            subs.append(SubQuery(part, self.classify(part)[0], deps, priority=len(parts) - i))
        aq.sub_queries = subs
        return aq
