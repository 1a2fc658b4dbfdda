"""Knowledge base behind ``/v1/lightbulb/knowledge/*`` (reference ``src/engine/knowledge_base.rs``,
routes ``src/api/lightbulb.rs:18-24``): facts with source and confidence, keyword-overlap
retrieval, and claim validation against stored facts.  Host-side logic, no tensors."""
from __future__ import annotations

import re
import threading
import time
import uuid
from dataclasses import asdict, dataclass, field
from typing import List, Optional

_WORD = re.compile(r"[a-z0-9]+")


def _toks(s: str) -> set:
    return set(_WORD.findall(s.lower()))


@dataclass
class Fact:
    content: str
    source: str = "user"
    confidence: float = 1.0
    key: Optional[str] = None          # optional name for exact lookup (e.g. "gdp_2023")
    id: str = field(default_factory=lambda: uuid.uuid4().hex[:12])
    created: float = field(default_factory=time.time)


class KnowledgeBase:
    def __init__(self):
        self.facts: List[Fact] = []
        self._lock = threading.Lock()

    def add(self, content: str, source: str = "user", confidence: float = 1.0,
            key: Optional[str] = None) -> Fact:
        f = Fact(content, source, float(confidence), key)
        with self._lock:
            self.facts.append(f)
        return f

    def __deepcopy__(self, memo):
        """Independent copy (facts cloned, fresh lock): used to explore branches of a plan."""
        kb = KnowledgeBase()
        with self._lock:
            kb.facts = [Fact(f.content, f.source, f.confidence, f.key, f.id, f.created)
                        for f in self.facts]
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
