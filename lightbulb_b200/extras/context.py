"""Context injection: providers contribute snippets for a query, a manager merges them under a
size budget, and the result is placed around the prompt.  Also the conversation history that
feeds recent turns back as context.

Reference: ``src/engine/context_injection.rs:83-560`` (positions, injections with priority
and an "essential" flag, provider configs that activate on intents / keywords, manager that
collects results and merges by priority under a byte budget) and
``src/engine/conversation_history.rs:13-190`` (bounded turn log, oldest turns dropped first
when the token or turn limit is exceeded, recent turns as essential chat-history context).

Differences: providers run in registration order (deterministic); a provider that raises is
reported as a failed result and skipped; :func:`assemble` renders the merged context into the
final prompt text.
"""
from __future__ import annotations

import enum
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Sequence

from .knowledge import KnowledgeBase
from .query import AnalyzedQuery, Intent


class ContextError(RuntimeError):
    pass


class Position(str, enum.Enum):
    BEFORE_PROMPT = "before_prompt"
    AFTER_PROMPT = "after_prompt"
    SYSTEM_MESSAGE = "system_message"
    CHAT_HISTORY = "chat_history"


@dataclass
class ContextInjection:
    content: str
    position: Position
    source: str
    priority: int = 50
    essential: bool = False
    metadata: Dict[str, str] = field(default_factory=dict)

    @property
    def size(self) -> int:
        return len(self.content.encode())


@dataclass
class ProviderConfig:
    id: str
    enabled: bool = True
    timeout_s: float = 5.0
    max_context_size: int = 10_000
    trigger_intents: List[Intent] = field(default_factory=list)
    trigger_keywords: List[str] = field(default_factory=list)
    params: Dict[str, str] = field(default_factory=dict)

    def should_activate(self, q: AnalyzedQuery) -> bool:
        if not self.enabled:
            return False
        if self.trigger_intents and q.intent not in self.trigger_intents:
            return False
        if self.trigger_keywords:
            low = q.original.lower()
            if not any(k.lower() in low for k in self.trigger_keywords):
                return False
        return True


@dataclass
class ProviderResult:
    provider_id: str
    success: bool
    injections: List[ContextInjection] = field(default_factory=list)
    error: Optional[str] = None
    elapsed_ms: float = 0.0


class ContextProvider:
    """Base class: override :meth:`provide`."""

    def __init__(self, config: ProviderConfig):
        self.config = config

    @property
    def id(self) -> str:
        return self.config.id

    def provide(self, q: AnalyzedQuery, prompt: str) -> List[ContextInjection]:
        raise NotImplementedError


class StaticContextProvider(ContextProvider):
    """Fixed snippets keyed by a keyword found in the query."""

    def __init__(self, id: str, config: Optional[ProviderConfig] = None):
        super().__init__(config or ProviderConfig(id))
        self.entries: List[tuple] = []

    def add(self, keyword: str, injection: ContextInjection) -> "StaticContextProvider":
        self.entries.append((keyword.lower(), injection))
        return self

    def provide(self, q, prompt):
        low = q.original.lower()
        return [inj for k, inj in self.entries if k in low]


class KnowledgeProvider(ContextProvider):
    """Facts from the knowledge base that overlap the query, as system-message context."""

    def __init__(self, kb: KnowledgeBase, top_k: int = 3, min_score: float = 0.1,
                 config: Optional[ProviderConfig] = None):
        super().__init__(config or ProviderConfig("knowledge_base"))
        self.kb, self.top_k, self.min_score = kb, top_k, min_score

    def provide(self, q, prompt):
        return [ContextInjection(f"Known fact: {h['content']}", Position.SYSTEM_MESSAGE,
                                 self.id, priority=int(60 + 40 * h["score"]))
                for h in self.kb.query(q.original, self.top_k, self.min_score)]


class FunctionProvider(ContextProvider):
    """Wraps ``fn(query, prompt) -> list[ContextInjection]``."""

    def __init__(self, id: str, fn: Callable, config: Optional[ProviderConfig] = None):
        super().__init__(config or ProviderConfig(id))
        self.fn = fn

    def provide(self, q, prompt):
        return list(self.fn(q, prompt))


class ContextManager:
    def __init__(self, max_total_size: int = 50_000):
        self.max_total_size = max_total_size
        self.providers: Dict[str, ContextProvider] = {}

    def register(self, p: ContextProvider) -> None:
        self.providers[p.id] = p

    def provide(self, q: AnalyzedQuery, prompt: str) -> List[ProviderResult]:
        out = []
        for p in self.providers.values():
            if not p.config.should_activate(q):
                continue
            t0 = time.perf_counter()
            try:
                inj = p.provide(q, prompt)
                inj = [i for i in inj if i.size <= p.config.max_context_size]
                out.append(ProviderResult(p.id, True, inj,
                                          elapsed_ms=(time.perf_counter() - t0) * 1e3))
            except Exception as e:   # a failing provider is reported, not fatal
                out.append(ProviderResult(p.id, False, error=str(e),
                                          elapsed_ms=(time.perf_counter() - t0) * 1e3))
        return out

    def merge(self, results: Sequence[ProviderResult]) -> Dict[Position, List[ContextInjection]]:
        """Highest priority first while the byte budget lasts; optional snippets that do not
        fit are dropped, an essential one that does not fit is an error."""
        items = [i for r in results if r.success for i in r.injections]
        items.sort(key=lambda i: -i.priority)           # stable: ties keep provider order
        merged: Dict[Position, List[ContextInjection]] = {}
        used = 0
        for inj in items:
            if used + inj.size > self.max_total_size:
                if inj.essential:
                    raise ContextError(f"context too large: {used + inj.size} bytes "
                                       f"(max {self.max_total_size})")
                continue
            used += inj.size
            merged.setdefault(inj.position, []).append(inj)
        return merged


def assemble(prompt: str, merged: Dict[Position, List[ContextInjection]],
             system: str = "") -> dict:
    """Render merged context: returns ``{"system": ..., "history": [...], "prompt": ...}``."""
    def txt(pos):
        return [i.content for i in merged.get(pos, [])]

    sys_parts = ([system] if system else []) + txt(Position.SYSTEM_MESSAGE)
    body = "\n\n".join(txt(Position.BEFORE_PROMPT) + [prompt] + txt(Position.AFTER_PROMPT))
    return {"system": "\n".join(sys_parts), "history": txt(Position.CHAT_HISTORY),
            "prompt": body}


# ---------------------------------------------------------------------------------------
# conversation history
# ---------------------------------------------------------------------------------------
class Role(str, enum.Enum):
    SYSTEM = "system"
    USER = "user"
    ASSISTANT = "assistant"


@dataclass
class Turn:
    id: int
    role: Role
    content: str
    timestamp: float = field(default_factory=time.time)

    @property
    def tokens(self) -> int:
        return len(self.content.split())


@dataclass
class ConversationConfig:
    max_recent_turns: int = 20
    max_total_tokens: int = 4000
    summarization_threshold: int = 10


class ConversationHistory:
    def __init__(self, config: Optional[ConversationConfig] = None):
        self.config = config or ConversationConfig()
        self.turns: Deque[Turn] = deque()
        self._next = 1
        self.total_tokens = 0

    def add(self, role: Role, content: str) -> int:
        t = Turn(self._next, Role(role), content)
        self._next += 1
        self.turns.append(t)
        self.total_tokens += t.tokens
        while self.turns and (self.total_tokens > self.config.max_total_tokens or
                              len(self.turns) > self.config.max_recent_turns):
            self.total_tokens -= self.turns.popleft().tokens
        return t.id

    def recent(self, n: int) -> List[Turn]:
        return list(self.turns)[-n:] if n > 0 else []

    def search(self, query: str, max_results: int = 5) -> List[Turn]:
        q = query.lower()
        return [t for t in self.turns if q in t.content.lower()][:max_results]

    def injections(self, n: int) -> List[ContextInjection]:
        return [ContextInjection(f"{t.role.value.capitalize()}: {t.content}",
                                 Position.CHAT_HISTORY, "conversation_history", priority=80,
                                 essential=True) for t in self.recent(n)]

    def clear(self) -> None:
        self.turns.clear()
        self.total_tokens = 0

    def summary(self) -> str:
        if not self.turns:
            return "Empty conversation"
        u = sum(t.role == Role.USER for t in self.turns)
        a = sum(t.role == Role.ASSISTANT for t in self.turns)
        return (f"Conversation with {len(self.turns)} turns ({u} user, {a} assistant), "
                f"{self.total_tokens} tokens")
