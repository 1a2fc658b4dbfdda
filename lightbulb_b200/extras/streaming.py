"""Streaming context (providers that react to generated tokens) and context compression.

Reference: ``src/engine/streaming_context.rs:25-300`` (stream of providers called per generated
token, at most once every ``min_token_interval`` positions, into a bounded buffer with
backpressure or drop-oldest) and ``src/engine/context_compression.rs:16-400`` (extractive,
entity-preserving, token-budget and hierarchical compression of context text to a target
ratio, code blocks kept intact).

Here the stream is driven from the engine's output: :meth:`ContextStream.feed` takes each
``RequestOutput`` delta of a request; :class:`KeywordStreamProvider` raises injections when
watched phrases appear in the generated text.  Compression scores sentences by the document
frequency of their content words (a sentence that shares many words with the rest of the
text carries its topic), with a bonus for the first sentence, and keeps the best ones in
their original order until the token budget is spent.
"""
from __future__ import annotations

import collections
import enum
import re
import threading
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence

from .context import ContextInjection, Position
from .query import AnalyzedQuery

_WORD = re.compile(r"[A-Za-z0-9_']+")
_STOP = set("a an the and or but of to in on at for with by is are was were be been it this "
            "that these those as from into than then so such".split())


# ---------------------------------------------------------------------------------------
# streaming context
# ---------------------------------------------------------------------------------------
class StreamingProvider:
    id = "stream"

    def start(self, q: AnalyzedQuery) -> None:
        pass

    def on_token(self, token: str, position: int, text: str) -> List[ContextInjection]:
        return []

    def stop(self) -> None:
        pass


class KeywordStreamProvider(StreamingProvider):
    """Emits a snippet the first time a watched phrase appears in the generated text."""

    def __init__(self, id: str, snippets: Dict[str, str], priority: int = 60):
        self.id, self.snippets, self.priority = id, {k.lower(): v for k, v in snippets.items()}, \
            priority
        self._fired: set = set()

    def start(self, q):
        self._fired = set()

    def on_token(self, token, position, text):
        low = text.lower()
        out = []
        for k, v in self.snippets.items():
            if k not in self._fired and k in low:
                self._fired.add(k)
                out.append(ContextInjection(v, Position.AFTER_PROMPT, self.id, self.priority))
        return out


@dataclass
class StreamConfig:
    max_buffer_size: int = 100
    min_token_interval: int = 10
    backpressure: bool = True           # full buffer: refuse new items (else drop oldest)


class ContextStream:
    def __init__(self, config: Optional[StreamConfig] = None):
        self.config = config or StreamConfig()
        self.providers: List[StreamingProvider] = []
        self.buffer: Deque[ContextInjection] = collections.deque()
        self._lock = threading.Lock()
        self._last: Optional[int] = None
        self._text = ""
        self._pos = 0
        self.active = False
        self.dropped = 0

    def register(self, p: StreamingProvider) -> None:
        self.providers.append(p)

    def start(self, q: AnalyzedQuery) -> None:
        self.active, self._last, self._text, self._pos = True, None, "", 0
        for p in self.providers:
            p.start(q)

    def on_token(self, token: str, position: int) -> List[ContextInjection]:
        if not self.active:
            return []
        self._text += token
        if self._last is not None and position - self._last < self.config.min_token_interval:
            return []
        new: List[ContextInjection] = []
        for p in self.providers:
            new.extend(p.on_token(token, position, self._text))
        with self._lock:
            for c in new:
                if len(self.buffer) >= self.config.max_buffer_size:
                    if self.config.backpressure:
                        self.dropped += 1
                        continue
                    self.buffer.popleft()
                    self.dropped += 1
                self.buffer.append(c)
        if new:
            self._last = position
        return new

    def feed(self, output) -> List[ContextInjection]:
        """Feed one engine ``RequestOutput`` (its text delta) into the stream."""
        self._pos += len(output.new_token_ids)
        return self.on_token(output.text_delta or "", self._pos)

    def drain(self) -> List[ContextInjection]:
        with self._lock:
            out = list(self.buffer)
            self.buffer.clear()
        return out

    def stop(self) -> None:
        self.active = False
        for p in self.providers:
            p.stop()


# ---------------------------------------------------------------------------------------
# compression
# ---------------------------------------------------------------------------------------
class CompressionStrategy(str, enum.Enum):
    EXTRACTIVE = "extractive"
    ENTITY_PRESERVING = "entity_preserving"
    TOKEN_BASED = "token_based"
    HIERARCHICAL = "hierarchical"


@dataclass
class CompressionConfig:
    strategy: CompressionStrategy = CompressionStrategy.EXTRACTIVE
    target_ratio: float = 0.5
    preserve_entities: bool = True
    preserve_code: bool = True


@dataclass
class CompressionResult:
    compressed: str
    original_tokens: int
    compressed_tokens: int
    preserved_entities: List[str] = field(default_factory=list)

    @property
    def ratio(self) -> float:
        return self.compressed_tokens / self.original_tokens if self.original_tokens else 0.0


def _tokens(s: str) -> int:
    return len(s.split())


def _sentences(text: str) -> List[str]:
    return [s.strip() for s in re.split(r"(?<=[.!?])\s+|\n{2,}", text) if s.strip()]


def _entities(text: str) -> List[str]:
    out: List[str] = []
    for i, w in enumerate(_WORD.findall(text)):
        if (w[0].isupper() and len(w) > 1 and i > 0) or any(ch.isdigit() for ch in w):
            if w not in out:
                out.append(w)
    return out


class ContextCompressor:
    def __init__(self, config: Optional[CompressionConfig] = None):
        self.config = config or CompressionConfig()

    def compress(self, text: str) -> CompressionResult:
        c = self.config
        code: List[str] = []
        if c.preserve_code:
            def keep(m):
                code.append(m.group(0))
                return f"\x00{len(code) - 1}\x00"
            text = re.sub(r"```.*?```", keep, text, flags=re.S)
        n0 = _tokens(text)
        budget = max(1, int(n0 * c.target_ratio))
        if c.strategy == CompressionStrategy.TOKEN_BASED:
            out = " ".join(text.split()[:budget])
        elif c.strategy == CompressionStrategy.HIERARCHICAL:
            paras = [p for p in re.split(r"\n{2,}", text) if p.strip()]
            share = max(1, budget // max(1, len(paras)))
            out = "\n\n".join(self._extract(p, share) for p in paras)
        else:
            out = self._extract(text, budget,
                                must=_entities(text) if c.strategy ==
                                CompressionStrategy.ENTITY_PRESERVING else ())
        out = re.sub(r"\x00(\d+)\x00", lambda m: code[int(m.group(1))], out)
        ents = [e for e in _entities(out)] if c.preserve_entities else []
        return CompressionResult(out, n0 + sum(_tokens(b) for b in code), _tokens(out), ents)

    @staticmethod
    def _extract(text: str, budget: int, must: Sequence[str] = ()) -> str:
        sents = _sentences(text)
        if not sents:
            return ""
        words = [[w.lower() for w in _WORD.findall(s) if w.lower() not in _STOP] for s in sents]
        df = collections.Counter(w for ws in words for w in set(ws))
        scores = []
        for i, ws in enumerate(words):
            s = sum(df[w] - 1 for w in set(ws)) / (len(ws) ** 0.5 if ws else 1.0)
            if i == 0:
                s += 1.0                      # leading sentence usually states the topic
            if "\x00" in sents[i] or any(m in sents[i] for m in must):
                s += 1e6                      # code placeholders / required entities stay
            scores.append(s)
        chosen, used = set(), 0
        for i in sorted(range(len(sents)), key=lambda i: -scores[i]):
            t = _tokens(sents[i])
            if used + t > budget and chosen and scores[i] < 1e6:
                continue
            chosen.add(i)
            used += t
        return " ".join(sents[i] for i in sorted(chosen))
