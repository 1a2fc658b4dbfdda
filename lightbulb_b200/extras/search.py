"""Relevance search over documents: keyword (BM25), semantic (cosine over embeddings), HyDE
(embed a hypothetical answer instead of the query), an overlap reranker, and a two-stage
hybrid pipeline (retrieve top-k, rerank).

Reference: ``src/engine/relevance_search.rs:34-900``.  There, semantic and HyDE search compare
documents against an all-zero placeholder query vector and the hypothetical answer is a fixed
template.  Here the query (or the hypothetical answer) is actually embedded: by default with a
deterministic hashed bag-of-words embedding (signed feature hashing of word unigrams and
bigrams, L2-normalised), or with any ``embed(texts) -> [n, d]`` callable the caller supplies
(e.g. mean-pooled hidden states of a model).  HyDE takes a ``generate(query) -> str``
callable (e.g. a short greedy completion from the engine) and falls back to the template.
Metadata filters follow the reference (document / info type, time window, source, custom
key-value equality).
"""
from __future__ import annotations

import hashlib
import math
import re
from collections import Counter
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import torch

_WORD = re.compile(r"[a-z0-9]+")


class SearchError(ValueError):
    pass


def words(text: str) -> List[str]:
    return _WORD.findall(text.lower())


def hashed_embedding(texts: Sequence[str], dim: int = 512) -> torch.Tensor:
    """[n, dim] L2-normalised signed feature hashing of unigrams and bigrams."""
    out = torch.zeros(len(texts), dim)
    for i, t in enumerate(texts):
        w = words(t)
        feats = w + [a + " " + b for a, b in zip(w, w[1:])]
        for f in feats:
            h = int.from_bytes(hashlib.blake2b(f.encode(), digest_size=8).digest(), "little")
            out[i, h % dim] += 1.0 if (h >> 63) & 1 else -1.0
    return torch.nn.functional.normalize(out, dim=1)


@dataclass
class DocumentMetadata:
    id: str
    doc_type: str = "text"
    info_type: str = "general"
    source: str = ""
    created_at: Optional[float] = None
    custom: Dict[str, str] = field(default_factory=dict)


@dataclass
class Document:
    content: str
    metadata: DocumentMetadata
    embedding: Optional[torch.Tensor] = None


@dataclass
class SearchResult:
    document: Document
    score: float
    strategy: str
    sub_scores: Dict[str, float] = field(default_factory=dict)
    explanation: str = ""


@dataclass
class MetadataFilter:
    doc_types: List[str] = field(default_factory=list)
    info_types: List[str] = field(default_factory=list)
    min_created_at: Optional[float] = None
    max_created_at: Optional[float] = None
    sources: List[str] = field(default_factory=list)
    custom: Dict[str, str] = field(default_factory=dict)

    def matches(self, m: DocumentMetadata) -> bool:
        if self.doc_types and m.doc_type not in self.doc_types:
            return False
        if self.info_types and m.info_type not in self.info_types:
            return False
        if m.created_at is not None:
            if self.min_created_at is not None and m.created_at < self.min_created_at:
                return False
            if self.max_created_at is not None and m.created_at > self.max_created_at:
                return False
        if self.sources and m.source not in self.sources:
            return False
        return all(m.custom.get(k) == v for k, v in self.custom.items())


@dataclass
class SearchConfig:
    max_results: int = 10
    min_score: float = 0.0
    metadata_filter: Optional[MetadataFilter] = None
    include_explanations: bool = False


class SearchStrategy:
    name = "base"

    def search(self, query: str, docs: Sequence[Document],
               cfg: SearchConfig) -> List[SearchResult]:
        raise NotImplementedError

    @staticmethod
    def _check(query: str) -> None:
        if not query.strip():
            raise SearchError("empty query")

    @staticmethod
    def _finish(results: List[SearchResult], cfg: SearchConfig) -> List[SearchResult]:
        results = [r for r in results if r.score >= cfg.min_score]
        results.sort(key=lambda r: -r.score)
        return results[:cfg.max_results]

    @staticmethod
    def _candidates(docs, cfg):
        f = cfg.metadata_filter
        return [d for d in docs if f is None or f.matches(d.metadata)]


class KeywordSearch(SearchStrategy):
    """BM25 (k1 = 1.2, b = 0.75) over the candidate documents."""
    name = "keyword_bm25"

    def __init__(self, k1: float = 1.2, b: float = 0.75):
        self.k1, self.b = k1, b

    def search(self, query, docs, cfg):
        self._check(query)
        cand = self._candidates(docs, cfg)
        toks = [Counter(words(d.content)) for d in cand]
        n = len(cand)
        avg = sum(sum(t.values()) for t in toks) / max(1, n)
        q = set(words(query))
        df = {w: sum(1 for t in toks if w in t) for w in q}
        out = []
        for d, tf in zip(cand, toks):
            dl = sum(tf.values())
            s = 0.0
            for w in q:
                if tf.get(w):
                    idf = math.log(1 + (n - df[w] + 0.5) / (df[w] + 0.5))
                    s += idf * tf[w] * (self.k1 + 1) / (tf[w] + self.k1 *
                                                       (1 - self.b + self.b * dl / max(avg, 1)))
            if s > 0:
                out.append(SearchResult(d, s, self.name))
        return self._finish(out, cfg)


class SemanticSearch(SearchStrategy):
    name = "semantic_search"

    def __init__(self, embed: Optional[Callable] = None, dim: int = 512):
        self.embed = embed or (lambda texts: hashed_embedding(texts, dim))

    def ensure_embeddings(self, docs: Sequence[Document]) -> None:
        missing = [d for d in docs if d.embedding is None]
        if missing:
            e = self.embed([d.content for d in missing])
            for d, v in zip(missing, e):
                d.embedding = v

    def _score(self, qvec: torch.Tensor, docs, cfg, name) -> List[SearchResult]:
        cand = self._candidates(docs, cfg)
        self.ensure_embeddings(cand)
        if not cand:
            return []
        m = torch.stack([d.embedding.float() for d in cand])
        sims = torch.nn.functional.cosine_similarity(m, qvec.float().unsqueeze(0), dim=1)
        out = [SearchResult(d, float(s), name) for d, s in zip(cand, sims.tolist())]
        if cfg.include_explanations:
            for r in out:
                r.explanation = f"cosine similarity {r.score:.3f}"
        return self._finish(out, cfg)

    def search(self, query, docs, cfg):
        self._check(query)
        return self._score(self.embed([query])[0], docs, cfg, self.name)


class HydeSearch(SemanticSearch):
    """Embed a hypothetical answer to the query (optionally averaged with the query)."""
    name = "hyde_search"

    def __init__(self, generate: Optional[Callable[[str], str]] = None,
                 embed: Optional[Callable] = None, dim: int = 512, mix_query: bool = False):
        super().__init__(embed, dim)
        self.generate = generate
        self.mix_query = mix_query

    def hypothetical(self, query: str) -> str:
        if self.generate is not None:
            return self.generate(query)
        return f"Here is a detailed explanation: {query}. This covers the key concepts " \
               f"and provides examples."

    def search(self, query, docs, cfg):
        self._check(query)
        texts = [self.hypothetical(query)] + ([query] if self.mix_query else [])
        v = self.embed(texts).float().mean(0)
        return self._score(v, docs, cfg, self.name)


class OverlapReranker(SearchStrategy):
    """Share of query words present in the (truncated) document."""
    name = "cross_encoder_rerank"

    def __init__(self, max_length: int = 512):
        self.max_length = max_length

    def search(self, query, docs, cfg):
        self._check(query)
        q = words(query)
        out = []
        for d in self._candidates(docs, cfg):
            dw = set(words(d.content[:self.max_length]))
            s = sum(w in dw for w in q) / len(q) if q else 0.0
            r = SearchResult(d, s, self.name)
            if cfg.include_explanations:
                r.explanation = f"query-word overlap {s:.3f}"
            out.append(r)
        return self._finish(out, cfg)


class HybridSearchPipeline(SearchStrategy):
    """Retrieve ``retrieval_top_k`` with the retriever, rerank them, and blend the two scores
    (``alpha`` x rerank + (1 - alpha) x normalised retrieval)."""
    name = "hybrid"

    def __init__(self, retriever: SearchStrategy, reranker: Optional[SearchStrategy] = None,
                 retrieval_top_k: int = 50, alpha: float = 0.5):
        self.retriever, self.reranker = retriever, reranker
        self.k, self.alpha = retrieval_top_k, alpha

    def search(self, query, docs, cfg):
        first = self.retriever.search(query, docs, SearchConfig(
            self.k, 0.0, cfg.metadata_filter, cfg.include_explanations))
        if self.reranker is None or not first:
            return self._finish(first, cfg)
        top = max(r.score for r in first) or 1.0
        base = {id(r.document): r.score / top for r in first}
        rr = self.reranker.search(query, [r.document for r in first],
                                  SearchConfig(len(first), 0.0, None, cfg.include_explanations))
        out = []
        for r in rr:
            s = self.alpha * r.score + (1 - self.alpha) * base[id(r.document)]
            out.append(SearchResult(r.document, s, self.name,
                                    {"retrieval": base[id(r.document)], "rerank": r.score}))
        return self._finish(out, cfg)
