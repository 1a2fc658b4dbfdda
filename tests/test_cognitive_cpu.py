"""Host-side cognitive extras: decomposition, query analysis, context injection, conversation
history, relevance search, consistency checking."""
import pytest
import torch

from lightbulb_b200.extras.consistency import CheckerConfig, ConflictType, ConsistencyChecker
from lightbulb_b200.extras.context import (ContextError, ContextInjection, ContextManager,
                                           ConversationConfig, ConversationHistory,
                                           FunctionProvider, KnowledgeProvider, Position,
                                           ProviderConfig, Role, StaticContextProvider, assemble)
from lightbulb_b200.extras.decomposition import (Complexity, Decomposition, DecompositionEngine,
                                                 DecompositionError, Problem, Strategy,
                                                 SubProblem)
from lightbulb_b200.extras.knowledge import KnowledgeBase
from lightbulb_b200.extras.query import Intent, QueryAnalysisError, QueryAnalyzer
from lightbulb_b200.extras.search import (Document, DocumentMetadata, HybridSearchPipeline,
                                          HydeSearch, KeywordSearch, MetadataFilter,
                                          OverlapReranker, SearchConfig, SearchError,
                                          SemanticSearch, hashed_embedding)


# ---- decomposition --------------------------------------------------------------------
def _kb(**facts):
    kb = KnowledgeBase()
    for k, v in facts.items():
        kb.add(v, key=k)
    return kb


def test_strategy_follows_coverage():
    e = DecompositionEngine(_kb(a="1", b="2", c="3"))
    assert e.decompose(Problem("x").with_complexity(Complexity.SIMPLE)).strategy == Strategy.ATOMIC
    assert e.decompose(Problem("x").requires("a").requires("b")).strategy == Strategy.COMPUTATIONAL
    d = e.decompose(Problem("x").requires("a").requires("q"))          # 0.5 -> hybrid
    assert d.strategy == Strategy.HYBRID
    assert [s.description for s in d.sub_problems] == ["Find q", "Compute: x"]
    assert d.parallel_groups == [[d.sub_problems[0].id], [d.sub_problems[1].id]]
    s = e.decompose(Problem("y").requires("p").requires("q").requires("r"))
    assert s.strategy == Strategy.STRUCTURAL and len(s.sub_problems) == 3
    assert len(s.parallel_groups) == 1 and len(s.parallel_groups[0]) == 3
    st = e.stats()
    assert st["total_decompositions"] == 4 and st["structural_count"] == 1


def test_execution_order_and_cycles():
    p = Problem("z")
    subs = [SubProblem("a", "A"), SubProblem("b", "B", depends_on=["a"]),
            SubProblem("c", "C", depends_on=["a"]), SubProblem("d", "D", depends_on=["b", "c"])]
    d = Decomposition(p, subs, Strategy.STRUCTURAL)
    assert d.execution_order() == ["a", "b", "c", "d"]
    assert d.compute_parallel_groups() == [["a"], ["b", "c"], ["d"]]
    assert d.complexity_score() == pytest.approx(4.0 * 3.0 * 1.0 * 1.0 * 1.8)
    subs[0].depends_on = ["d"]
    with pytest.raises(DecompositionError):
        d.execution_order()


def test_redecompose_after_kb_grows_and_variants():
    kb = _kb(a="1")
    e = DecompositionEngine(kb)
    p = Problem("plan").requires("a").requires("b").requires("c").requires("d")
    d = e.decompose(p)
    assert d.strategy == Strategy.STRUCTURAL and not e.should_redecompose(p.id)
    kb.add("2", key="b")
    kb.add("3", key="c")
    assert e.should_redecompose(p.id)
    nd = e.redecompose(p.id)
    assert nd.strategy == Strategy.HYBRID and e.history[-1].was_redecomposed
    n_before = len(e.history)
    ranked = e.explore_variants([Problem("v").requires("zz"), Problem("v").requires("a")])
    assert ranked[0][1].strategy == Strategy.COMPUTATIONAL and ranked[0][2] > ranked[1][2]
    assert len(e.history) == n_before                 # variants ran on copies
    with pytest.raises(DecompositionError):
        DecompositionEngine(kb).decompose(Problem("deep"), depth=6)


# ---- query analysis -------------------------------------------------------------------
@pytest.mark.parametrize("q,intent", [
    ("What is Rust?", Intent.DEFINITION), ("Define machine learning", Intent.DEFINITION),
    ("How to install Rust?", Intent.PROCEDURE), ("How do I create a file?", Intent.PROCEDURE),
    ("Rust vs Go for web servers", Intent.COMPARISON),
    ("Why doesn't my build work?", Intent.TROUBLESHOOTING),
    ("Explain the borrow checker", Intent.EXPLANATION),
    ("Should I use async here?", Intent.ANALYSIS),
    ("Summarize the release notes", Intent.SYNTHESIS),
    ("When was Python released?", Intent.FACTUAL), ("hello there", Intent.UNKNOWN)])
def test_intent(q, intent):
    a = QueryAnalyzer().analyze(q)
    assert a.intent == intent
    assert a.confidence > 0.7 or intent in (Intent.UNKNOWN, Intent.COMPARISON)


def test_entities_constraints_ambiguities_subqueries():
    qa = QueryAnalyzer()
    a = qa.analyze("Show only Rust files in src/main.rs changed after Tuesday")
    assert {"Rust", "Tuesday"} <= {e.text for e in a.entities}
    assert any(e.kind == "path" for e in a.entities) is False   # lower-case path: no entity
    kinds = {(c.kind, c.operator) for c in a.constraints}
    assert ("temporal", "gt") in kinds and ("category", "eq") in kinds
    b = qa.decompose(qa.analyze("What is Rust? What is Go? Compare them?"))
    assert len(b.sub_queries) == 3 and b.sub_queries[2].depends_on == [0, 1]
    assert any("multiple questions" in s for s in b.ambiguities)
    with pytest.raises(QueryAnalysisError):
        qa.analyze("   ")


# ---- context injection / conversation -------------------------------------------------
def test_context_merge_priority_budget_and_essential():
    qa = QueryAnalyzer()
    q = qa.analyze("How to configure the cache?")
    kb = KnowledgeBase()
    kb.add("the cache size is configured with CACHE_MB")
    m = ContextManager(max_total_size=120)
    m.register(KnowledgeProvider(kb))
    m.register(StaticContextProvider("docs").add("cache", ContextInjection(
        "x" * 100, Position.BEFORE_PROMPT, "docs", priority=10)))
    m.register(FunctionProvider("boom", lambda q, p: 1 / 0))
    m.register(StaticContextProvider("off", ProviderConfig("off", trigger_intents=[
        Intent.DEFINITION])).add("cache", ContextInjection("never", Position.AFTER_PROMPT, "off")))
    res = m.provide(q, q.original)
    assert {r.provider_id for r in res} == {"knowledge_base", "docs", "boom"}
    assert not [r for r in res if r.provider_id == "boom"][0].success
    merged = m.merge(res)
    assert Position.SYSTEM_MESSAGE in merged and Position.BEFORE_PROMPT not in merged  # budget
    out = assemble("How to configure the cache?", merged, system="You are helpful.")
    assert out["system"].startswith("You are helpful.") and "CACHE_MB" in out["system"]
    big = ContextInjection("y" * 500, Position.AFTER_PROMPT, "t", essential=True)
    with pytest.raises(ContextError):
        m.merge([type(res[0])("t", True, [big])])


def test_conversation_history_limits_and_injections():
    h = ConversationHistory(ConversationConfig(max_recent_turns=3, max_total_tokens=10))
    for i in range(5):
        h.add(Role.USER if i % 2 == 0 else Role.ASSISTANT, f"turn {i} word")
    assert len(h.turns) == 3 and h.total_tokens == 9
    assert [t.content for t in h.recent(2)] == ["turn 3 word", "turn 4 word"]
    inj = h.injections(2)
    assert inj[0].content == "Assistant: turn 3 word" and inj[0].essential
    assert inj[0].position == Position.CHAT_HISTORY and inj[0].priority == 80
    h.add(Role.USER, "a b c d e f g h i j k")               # alone over the token budget
    assert h.total_tokens <= 10
    assert "turns" in h.summary() or h.summary() == "Empty conversation"


# ---- relevance search -----------------------------------------------------------------
def _docs():
    texts = ["rust borrow checker ownership rules", "python garbage collector reference counts",
             "rust async runtime tokio executor", "cooking pasta with tomato sauce"]
    return [Document(t, DocumentMetadata(str(i), doc_type="code" if i < 3 else "recipe",
                                         created_at=float(i))) for i, t in enumerate(texts)]


def test_keyword_semantic_hyde_and_filters():
    docs = _docs()
    cfg = SearchConfig(max_results=2)
    kw = KeywordSearch().search("rust ownership", docs, cfg)
    assert kw[0].document.metadata.id == "0"
    sem = SemanticSearch().search("rust ownership rules", docs, cfg)
    assert sem[0].document.metadata.id == "0" and sem[0].score > sem[-1].score
    hy = HydeSearch(generate=lambda q: "tokio is an async runtime for rust").search(
        "what runs rust futures", docs, cfg)
    assert hy[0].document.metadata.id == "2"
    f = SearchConfig(max_results=5, metadata_filter=MetadataFilter(doc_types=["recipe"]))
    assert [r.document.metadata.id for r in KeywordSearch().search("pasta", docs, f)] == ["3"]
    win = SearchConfig(metadata_filter=MetadataFilter(min_created_at=1.0, max_created_at=2.0))
    assert {r.document.metadata.id for r in OverlapReranker().search("rust python", docs, win)} \
        <= {"1", "2"}
    with pytest.raises(SearchError):
        KeywordSearch().search(" ", docs, cfg)
    e = hashed_embedding(["a b", "a b"])
    assert torch.allclose(e[0], e[1]) and abs(float(e[0].norm()) - 1) < 1e-5


def test_hybrid_pipeline_blends_scores():
    docs = _docs()
    pipe = HybridSearchPipeline(SemanticSearch(), OverlapReranker(), retrieval_top_k=3)
    r = pipe.search("rust async executor", docs, SearchConfig(max_results=3))
    assert r[0].document.metadata.id == "2"
    assert set(r[0].sub_scores) == {"retrieval", "rerank"}


# ---- consistency ----------------------------------------------------------------------
def test_consistency_rules():
    c = ConsistencyChecker()
    r = c.validate("The sky is not blue", ["The sky is blue"])
    assert not r.valid and r.conflicts[0].kind == ConflictType.DIRECT_CONTRADICTION
    r = c.validate("The server is dead", ["The server is alive"])
    assert not r.valid
    assert ConflictType.LOGICAL_INCONSISTENCY in {x.kind for x in r.conflicts}
    r = c.validate("Event happened in 2021", ["Event happened in 2020"])
    assert not r.valid and [x.kind for x in r.conflicts] == [ConflictType.TEMPORAL_CONFLICT]
    r = c.validate("London is capital of England", ["Paris is capital of France"])
    assert r.valid and not r.conflicts and r.coherence_score > 0.9
    assert c.validate("Any fact", []).valid
    r = c.validate("Python is a snake", ["Python is a programming language"])
    assert r.valid and r.conflicts[0].kind == ConflictType.SEMANTIC_CONFLICT   # 0.75 < 0.8
    nli = ConsistencyChecker(CheckerConfig(nli=lambda p, h: 0.9))
    assert not nli.validate("Water boils at 50 C", ["Water boils at 100 C"]).valid
    assert c.stats.total_validations == 6 and c.stats.temporal_conflicts == 1
