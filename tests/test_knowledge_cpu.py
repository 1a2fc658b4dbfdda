"""Knowledge base depth (reference src/engine/knowledge_base.rs): categories, eviction
records with placeholders, retrieval counting, stats, limits and the convergence detector."""
import copy

import pytest

from lightbulb_b200.extras.knowledge import (ConvergenceDetector, Fact, KnowledgeBase,
                                             KnowledgeBaseConfig, KnowledgeBaseError)


def test_fact_placeholder_category_and_confidence_clamp():
    f = Fact("Paris is the capital of France. Population 2.1M.", key="paris",
             summary="Paris is capital of France", category="factual", confidence=1.7)
    assert f.as_placeholder() == "[KB:paris] Paris is capital of France"
    assert f.confidence == 1.0 and f.retrieval_count == 0
    with pytest.raises(ValueError):
        Fact("x", category="gossip")


def test_eviction_creates_fact_record_and_retrieval():
    kb = KnowledgeBase()
    k1 = kb.create_fact_from_eviction("GDP 25.5T", "US GDP was $25.5T in 2022 ...", (150, 200),
                                      tokens=[5, 6, 7], category="numerical")
    k2 = kb.create_fact_from_eviction("war ended 1945", "The war ended in 1945.", (200, 260),
                                      category="temporal")
    assert (k1, k2) == ("fact_1", "fact_2")
    rec = kb.eviction_history()
    assert [r.position_range for r in rec] == [(150, 200), (200, 260)]
    assert rec[0].placeholder_text == "[KB:fact_1] GDP 25.5T"
    f = kb.peek_fact(k1)
    assert f.source == "evicted_150_200" and f.source_tokens == [5, 6, 7]
    assert f.retrieval_count == 0
    assert kb.get_fact(k1).retrieval_count == 1 and kb.get_fact(k1).retrieval_count == 2
    st = kb.stats()
    assert st["fact_count"] == 2 and st["eviction_count"] == 2 and st["retrieval_count"] == 2
    assert st["facts_by_category"] == {"numerical": 1, "temporal": 1}
    assert st["most_retrieved_key"] == "fact_1"
    assert [f.key for f in kb.facts_by_category("temporal")] == ["fact_2"]
    assert "[fact_2] war ended 1945 (confidence: 1.00)" in kb.to_context_string()
    with pytest.raises(KnowledgeBaseError):
        kb.get_fact("nope")


def test_duplicates_limits_clear_and_copy():
    kb = KnowledgeBase(KnowledgeBaseConfig(max_facts=2))
    kb.add_fact(Fact("a", key="k"))
    with pytest.raises(KnowledgeBaseError):
        kb.add_fact(Fact("b", key="k"))
    kb.add_fact(Fact("c", key="j"))
    with pytest.raises(KnowledgeBaseError):
        kb.add_fact(Fact("d", key="z"))                       # full
    twin = copy.deepcopy(kb)
    kb.clear()
    assert len(kb) == 0 and len(twin) == 2 and twin.get("j").content == "c"
    # the older free-form API keeps working (newest fact wins a shared key)
    kb.add("GDP was 25 trillion", key="gdp")
    kb.add("GDP was 26 trillion", key="gdp")
    assert kb.get("gdp").content.endswith("26 trillion")
    assert kb.query("GDP trillion")[0]["content"].startswith("GDP")


def test_convergence_detector():
    c = ConvergenceDetector(max_iterations=5, min_new_facts=2)
    c.record_iteration(4)
    c.record_iteration(3)
    assert not c.has_converged()
    c.record_iteration(1)
    assert c.has_converged() and "saturation" in c.reason and c.total_facts() == 8
    d = ConvergenceDetector(max_iterations=2, min_new_facts=0)
    d.record_iteration(9)
    d.record_iteration(9)
    assert d.has_converged() and d.reason == "Max iterations (2) reached"
