"""Pipelines, routing / provider selection / context cache, streaming context, compression,
mixed-precision profiler."""
import time

import pytest
import torch

from lightbulb_b200.extras.context import (ContextInjection, ContextManager, FunctionProvider,
                                           Position, StaticContextProvider)
from lightbulb_b200.extras.pipeline import (Pipeline, PipelineConfig, PipelineError, Stage,
                                            StageState, StageType)
from lightbulb_b200.extras.precision import (ActivationStats, MixedPrecisionConfig, Precision,
                                             PrecisionProfiler)
from lightbulb_b200.extras.query import Intent, QueryAnalyzer
from lightbulb_b200.extras.routing import (CacheConfig, ConstraintValidator, ContextCache,
                                           Priority, ProviderSelector, RequestMetadata,
                                           RoutingPolicy, SelectionConfig, SelectionStrategy,
                                           provide_cached)
from lightbulb_b200.extras.streaming import (CompressionConfig, CompressionStrategy,
                                             ContextCompressor, ContextStream,
                                             KeywordStreamProvider, StreamConfig)

QA = QueryAnalyzer()


def test_pipeline_levels_parallel_sharing_and_failures():
    p = Pipeline("p", PipelineConfig(max_concurrent_stages=3))
    p.add(Stage("split", StageType.DECOMPOSE, prompt_template="split: {input}"))
    p.add(Stage("a", depends_on=["split"], prompt_template="A {split}"))
    p.add(Stage("b", depends_on=["split"], prompt_template="B {split}"))
    p.add(Stage("bad", depends_on=["split"]))
    p.add(Stage("join", StageType.SYNTHESIZE, depends_on=["a", "b"],
                prompt_template="join {deps}"))
    p.add(Stage("after_bad", depends_on=["bad"]))
    assert p.levels()[0] == ["split"] and set(p.levels()[1]) == {"a", "b", "bad"}
    seen = []

    def ex(prompt, stage):
        seen.append(prompt)
        if stage.id == "bad":
            raise RuntimeError("boom")
        time.sleep(0.01)
        return f"<{stage.id}>"

    res = p.run("q", ex)
    assert res["join"].output == "<join>" and res["join"].cache_shared
    assert p.state["bad"] == StageState.FAILED and p.state["after_bad"] == StageState.SKIPPED
    jp = [s for s in seen if "join" in s][0]
    assert jp.startswith("<a>") and "<b>" in jp          # shared prefix + all deps
    assert p.stats.parallel_stages == 3 and p.stats.failed == 1
    q = Pipeline().add(Stage("x", depends_on=["y"])).add(Stage("y", depends_on=["x"]))
    with pytest.raises(PipelineError):
        q.levels()


def test_routing_and_constraints():
    pol = (RoutingPolicy("default", "general")
           .add_rule(["reasoning", "comparison"], "deliberate", priority=10)
           .add_rule(["factual"], "retrieval", priority=5)
           .add_rule(["troubleshooting"], "debug", priority=1, min_priority=Priority.HIGH))
    m = RequestMetadata.from_query("r1", QA.analyze("Compare apples vs oranges"))
    d = pol.route(m)
    assert d.pipeline == "deliberate" and d.confidence == pytest.approx(1.0)
    assert pol.route(RequestMetadata.from_query("r2", QA.analyze("What is Rust?"))).pipeline \
        == "retrieval"
    t = RequestMetadata.from_query("r3", QA.analyze("Why doesn't my build work?"))
    assert pol.route(t).pipeline == "general"       # troubleshooting rule needs HIGH
    t.priority = Priority.HIGH
    assert pol.route(t).pipeline == "debug"
    v = ConstraintValidator(blocked_flags=["harm"], max_inflight={Priority.LOW: 1})
    low = RequestMetadata("x", Priority.LOW)
    assert v.admit(low)[0] and not v.admit(RequestMetadata("y", Priority.LOW))[0]
    v.release(low)
    assert v.admit(RequestMetadata("z", Priority.LOW))[0]
    assert not v.admit(RequestMetadata("w", ethical_flags={"harm"}))[0]


def test_provider_selection_metrics_and_fallbacks():
    q = QA.analyze("How to configure the cache?")
    sel = ProviderSelector(SelectionConfig(SelectionStrategy.TOP_N, top_n=2,
                                           confidence_threshold=0.3))
    ok = FunctionProvider("ok", lambda q, p: [ContextInjection("x", Position.BEFORE_PROMPT, "ok")])
    flaky = FunctionProvider("flaky", lambda q, p: 1 / 0)
    backup = FunctionProvider("backup", lambda q, p: [ContextInjection("b", Position.AFTER_PROMPT,
                                                                      "backup")])
    sel.register(ok, lambda q: 0.6)
    sel.register(flaky, lambda q: 0.9)
    sel.register(backup, lambda q: 0.1)
    sel.register(FunctionProvider("def", lambda q, p: []), lambda q: 1.0, intents=[Intent.DEFINITION])
    sel.set_fallbacks("flaky", ["backup"])
    assert [p for p, _ in sel.select(q)] == ["flaky", "ok"]
    res = sel.execute(q, q.original)
    assert [r.provider_id for r in res] == ["backup", "ok"] and all(r.success for r in res)
    assert sel.metrics["flaky"].success_rate == 0.0
    assert [p for p, _ in sel.select(q)][0] == "ok"    # flaky demoted: 0.9 * 0.5 < 0.6


def test_context_cache_ttl_lru_and_cached_manager():
    now = [0.0]
    cache = ContextCache(CacheConfig(max_entries=2, ttl_s=10), clock=lambda: now[0])
    q = QA.analyze("What is Rust?")
    inj = [ContextInjection("rust is a language", Position.SYSTEM_MESSAGE, "s")]
    cache.put("What is  Rust?", q, inj)
    assert cache.get("what is rust?", q)[0].content == "rust is a language"
    now[0] = 11
    assert cache.get("What is Rust?", q) is None
    for i in range(3):
        cache.put(f"q{i}", q, inj)
    assert cache.stats()["entries"] == 2 and cache.stats()["evictions"] == 1
    m = ContextManager()
    calls = []
    m.register(FunctionProvider("f", lambda q, p: calls.append(1) or inj))
    c2 = ContextCache(clock=lambda: 0.0)
    provide_cached(m, c2, q, "prompt")
    r = provide_cached(m, c2, q, "prompt")
    assert len(calls) == 1 and r[0].provider_id == "cache"


def test_streaming_interval_backpressure_and_feed():
    s = ContextStream(StreamConfig(max_buffer_size=1, min_token_interval=2))
    s.register(KeywordStreamProvider("kw", {"tokio": "Tokio docs", "serde": "Serde docs"}))
    s.start(QA.analyze("write a server"))
    assert s.on_token("use ", 1) == []
    assert [c.content for c in s.on_token("tokio", 2)] == ["Tokio docs"]
    assert s.on_token(" serde", 3) == []                 # within the interval
    assert [c.content for c in s.on_token(";", 5)] == ["Serde docs"]
    assert [c.content for c in s.drain()] == ["Tokio docs"] and s.dropped == 1   # backpressure

    class Out:
        def __init__(self, t):
            self.new_token_ids, self.text_delta = [0], t
    s2 = ContextStream(StreamConfig(min_token_interval=0))
    s2.register(KeywordStreamProvider("kw", {"tokio": "T"}))
    s2.start(QA.analyze("x"))
    assert s2.feed(Out("to")) == [] and len(s2.feed(Out("kio"))) == 1


def test_compression_strategies():
    text = ("Rust is a systems language focused on safety. Rust ownership rules prevent data "
            "races at compile time. The weather was nice yesterday. Cargo builds Rust crates "
            "and manages dependencies. Lunch had soup.\n\n```fn main() {}```\n\nRust 2021 "
            "edition changed closures.")
    r = ContextCompressor(CompressionConfig(target_ratio=0.5)).compress(text)
    assert r.compressed_tokens < r.original_tokens and "```fn main() {}```" in r.compressed
    assert r.compressed.startswith("Rust is a systems language")
    assert "soup" not in r.compressed
    e = ContextCompressor(CompressionConfig(CompressionStrategy.ENTITY_PRESERVING, 0.3))
    assert "2021" in e.compress(text).compressed
    t = ContextCompressor(CompressionConfig(CompressionStrategy.TOKEN_BASED, 0.2,
                                            preserve_code=False)).compress("a b c d e f g h i j")
    assert t.compressed == "a b" and t.ratio == pytest.approx(0.2)
    h = ContextCompressor(CompressionConfig(CompressionStrategy.HIERARCHICAL, 0.5)).compress(text)
    assert h.compressed_tokens <= r.original_tokens


def test_precision_profiler():
    st = ActivationStats()
    st.update(torch.randn(1000) * 0.5)
    st.update(torch.randn(1000) * 0.5)
    assert abs(st.std - 0.5) < 0.05 and st.recommend() == Precision.INT8
    wide = ActivationStats()
    wide.update(torch.tensor([-3e3, 3e3]))
    assert wide.recommend() == Precision.BF16
    huge = ActivationStats()
    huge.update(torch.tensor([0.0, 2e6]))
    assert huge.recommend() == Precision.FP32
    prof = PrecisionProfiler(MixedPrecisionConfig(profiling_window=2,
                                                  overrides={"layers.0.mlp": Precision.FP32}))
    prof.record_activation("layers.1.mlp", torch.randn(100) * 0.1)
    prof.record_activation("lm_head", torch.randn(100) * 0.1)
    plan = prof.plan(["layers.0.mlp", "layers.1.mlp", "lm_head", "layers.2.attn"])
    assert plan["layers.0.mlp"]["precision"] == "fp32"
    assert plan["layers.1.mlp"] == {"precision": "int8", "format": "q8_0", "memory_ratio": 0.25}
    assert plan["lm_head"]["precision"] == "bf16" and plan["layers.2.attn"]["precision"] == "bf16"
    for _ in range(3):
        prof.end_batch()
    prof.record_accuracy("layers.1.mlp", 0.5)
    assert prof.select("layers.1.mlp") == Precision.FP16       # stepped up
    for us in range(20):
        prof.record_latency("layers.1.mlp", us)
    assert prof.avg_latency("layers.1.mlp") == pytest.approx(sum(range(18, 20)) / 2)
