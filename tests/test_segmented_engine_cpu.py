"""Segmented spans + tiered storage + <RETRIEVE:key> driven by the engine step loop
(reference src/model/parallel_model_manager.rs:626-660,689-853) on the CPU path."""
import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.extras.knowledge import KnowledgeBase
from lightbulb_b200.kv.spans import CacheTag, SegmentedCacheConfig
from lightbulb_b200.models.weights import pack_model, random_weights


def _engine():
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=2, std=0.05)
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=64, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=2, max_num_batched_tokens=128,
                                                  chunk_size=64, max_model_len=400),
                        use_cuda_graphs=False)
    return LLMEngine(ecfg, packed)


def test_long_generation_demotes_then_retrieve_promotes():
    eng = _engine()
    kb = KnowledgeBase()
    pol = eng.enable_segmented_cache(SegmentedCacheConfig.live(), context_limit=96,
                                     segment_tokens=16, knowledge_base=kb)
    rid = "r0"
    eng.add_request(rid, prompt_token_ids=list(range(5, 37)),
                    params=SamplingParams(temperature=0.0, max_tokens=150, ignore_eos=True))
    seq = eng.scheduler.running[0] if eng.scheduler.running else eng.scheduler.waiting[0]
    for _ in range(110):
        eng.step()
        if pol.stats["evicted_spans"] >= 2:
            break
    # pressure above 0.8 of the 96-token context evicted spans into the tier store
    assert pol.stats["evicted_spans"] >= 2 and pol.tiers.entries
    assert seq.num_computed_tokens < seq.num_tokens - 1          # KV shorter than the text
    assert seq.evicted > 0
    key = next(iter(pol.tiers.entries))
    entry = pol.tiers.entries[key]
    assert kb.peek_fact(key) is not None                          # a fact per demoted span
    assert any(p.startswith(f"[KB:{key}]") for p in pol.placeholders(seq))
    # the marker arrives in the token stream (here as injected context), next step promotes
    eng.inject_context(rid, text=f"<RETRIEVE:{key}>")
    eng.step()
    assert pol.stats["promoted"] == 1 and key not in pol.tiers.entries
    reg = pol.seg.registry(seq)
    back = [s for s in reg.spans() if s.tag == CacheTag.LONG_TERM_MEMORY and s.name == key]
    assert back and not back[0].evicted                        # the restored span is live
    assert back[0].end - back[0].start == len(entry.positions)
    assert back[0].end <= seq.num_computed_tokens
    # generation continues to the budget; the block manager stays consistent
    while eng.has_unfinished():
        eng.step()
    assert len(seq.output_token_ids) == 150
    assert eng.blocks.check_invariants()


def test_shadow_mode_only_logs():
    eng = _engine()
    pol = eng.enable_segmented_cache(SegmentedCacheConfig.observation(), context_limit=64,
                                     segment_tokens=16)
    seqs = eng.generate(prompt_token_ids=[list(range(3, 40))],
                        params=SamplingParams(temperature=0.0, max_tokens=60, ignore_eos=True))
    assert pol.seg.shadow_log and pol.stats["evicted_spans"] == 0
    assert seqs[0].evicted == 0 and not pol.tiers.entries
