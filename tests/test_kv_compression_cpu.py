"""H2O and StreamingLLM KV compression on CPU: bounded KV, true positions, invariants."""
import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.models.weights import pack_model, random_weights


def _engine(**cache):
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=1, std=0.05)
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=256, block_size=16, **cache),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=256,
                                                  chunk_size=128, max_model_len=1024),
                        use_cuda_graphs=False)
    return LLMEngine(ecfg, packed)


def test_h2o_bounds_kv_and_keeps_generating():
    eng = _engine(h2o_budget=64, sink_tokens=4)
    pol = eng.kv_policy
    pol.slack, pol.recent = 16, 8
    prompt = list(range(3, 203))  # 200 tokens > 64 + 4
    sp = SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True)
    seq = eng.generate(prompt_token_ids=[prompt], params=sp)[0]
    assert len(seq.output_token_ids) == 40
    assert pol.compactions >= 1
    assert seq.evicted > 0
    assert eng.blocks.check_invariants()
    assert eng.blocks.num_free_blocks() == eng.blocks.num_blocks


def test_h2o_keeps_sinks_and_recent_tokens():
    eng = _engine(h2o_budget=48, sink_tokens=4)
    pol = eng.kv_policy
    pol.slack, pol.recent = 8, 8
    seq = eng.add_request("a", prompt_token_ids=list(range(3, 123)),
                          params=SamplingParams(temperature=0.0, max_tokens=100, ignore_eos=True))
    while seq.evicted == 0:
        eng.step()
    bm = eng.blocks
    assert seq.num_computed_tokens == 4 + 48
    assert bm.num_tokens(seq.seq_id) == seq.num_computed_tokens
    # positions stay true: next token's RoPE position = KV index + evicted
    assert seq.num_computed_tokens + seq.evicted == seq.num_tokens - 1
    eng.abort("a")


def test_streaming_drops_middle_blocks():
    eng = _engine(streaming_window=32, sink_tokens=4)
    seq = eng.generate(prompt_token_ids=[list(range(3, 160))],
                       params=SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True))[0]
    assert len(seq.output_token_ids) == 30
    assert eng.kv_policy.evictions >= 1 and seq.evicted % 16 == 0 and seq.evicted > 0
    assert eng.blocks.check_invariants()
