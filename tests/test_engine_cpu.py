"""Engine + scheduler + block manager + model plumbing on CPU vs the fp32 oracle."""
import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.models.reference import ReferenceLlama, greedy_generate
from lightbulb_b200.models.weights import pack_model, random_weights


def assert_greedy_consistent(ref, prompt, out, tol=0.02):
    """Teacher-forced check: each emitted token is the oracle argmax along the emitted
    trajectory, unless the oracle's top-2 logits are within ``tol`` (bf16 near-tie)."""
    ref.reset()
    lg = ref.forward(torch.tensor(prompt + out[:-1]))[len(prompt) - 1:]
    for i, t in enumerate(out):
        v, ix = torch.topk(lg[i], 2)
        assert int(ix[0]) == t or (v[0] - v[1]) < tol, (i, t, ix.tolist(), (v[0] - v[1]).item())


def _engine(num_blocks=64, budget=64, chunk=32, max_seqs=8, prefix=True):
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=1, std=0.05)
    w = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=cfg,
                        cache=CacheConfig(num_blocks=num_blocks, block_size=16,
                                          enable_prefix_caching=prefix),
                        scheduler=SchedulerConfig(max_num_seqs=max_seqs,
                                                  max_num_batched_tokens=budget,
                                                  chunk_size=chunk, max_model_len=256),
                        use_cuda_graphs=False)
    return cfg, w, LLMEngine(ecfg, packed)


def test_batched_chunked_prefill_matches_oracle():
    cfg, w, eng = _engine()
    ref = ReferenceLlama(cfg, w)
    prompts = [list(range(5, 41)), [100, 200, 300], [7] * 50, [1]]
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    seqs = eng.generate(prompt_token_ids=prompts, params=sp)
    for p, s in zip(prompts, seqs):
        assert_greedy_consistent(ref, p, s.output_token_ids)
        assert s.finish_reason == "length" and len(s.output_token_ids) == 10
    assert eng.blocks.check_invariants()
    assert eng.blocks.num_free_blocks() == 64


def test_prefix_cache_hit_same_tokens():
    cfg, w, eng = _engine()
    shared = list(range(10, 58))  # 3 full blocks
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    a = eng.generate(prompt_token_ids=[shared + [1, 2, 3]], params=sp)[0]
    b = eng.generate(prompt_token_ids=[shared + [1, 2, 3]], params=sp)[0]
    assert b.num_cached_prefix >= 48
    assert a.output_token_ids == b.output_token_ids
    assert eng.blocks.check_invariants()


def test_preemption_under_block_pressure():
    cfg, w, eng = _engine(num_blocks=12, budget=64, chunk=64)
    ref = ReferenceLlama(cfg, w)
    prompts = [[3 + i] * 40 for i in range(4)]
    sp = SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True)
    seqs = eng.generate(prompt_token_ids=prompts, params=sp)
    for p, s in zip(prompts, seqs):
        assert len(s.output_token_ids) == 20
        assert_greedy_consistent(ref, p, s.output_token_ids)
    assert eng.scheduler.num_preemptions > 0
    assert eng.blocks.check_invariants()


def test_eos_and_budget_truncation():
    cfg, w, eng = _engine()
    seq = eng.add_request("x", prompt_token_ids=list(range(3, 250)),
                          params=SamplingParams(temperature=0.0, max_tokens=100))
    assert seq.truncated and seq.max_new_tokens == 256 - 247
    while eng.has_unfinished():
        eng.step()
    assert seq.finish_reason in ("length", "stop")
    assert len(seq.output_token_ids) <= 9


import pytest  # noqa: E402


@pytest.mark.parametrize("hidden,heads,kv", [(256, 4, 4), (384, 4, 2), (512, 4, 4)])
def test_padded_head_widths_match_oracle(hidden, heads, kv):
    # head_dim 64 (TinyLlama / Llama-3.2-1B), 96 (Phi-3-mini) and 128: heads are zero-padded
    # to the 128-wide device layout; greedy output must follow the unpadded fp32 oracle
    cfg = get_preset("tiny-test", hidden_size=hidden, num_heads=heads, num_kv_heads=kv,
                     head_dim=hidden // heads)
    assert cfg.head_dim == hidden // heads and cfg.head_dim_padded == 128
    w = random_weights(cfg, seed=3, std=0.05)
    w = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    assert packed["layers"][0]["qkv"].shape[0] == (heads + 2 * kv) * 128
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=32, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                  chunk_size=32, max_model_len=256),
                        use_cuda_graphs=False)
    eng = LLMEngine(ecfg, packed)
    ref = ReferenceLlama(cfg, w)
    prompts = [list(range(5, 45)), [9, 8, 7]]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    for p, s in zip(prompts, eng.generate(prompt_token_ids=prompts, params=sp)):
        assert_greedy_consistent(ref, p, s.output_token_ids)


def test_tool_call_pause_and_inject_resumes_in_place():
    from lightbulb_b200.engine.sequence import SeqStatus
    cfg, w, eng = _engine()
    ref = ReferenceLlama(cfg, w)

    class AfterThreeChars:   # stands in for a <tool_call>...</tool_call> match
        def __init__(self):
            self.fired = False

        def find(self, text):
            if not self.fired and len(text) >= 3:
                self.fired = True
                return {"raw": "lookup", "call": {"name": "lookup"}}
            return None

    eng.enable_tool_calls(AfterThreeChars())
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True, detokenize=True)
    seq = eng.add_request("t", prompt_token_ids=list(range(5, 40)), params=sp)
    outs = []
    while eng.has_runnable():
        outs += eng.step()
    assert seq.status == SeqStatus.AWAITING_TOOL and seq.pending_tool_call["raw"] == "lookup"
    assert any(o.tool_call is not None for o in outs)
    n_before = len(seq.output_token_ids)
    assert 0 < n_before < 10 and eng.step() == []          # paused: nothing to run
    eng.inject_tool_result("t", token_ids=[300, 301, 302, 303])
    while eng.has_unfinished():
        eng.step()
    assert len(seq.output_token_ids) == 10 and seq.injected_tokens == 4
    toks = seq.all_token_ids
    assert toks[35 + n_before:35 + n_before + 4] == [300, 301, 302, 303]
    # every output after the injection follows the oracle on the full token list
    ref.reset()
    lg = ref.forward(torch.tensor(toks[:-1]))
    for j in range(35 + n_before + 4, len(toks)):
        v, ix = torch.topk(lg[j - 1], 2)
        assert int(ix[0]) == toks[j] or (v[0] - v[1]) < 0.02
    assert eng.blocks.check_invariants()
