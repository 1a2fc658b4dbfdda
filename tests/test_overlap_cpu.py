"""Overlapped decode (step N+1 launched before step N's ids are read back) must emit exactly
the tokens of the synchronous engine: same ids, same lengths, same finish reasons, and a
consistent block manager afterwards."""
import random

import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.engine.sequence import PENDING_TOKEN
from lightbulb_b200.models.weights import pack_model, random_weights


def _engine(overlap, num_blocks=96, max_seqs=8, budget=64):
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=3, std=0.05)
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=cfg,
                        cache=CacheConfig(num_blocks=num_blocks, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=max_seqs,
                                                  max_num_batched_tokens=budget,
                                                  chunk_size=32, max_model_len=256),
                        use_cuda_graphs=False, overlap_decode=overlap)
    return LLMEngine(ecfg, packed)


def _run(overlap, prompts, params, late=(), num_blocks=96):
    eng = _engine(overlap, num_blocks=num_blocks)
    seqs = [eng.add_request(f"r{i}", prompt_token_ids=p, params=sp)
            for i, (p, sp) in enumerate(zip(prompts, params))]
    steps = 0
    overlapped = 0
    late = list(late)
    while eng.has_unfinished():
        if late and steps == 6:
            p, sp = late.pop()
            seqs.append(eng.add_request(f"late{steps}", prompt_token_ids=p, params=sp))
        outs = eng.step()
        overlapped += eng._pending is not None
        for o in outs:
            assert o.new_token_ids[0] != PENDING_TOKEN
        steps += 1
        assert steps < 500
    eng.blocks.check_invariants()
    assert eng.blocks.num_free_blocks() == num_blocks
    return [(s.output_token_ids, s.finish_reason) for s in seqs], overlapped


def test_overlap_matches_sync_mixed_lengths_and_arrivals():
    rng = random.Random(0)
    prompts = [[rng.randrange(3, 500) for _ in range(rng.randint(3, 60))] for _ in range(6)]
    params = [SamplingParams(temperature=0.0, max_tokens=m, ignore_eos=True)
              for m in (1, 2, 7, 20, 33, 12)]
    late = [([5, 6, 7, 8], SamplingParams(temperature=0.0, max_tokens=9, ignore_eos=True))]
    a, n_a = _run(False, prompts, params, late)
    b, n_b = _run(True, prompts, params, late)
    assert n_a == 0 and n_b > 0
    assert a == b
    for (out, reason), sp in zip(b, params + [late[0][1]]):
        assert len(out) == sp.max_tokens and reason == "length"


def test_overlap_matches_sync_with_eos_and_sampling():
    rng = random.Random(1)
    prompts = [[rng.randrange(3, 500) for _ in range(rng.randint(3, 40))] for _ in range(5)]
    # EOS = the tiny preset's eos id; sampled rows use per-request seeds (deterministic)
    params = [SamplingParams(temperature=0.0, max_tokens=40),
              SamplingParams(temperature=0.8, top_k=20, seed=5, max_tokens=30),
              SamplingParams(temperature=1.0, top_p=0.9, seed=9, max_tokens=25),
              SamplingParams(temperature=0.0, max_tokens=40, stop_token_ids=[]),
              SamplingParams(temperature=0.7, seed=1, max_tokens=35)]
    a, _ = _run(False, prompts, params)
    b, n_b = _run(True, prompts, params)
    assert n_b > 0
    assert a == b


def test_overlap_drains_under_block_pressure():
    # few blocks: overlap must step aside whenever a decode step could preempt
    prompts = [[i + 3] * 30 for i in range(6)]
    params = [SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True)] * 6
    a, _ = _run(False, prompts, params, num_blocks=16)
    b, _ = _run(True, prompts, params, num_blocks=16)
    assert a == b


def test_overlap_stop_token_mid_stream():
    # stop on a token the greedy stream is known to emit: the overlapped engine launched one
    # more step for that sequence, whose id must be dropped
    prompts = [[11, 12, 13, 14], [40, 41], [99] * 20]
    base = [SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True)] * 3
    ref, _ = _run(False, prompts, base)
    stop = ref[0][0][5]
    params = [SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=False,
                             stop_token_ids=[stop])] * 3
    a, _ = _run(False, prompts, params)
    b, n_b = _run(True, prompts, params)
    assert n_b > 0 and a == b
    assert a[0][1] == "stop" and a[0][0][-1] == stop and len(a[0][0]) <= 6


def test_overlap_abort_mid_stream_and_stop_strings():
    # abort a request while its newest id is still pending, and finish another on a text stop
    # string: the other requests must match the synchronous engine and every block be freed
    prompts = [[21, 22, 23], [31, 32, 33, 34], [41] * 12]
    sp = [SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True) for _ in prompts]
    ref, _ = _run(False, prompts, sp)
    stop_text = None

    def go(overlap):
        eng = _engine(overlap)
        seqs = [eng.add_request(f"r{i}", prompt_token_ids=p, params=s)
                for i, (p, s) in enumerate(zip(prompts, sp))]
        for _ in range(10):
            eng.step()
        eng.abort("r1")
        while eng.has_unfinished():
            eng.step()
        eng.blocks.check_invariants()
        assert eng.blocks.num_free_blocks() == 96
        return [(s.output_token_ids, s.finish_reason) for s in seqs]

    a, b = go(False), go(True)
    assert a[0] == b[0] == ref[0] and a[2] == b[2] == ref[2]
    assert a[1][1] == b[1][1] == "abort"
    assert PENDING_TOKEN not in b[1][0] and b[1][0] == ref[1][0][:len(b[1][0])]

    # stop string: take a piece of the greedy text of request 0 and stop on it
    eng = _engine(False)
    s0 = eng.add_request("t", prompt_token_ids=prompts[0], params=SamplingParams(
        temperature=0.0, max_tokens=40, ignore_eos=True))
    while eng.has_unfinished():
        eng.step()
    text = s0.output_text
    if len(text) >= 8:
        stop_text = text[4:8]
        outs = []
        for overlap in (False, True):
            e = _engine(overlap)
            s = e.add_request("t", prompt_token_ids=prompts[0], params=SamplingParams(
                temperature=0.0, max_tokens=40, ignore_eos=True, stop=[stop_text]))
            while e.has_unfinished():
                e.step()
            outs.append((s.output_token_ids, s.output_text, s.finish_reason))
            e.blocks.check_invariants()
        assert outs[0] == outs[1] and outs[0][2] == "stop"
