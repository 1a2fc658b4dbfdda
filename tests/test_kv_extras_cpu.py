"""Eviction policies / voting, segmented spans, tiered storage and KIVI / R-KV on CPU."""
import math
import os
import tempfile

import pytest
import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.kv import kivi
from lightbulb_b200.kv.policy import (H2OScorePolicy, RecencyPolicy, SinkPolicy,
                                      VotingAggregator)
from lightbulb_b200.kv.spans import (CacheTag, SegmentedCacheConfig, SegmentedEvictionPolicy,
                                     SegmentedKV, SpanRegistry, PerTokenTracker)
from lightbulb_b200.kv.tiers import (BlockTierMover, FileDiskStore, MemoryDiskStore,
                                     decode_tensors, encode_tensors, find_retrieve_requests)
from lightbulb_b200.models.weights import pack_model, random_weights


def test_voting_keeps_plus_inf_and_vetoes():
    pos = {10: 0, 11: 1, 12: 2, 13: 3, 14: 4, 15: 5}
    mass = {10: 0.5, 11: 0.0, 12: 2.0, 13: 1.0, 14: 3.0, 15: 1.0}
    agg = (VotingAggregator().add_policy(RecencyPolicy(1), 1.0)
           .add_policy(H2OScorePolicy(mass, 1), 2.0).add_policy(SinkPolicy(1), 1.0))
    sc = dict(agg.compute_aggregated_scores(pos))
    assert sc[11] == math.inf                 # never attended -> first (reference dropped it)
    assert sc[10] == -math.inf and sc[15] == -math.inf   # sink and most recent: vetoed
    assert agg.select_eviction_candidate(pos) == 11
    order = agg.select_evictions(pos, 10)
    assert order[0] == 11 and 10 not in order and 15 not in order
    assert order.index(13) < order.index(14)  # less attention mass -> evicted earlier


def test_segmented_scoring_and_plan():
    reg = SpanRegistry()
    sp = reg.tag_range(0, 10, CacheTag.SYSTEM_PROMPT)
    u = reg.tag_range(10, 40, CacheTag.USER_INPUT)
    g = reg.tag_range(40, 80, CacheTag.MODEL_GENERATION)
    t = reg.tag_range(80, 100, CacheTag.TOOL_OUTPUT)
    pol = SegmentedEvictionPolicy(SegmentedCacheConfig.live())
    att = lambda p: 0.6 if 10 <= p < 40 else (0.3 if 80 <= p < 100 else 0.0)  # noqa: E731
    for _ in range(8):
        pol.update_scores(reg, att, 0.95)
    assert pol.smoothed_pressure > 0.8 and pol.pressure_decay_modifier() > 1.0
    rank = pol.rank_spans_for_eviction(reg)
    ids = [r[0] for r in rank]
    assert sp not in ids and ids[0] == g      # unattended generation first; system protected
    assert pol.scores[u].relevance > pol.scores[t].relevance   # 0.6^2*0.7 > 0.3^2*0.8
    assert pol.plan(reg, 30) == [g]
    reg.insert_context_at(40, 5)
    assert reg.get(g).start == 45 and reg.get(u).end == 40
    tr = PerTokenTracker(reg.get(t))
    tr.update(lambda p: 0.9 if p % 2 else 0.0)
    ev = tr.select_evictions(4, 1.0)
    assert all(p % 2 == 0 for p in ev) and len(ev) == 4


def _engine(blocks=64):
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=1, std=0.05)
    w = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=blocks, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=128,
                                                  chunk_size=128, max_model_len=512),
                        use_cuda_graphs=False)
    return LLMEngine(ecfg, packed)


def test_tensor_codec_and_file_store():
    t = {"a": torch.randn(3, 5).to(torch.bfloat16), "b": torch.arange(7, dtype=torch.int32)}
    blob = encode_tensors(t, {"x": 1})
    back, meta = decode_tensors(blob)
    assert meta == {"x": 1} and torch.equal(back["a"], t["a"]) and torch.equal(back["b"], t["b"])
    bad = bytearray(blob)
    bad[20] ^= 1
    with pytest.raises(ValueError):
        decode_tensors(bytes(bad))
    with tempfile.TemporaryDirectory() as d:
        st = FileDiskStore(d)
        st.put("k1", blob)
        assert FileDiskStore(d).get("k1") == blob   # index persists
        st.delete("k1")
        assert st.get("k1") is None and st.keys() == []


def test_tier_demote_evict_promote_roundtrip():
    eng = _engine()
    seq = eng.add_request("r", prompt_token_ids=list(range(3, 70)),
                          params=SamplingParams(temperature=0.0, max_tokens=50, ignore_eos=True))
    for _ in range(4):
        eng.step()
    bs = eng.kv.block_size
    table = eng.blocks.block_table(seq.seq_id)
    kvlen = seq.num_computed_tokens
    before = eng.kv.storage[:, :, [table[p // bs] for p in range(kvlen)], :,
                            [p % bs for p in range(kvlen)]].clone()
    mover = BlockTierMover(eng, disk=MemoryDiskStore(), max_ram_entries=1)
    k1 = mover.demote(seq, list(range(16, 32)), key="span-a")
    k2 = mover.demote(seq, list(range(32, 40)), key="span-b")   # pushes span-a to disk
    assert mover.entries["span-a"].tier == "disk" and mover.stats["to_disk"] == 1
    # evict positions 16..39 from the device with the spans machinery (no shadow mode)
    skv = SegmentedKV(eng, SegmentedCacheConfig.live())
    reg = skv.registry(seq)
    sid = reg.tag_range(16, 40, CacheTag.USER_INPUT)
    skv.evict_spans(seq, [sid])
    assert seq.num_computed_tokens == kvlen - 24 and seq.evicted == 24
    n = mover.promote(seq, k1) + mover.promote(seq, k2)
    assert n == 24 and seq.num_computed_tokens == kvlen and seq.evicted == 0
    table = eng.blocks.block_table(seq.seq_id)
    after = eng.kv.storage[:, :, [table[p // bs] for p in range(kvlen)], :,
                           [p % bs for p in range(kvlen)]]
    order = list(range(16)) + list(range(40, kvlen)) + list(range(16, 40))
    # rows are [tokens, layers, 2, Hkv, D] (advanced indices first)
    assert torch.equal(after, before[order])                 # same rows, restored at the end
    assert eng.blocks.check_invariants()
    assert find_retrieve_requests("see <RETRIEVE:span-a> and <RETRIEVE:x>") == ["span-a", "x"]


def test_span_eviction_keeps_engine_generating():
    eng = _engine()
    seq = eng.add_request("r", prompt_token_ids=list(range(3, 100)),
                          params=SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
    while seq.num_computed_tokens < 97:
        eng.step()
    skv = SegmentedKV(eng, SegmentedCacheConfig.live())
    reg = skv.registry(seq)
    reg.tag_range(0, 4, CacheTag.SYSTEM_PROMPT)
    victim = reg.tag_range(4, 60, CacheTag.USER_INPUT)
    reg.tag_range(60, 97, CacheTag.USER_INPUT)
    skv.evict_spans(seq, [victim])
    while eng.has_unfinished():
        eng.step()
    assert len(seq.output_token_ids) == 12 and eng.blocks.check_invariants()
    # same continuation as an engine that saw only the kept tokens at their true positions
    # is not expected token-for-token (eviction changes attention); generation must proceed.


@pytest.mark.parametrize("bits,tol", [(8, 0.03), (4, 0.3), (2, 1.3)])
def test_kivi_roundtrip_error_and_size(bits, tol):
    torch.manual_seed(0)
    k, v = torch.randn(100, 4, 128), torch.randn(100, 4, 128)
    c = kivi.KiviCompressor(bits, group=32, residual=16)
    b = c.compress(k, v)
    k2, v2 = c.decompress(b, torch.float32)
    assert torch.equal(k2[-16:], k[-16:])                      # full-precision residual
    assert (k2 - k).abs().max() < tol and (v2 - v).abs().max() < tol
    assert b.nbytes() < k.numel() * 4 * 2 * (bits / 32 + 0.2)


def test_rkv_and_lowrank_and_relationship():
    torch.manual_seed(1)
    base = torch.randn(1, 2, 16)
    keys = torch.cat([base.repeat(10, 1, 1) + 0.01 * torch.randn(10, 2, 16),
                      torch.randn(10, 2, 16)])
    imp = torch.ones(20)
    sel = kivi.rkv_select(keys, imp, 6, lam=1.0)
    assert sum(1 for i in sel if i < 10) <= 2                # near-duplicates are not all kept
    sel2 = kivi.rkv_select(keys, imp, 5, protect_first=1, protect_last=2)
    assert 0 in sel2 and 18 in sel2 and 19 in sel2
    x = torch.randn(50, 2, 8) @ torch.randn(8, 8)            # rank <= 8 per head
    lr = kivi.lowrank_compress(x, 8)
    assert torch.allclose(kivi.lowrank_decompress(lr), x, atol=1e-4)
    imp = torch.zeros(40)
    imp[20] = 1.0
    rs = kivi.relationship_select(torch.randn(40, 1, 4), imp, 5)
    assert 20 in rs and all(abs(i - 20) <= 8 for i in rs)
