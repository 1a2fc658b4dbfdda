"""GPU paths of speculative decoding and KV compression (kernels vs CPU restatements)."""
import pytest
import torch

from lightbulb_b200 import ops
from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.models.reference import ReferenceLlama
from lightbulb_b200.models.weights import pack_model, random_weights

pytestmark = pytest.mark.gpu


def _cfg():
    return get_preset("tiny-test", hidden_size=512, intermediate_size=1024, num_heads=4,
                      num_kv_heads=1, head_dim=128, vocab_size=1024)


def _engine(w, cfg, **cache):
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cuda")
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=256, block_size=16, **cache),
                        scheduler=SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=256,
                                                  chunk_size=128, max_model_len=1024))
    return LLMEngine(ecfg, packed), packed


@pytest.mark.parametrize("hq,hkv,L", [(8, 2, [5, 40, 130]), (32, 8, [300, 700, 17]),
                                      (16, 16, [1030, 1])])
def test_h2o_accumulate_matches_cpu(hq, hkv, L):
    from lightbulb_b200.kv.compression import H2OPolicy
    torch.manual_seed(0)
    bs = 16
    nper = max((l + bs - 1) // bs for l in L)
    nblocks = sum((l + bs - 1) // bs for l in L) + 4
    kc = torch.randn(nblocks, hkv, bs, 128).to(torch.bfloat16)
    bt = torch.zeros(len(L), nper + 1, dtype=torch.int32)
    perm = torch.randperm(nblocks)
    o = 0
    for i, l in enumerate(L):
        n = (l + bs - 1) // bs
        bt[i, :n] = perm[o:o + n]
        o += n
    q = torch.randn(len(L), hq, 128).to(torch.bfloat16)
    sl = torch.tensor(L, dtype=torch.int32)

    class E:  # minimal engine stub for the policy
        class kv:
            num_blocks, block_size = nblocks, bs
            storage = torch.zeros(1, device="cpu")

        class model:
            h2o = None

    cpu = H2OPolicy(E)
    cpu.score.fill_(0.5)
    cpu.accumulate(q, kc, bt, sl)
    E.kv.storage = torch.zeros(1, device="cuda")
    gpu = H2OPolicy(E)
    gpu.score.fill_(0.5)
    gpu.accumulate(q.cuda(), kc.cuda(), bt.cuda(), sl.cuda())
    torch.cuda.synchronize()
    assert torch.allclose(gpu.score.cpu(), cpu.score, atol=2e-3, rtol=1e-3)


def test_kv_compact_kernel():
    st = torch.randn(2, 2, 8, 2, 16, 128, device="cuda").to(torch.bfloat16)
    src = torch.tensor([3, 17, 40, 100], dtype=torch.int32, device="cuda")
    dst = torch.tensor([112, 113, 114, 127], dtype=torch.int32, device="cuda")
    ref = st.clone()
    ops._need_c().kv_compact(st, src, dst, None)
    torch.cuda.synchronize()
    for s_, d_ in zip(src.tolist(), dst.tolist()):
        assert torch.equal(st[:, :, d_ // 16, :, d_ % 16], ref[:, :, s_ // 16, :, s_ % 16])


def test_speculative_on_gpu_is_oracle_consistent():
    cfg = _cfg()
    w = random_weights(cfg, seed=3, std=0.05)
    w = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    eng, packed = _engine(w, cfg)
    spec = eng.attach_draft(packed, cfg, k=4)
    prompts = [list(range(3, 60)), [7, 8, 9]]
    seqs = eng.generate(prompt_token_ids=prompts,
                        params=SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
    ops.check_errors()
    ref = ReferenceLlama(cfg, w)
    for p, s in zip(prompts, seqs):
        ref.reset()
        lg = ref.forward(torch.tensor(p + s.output_token_ids[:-1]))[len(p) - 1:]
        for i, t in enumerate(s.output_token_ids):
            v, ix = torch.topk(lg[i], 2)
            assert int(ix[0]) == t or float(v[0] - v[1]) < 0.05
    assert spec.stats.acceptance_rate() > 0.8


def test_h2o_engine_on_gpu():
    cfg = _cfg()
    w = random_weights(cfg, seed=4, std=0.05)
    eng, _ = _engine(w, cfg, h2o_budget=64, sink_tokens=4)
    eng.kv_policy.slack, eng.kv_policy.recent = 16, 8
    s = eng.generate(prompt_token_ids=[list(range(3, 300))],
                     params=SamplingParams(temperature=0.0, max_tokens=48, ignore_eos=True))[0]
    ops.check_errors()
    assert len(s.output_token_ids) == 48 and s.evicted > 0
    assert eng.kv_policy.compactions >= 1 and eng.blocks.check_invariants()
