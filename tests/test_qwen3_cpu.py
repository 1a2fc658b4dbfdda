"""Qwen3 architecture (per-head q/k RMSNorm before RoPE, reference
src/model/awq_qwen3.rs:183-301) on the CPU path of the engine vs the fp32 oracle."""
import json

import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.models.reference import ReferenceLlama
from lightbulb_b200.models.weights import pack_model, random_weights, weight_shapes
from test_engine_cpu import assert_greedy_consistent


def _qwen3(**kw):
    cfg = get_preset("qwen3-tiny-test", **kw)
    w = random_weights(cfg, seed=4, std=0.05)
    w = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    return cfg, w


def test_qwen3_weights_and_config_roundtrip():
    cfg, w = _qwen3()
    assert cfg.qk_norm and "model.layers.0.self_attn.q_norm.weight" in weight_shapes(cfg)
    d = cfg.to_hf_dict()
    assert d["model_type"] == "qwen3" and d["architectures"] == ["Qwen3ForCausalLM"]
    back = ModelConfig.from_hf_dict(json.loads(json.dumps(d)))
    assert back.qk_norm and back.head_dim == 128
    assert not ModelConfig.from_hf_dict(get_preset("tiny-test").to_hf_dict()).qk_norm
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    assert packed["layers"][0]["q_norm"].shape == (128,)


def test_qwen3_norm_changes_the_model():
    # the per-head norms are live: scaling k_norm changes the logits
    cfg, w = _qwen3()
    ref = ReferenceLlama(cfg, w)
    a = ref.forward(torch.tensor([3, 4, 5, 6]))
    w2 = dict(w)
    w2["model.layers.0.self_attn.k_norm.weight"] = w["model.layers.0.self_attn.k_norm.weight"] * 3
    ref2 = ReferenceLlama(cfg, w2)
    b = ref2.forward(torch.tensor([3, 4, 5, 6]))
    assert (a - b).abs().max() > 1e-3


def test_qwen3_engine_matches_oracle():
    cfg, w = _qwen3()
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
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
