"""Offline tools (norm tweaking, pruning, LoRA, hub, capabilities) and the MoE router, on CPU."""
import json
import os
import tempfile

import numpy as np
import pytest
import torch

from lightbulb_b200.config import get_preset
from lightbulb_b200.extras.moe import MoERouter, RouterConfig, combine
from lightbulb_b200.models.reference import ReferenceLlama
from lightbulb_b200.models.weights import random_weights
from lightbulb_b200.tools import capabilities, hub, lora, norm_tweaking, pruning


def _model():
    cfg = get_preset("tiny-test", num_layers=2)
    return cfg, random_weights(cfg, seed=4, std=0.05)


def _quantize_like(w):
    """Crude 3-bit per-row rounding of every projection (a stand-in for weight quantisation)."""
    out = dict(w)
    for k, v in w.items():
        if k.endswith("proj.weight"):
            s = v.abs().amax(1, keepdim=True) / 3
            out[k] = torch.round(v / s).clamp(-3, 3) * s
    return out


def test_norm_tweaking_reduces_output_error():
    cfg, w = _model()
    wq = _quantize_like(w)
    calib = [torch.randint(0, cfg.vocab_size, (24,), generator=torch.Generator().manual_seed(i))
             for i in range(3)]
    gains = norm_tweaking.tweak(cfg, w, wq, calib)
    assert len(gains) == 2 * cfg.num_layers
    wt = norm_tweaking.apply(wq, gains)
    test = torch.randint(0, cfg.vocab_size, (32,), generator=torch.Generator().manual_seed(9))
    ref = ReferenceLlama(cfg, w).forward(test)
    e_q = (ReferenceLlama(cfg, wq).forward(test) - ref).norm()
    e_t = (ReferenceLlama(cfg, wt).forward(test) - ref).norm()
    assert e_t < e_q
    st = norm_tweaking.collect_statistics(cfg, w, wq, calib)
    assert len(st) == 2 * cfg.num_layers and all(s.shift_magnitude() >= 0 for s in st)


def test_pruning_methods_and_manifest():
    cfg, w = _model()
    calib = [torch.randint(0, cfg.vocab_size, (16,), generator=torch.Generator().manual_seed(1))]
    pw, man = pruning.prune(cfg, w, "wanda", 0.5, calib)
    W = pw["model.layers.0.mlp.up_proj.weight"]
    assert abs((W == 0).float().mean().item() - 0.5) < 0.02
    assert all(abs(e.sparsity - 0.5) < 0.02 for e in man.entries)
    nm, _ = pruning.prune(cfg, w, "nm24", calib=calib)
    g = nm["model.layers.1.self_attn.q_proj.weight"].reshape(-1, 4)
    assert ((g != 0).sum(1) <= 2).all()
    mg, m2 = pruning.prune(cfg, w, "magnitude", 0.25, skip_last=1)
    assert len(m2.entries) == 7 and torch.equal(mg["model.layers.1.mlp.down_proj.weight"],
                                                w["model.layers.1.mlp.down_proj.weight"])
    assert pruning.PruneManifest.from_json(man.to_json()).entries[3].name == man.entries[3].name
    # wanda keeps weights on high-activation input channels
    sc = pruning.wanda_scores(torch.ones(2, 4), torch.tensor([1.0, 5.0, 2.0, 0.1]))
    assert pruning.mask_unstructured(sc, 0.5)[0].tolist() == [False, True, True, False]


def test_pruning_on_gguf_q8_tensor():
    from lightbulb_b200.formats import gguf as G
    x = torch.randn(4, 64)
    raw = np.frombuffer(G.quantize(x, G.GGML_Q8_0), dtype=np.uint8).copy()
    mask = torch.rand(4, 64) > 0.5
    out = np.frombuffer(pruning.apply_to_gguf(raw, G.GGML_Q8_0, 4, 64, mask), dtype=np.uint8)
    from lightbulb_b200 import _native as N
    back = N.dequantize(G.GGML_Q8_0, torch.from_numpy(out.copy()), 256).reshape(4, 64)
    assert (back[~mask] == 0).all() and torch.allclose(back[mask], x[mask], atol=0.05)


def test_lora_peft_load_merge_unmerge():
    cfg, w = _model()
    r, alpha = 4, 8.0
    name = "model.layers.0.self_attn.q_proj.weight"
    out_f, in_f = w[name].shape
    A, B = torch.randn(r, in_f) * 0.1, torch.randn(out_f, r) * 0.1
    with tempfile.TemporaryDirectory() as d:
        from safetensors.torch import save_file
        save_file({"base_model.model.model.layers.0.self_attn.q_proj.lora_A.weight": A,
                   "base_model.model.model.layers.0.self_attn.q_proj.lora_B.weight": B},
                  os.path.join(d, "adapter_model.safetensors"))
        with open(os.path.join(d, "adapter_config.json"), "w") as f:
            json.dump({"r": r, "lora_alpha": alpha, "target_modules": ["q_proj"]}, f)
        ad = lora.load_adapter(d)
    assert list(ad.pairs) == [name] and ad.pairs[name].scale == alpha / r
    m = lora.merge(w, ad)
    assert torch.allclose(m[name], w[name] + (alpha / r) * B @ A, atol=1e-6)
    back = lora.merge(m, ad, unmerge=True)
    assert torch.allclose(back[name], w[name], atol=1e-6)
    bad = lora.from_tensors({"model.layers.0.self_attn.q_proj.lora_A": torch.randn(r, 3),
                             "model.layers.0.self_attn.q_proj.lora_B": torch.randn(out_f, r)})
    with pytest.raises(ValueError):
        lora.merge(w, bad)


def test_hub_resolution_offline():
    with tempfile.TemporaryDirectory() as root:
        snap = os.path.join(root, "models--org--tiny", "snapshots", "abc123")
        os.makedirs(snap)
        os.makedirs(os.path.join(root, "models--org--tiny", "refs"))
        with open(os.path.join(root, "models--org--tiny", "refs", "main"), "w") as f:
            f.write("abc123")
        assert hub.resolve("org/tiny", roots=[root]) == snap
        assert hub.resolve("org/tiny@abc123", roots=[root]) == snap
        with pytest.raises(FileNotFoundError):
            hub.resolve("org/other", roots=[root])
        assert hub.resolve(root) == root
    with pytest.raises(ValueError):
        hub.ModelSource.parse("not-a-hub-id")


def test_capabilities():
    names = ["model.embed_tokens.weight", "lm_head.weight", "vision_tower.blocks.0.weight",
             "model.layers.0.block_sparse_moe.experts.0.w1.weight"]
    caps = capabilities.detect(names, chat_template="{% if tools %}...{% endif %}")
    assert caps == {"text", "vision", "function_calling", "mixture_of_experts"}
    assert capabilities.detect(["token_embd.weight", "output.weight"]) == {"text"}


@pytest.mark.parametrize("policy", ["token_drop", "expanded_drop", "reroute", "unlimited"])
def test_moe_router_policies(policy):
    torch.manual_seed(0)
    T, E = 64, 4
    logits = torch.randn(T, E)
    logits[:, 0] += 3.0                                  # hot expert 0
    r = MoERouter(RouterConfig(E, top_k=2, capacity_factor=1.0, policy=policy,
                               expansion_factor=4))
    res = r.route(logits)
    cap = r.capacity(T)
    if policy == "unlimited":
        assert res.num_dropped == 0
    else:
        assert (res.expert_loads <= cap).all()
    if policy == "token_drop":
        assert cap == 16 and res.num_dropped > 0
        # earlier tokens win: the first 16 tokens choosing expert 0 keep it
        first0 = [t for t in range(T) if 0 in res.expert_ids[t].tolist()][:16]
        assert all(not res.dropped[t][(res.expert_ids[t] == 0).nonzero()[0, 0]] for t in first0)
    if policy == "reroute":
        # with room for every assignment (capacity factor 2), rerouting recovers all drops
        full = MoERouter(RouterConfig(E, 2, 2.0, policy="reroute")).route(logits)
        assert full.num_dropped == 0 < MoERouter(RouterConfig(E, 2, 2.0)).route(logits).num_dropped
    kept = ~res.dropped
    assert torch.allclose(res.weights.sum(-1)[kept.any(-1)], torch.ones(int(kept.any(-1).sum())))
    assert res.aux_loss > 1.0                            # imbalanced routing
    outs = {e: torch.full((len(ts), 3), float(e)) for e, ts in res.expert_batches().items()}
    y = combine(outs, res, T, 3)
    assert y.shape == (T, 3)
