"""Architecture detection and tensor-name mapping (reference src/pruning/name_mapping.rs)."""
from lightbulb_b200.formats.name_map import (GPT, LLAMA, MISTRAL, UNKNOWN, TensorNameMapper,
                                             detect_architecture, parse_abstract, translate)
from lightbulb_b200.tools.pruning import PruneEntry, PruneManifest, map_manifest


def test_detects_families_in_reference_order():
    assert detect_architecture(["blk.0.attn_q.weight", "blk.1.ffn_gate.weight"]) == LLAMA
    assert detect_architecture(["h.0.attn.c_attn.weight", "h.0.mlp.c_fc.weight"]) == GPT
    assert detect_architecture(["transformer.h.3.attn.c_attn.weight"]) == GPT
    assert detect_architecture(["model.layers.0.self_attn.q_proj.weight"]) == MISTRAL
    assert detect_architecture(["token_embd.weight"]) == UNKNOWN
    # GGUF names win when both appear
    assert detect_architecture(["model.layers.0.self_attn.q_proj.weight",
                                "blk.0.attn_q.weight"]) == LLAMA


def test_llama_mapping_and_layers():
    names = ["blk.0.attn_q.weight", "blk.0.attn_k.weight", "blk.0.ffn_gate.weight",
             "blk.1.attn_q.weight", "blk.1.attn_q_norm.weight", "output.weight"]
    m = TensorNameMapper.from_tensor_names(names)
    assert m.architecture == LLAMA and m.layer_indices == [0, 1]
    assert m.map_name("layer_0") == "blk.0.attn_q.weight"
    assert m.map_name("layer_0.attention.key") == "blk.0.attn_k.weight"
    assert m.map_name("layer_0.attn.k") == "blk.0.attn_k.weight"
    assert m.map_name("layer_1.attention.q_norm") == "blk.1.attn_q_norm.weight"
    assert m.map_name("layer_0.ffn.down") is None          # absent in this checkpoint
    assert m.map_name("block_0") is None and parse_abstract("layer_x") is None
    assert [c for c, _ in m.map_layer(0)] == ["attn_q", "attn_k", "ffn_gate"]
    assert m.get_layer_tensors(0) == sorted(["blk.0.attn_q.weight", "blk.0.attn_k.weight",
                                             "blk.0.ffn_gate.weight"])


def test_gpt_fused_qkv_and_mistral():
    g = TensorNameMapper(["h.0.attn.c_attn.weight", "h.0.attn.c_proj.weight",
                          "h.0.mlp.c_fc.weight", "h.0.mlp.c_proj.weight"])
    assert g.architecture == GPT
    assert g.map_name("layer_0.attention.query") == g.map_name("layer_0.attention.value") == \
        "h.0.attn.c_attn.weight"
    assert g.map_name("layer_0.ffn.up") == "h.0.mlp.c_fc.weight"
    assert g.map_name("layer_0.ffn.gate") is None          # GPT MLP has no gate
    hf = TensorNameMapper(["model.layers.2.mlp.down_proj.weight",
                           "model.layers.2.self_attn.o_proj.weight"])
    assert hf.architecture == MISTRAL and hf.layer_indices == [2]
    assert hf.map_name("layer_2.attention.output") == "model.layers.2.self_attn.o_proj.weight"
    assert translate("model.layers.2.mlp.down_proj.weight", hf, LLAMA) == "blk.2.ffn_down.weight"


def test_prune_manifest_maps_onto_gguf_names():
    man = PruneManifest([PruneEntry("model.layers.0.self_attn.q_proj.weight", "wanda", 0.5),
                         PruneEntry("model.layers.0.mlp.up_proj.weight", "wanda", 0.5),
                         PruneEntry("model.layers.9.mlp.up_proj.weight", "wanda", 0.5)])
    gguf = ["blk.0.attn_q.weight", "blk.0.ffn_up.weight", "token_embd.weight"]
    assert map_manifest(man, gguf) == {
        "model.layers.0.self_attn.q_proj.weight": "blk.0.attn_q.weight",
        "model.layers.0.mlp.up_proj.weight": "blk.0.ffn_up.weight"}
