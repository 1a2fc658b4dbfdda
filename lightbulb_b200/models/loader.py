"""Checkpoint loading: safetensors directory, GGUF file, AWQ int4 directory.

Reference entry points: ``load_local_llama`` (``src/loaders/mod.rs:57-126``),
``load_gguf_llama`` (``:127-284``), ``load_awq_llama`` (``:285-395``) and the model
manager's GGUF metadata handling (``src/model/parallel_model_manager.rs:226-502``).

Returns ``(ModelConfig, packed device weights, tokenizer)``.  Quantized linears keep their
quantized form on the device (``packed["layers"][i]["quant"]``) when the int4 / GGUF GEMM
kernels are built for it; otherwise (and always on CPU) they are dequantized to bf16.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Optional, Tuple

import torch

from ..config import ModelConfig
from ..engine.tokenizer import BaseTokenizer, ByteTokenizer, GGUFTokenizer, load_tokenizer
from .weights import load_safetensors_dir, pack_model

PROJ = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
        "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def detect_format(path: str) -> str:
    if os.path.isfile(path) and path.endswith(".gguf"):
        return "gguf"
    cfg = os.path.join(path, "config.json")
    if os.path.isdir(path) and os.path.exists(cfg):
        with open(cfg) as f:
            d = json.load(f)
        q = d.get("quantization_config") or {}
        if q.get("quant_method", "awq" if "group_size" in q else "") == "awq":
            return "awq"
        return "safetensors"
    if os.path.isdir(path):
        ggufs = sorted(f for f in os.listdir(path) if f.endswith(".gguf"))
        if ggufs:
            return "gguf"
    raise FileNotFoundError(f"no checkpoint (config.json + *.safetensors, or *.gguf) at {path}")


def load_hf_weights(path: str) -> Tuple[ModelConfig, Dict[str, torch.Tensor]]:
    with open(os.path.join(path, "config.json")) as f:
        d = json.load(f)
    return ModelConfig.from_hf_dict(d), load_safetensors_dir(path)


def load_gguf_weights(path: str):
    from ..formats.gguf import GGUFReader, config_from_gguf, gguf_name_to_hf
    if os.path.isdir(path):
        path = os.path.join(path, sorted(f for f in os.listdir(path) if f.endswith(".gguf"))[0])
    r = GGUFReader(path)
    cfg = config_from_gguf(r.metadata)
    w = {}
    for name in r.tensors:
        hf = gguf_name_to_hf(name)
        if hf is not None:
            w[hf] = r.dequantize(name)
    if "lm_head.weight" not in w:
        cfg.tie_word_embeddings = True
    tok = GGUFTokenizer(r.metadata) if r.metadata.get("tokenizer.ggml.tokens") else None
    return cfg, w, tok, r


def load_awq_weights(path: str):
    from ..formats.awq import AwqConfig, awq_dequant, awq_unpack
    with open(os.path.join(path, "config.json")) as f:
        d = json.load(f)
    acfg = AwqConfig.from_config(d)
    if acfg.bits != 4:
        raise ValueError(f"only 4-bit AWQ is supported (got {acfg.bits})")
    raw = load_safetensors_dir(path)
    cfg = ModelConfig.from_hf_dict(d)
    w, quant = {}, {}
    for name, t in raw.items():
        if name.endswith(".qweight"):
            base = name[:-len(".qweight")]
            q, z, s = awq_unpack(t, raw[base + ".qzeros"], raw[base + ".scales"],
                                 acfg.group_size)
            quant[base] = (q, z, s)
            w[base + ".weight"] = awq_dequant(q, z, s, acfg.group_size)
        elif name.endswith((".qzeros", ".scales")):
            continue
        else:
            w[name] = t.float()
    return cfg, w, quant, acfg


def quantized_layers(cfg, fmt, path, quant=None, reader=None):
    """HF-named projection -> QuantWeight for AWQ / GGUF Q4_K / Q8_0 checkpoints (None when
    a projection is stored in another type; the caller then keeps the bf16 path)."""
    from ..formats import quant as Q
    out = {}
    if fmt == "awq":
        for base, (q, z, s) in quant.items():
            out[base + ".weight"] = Q.from_awq(q, z, s, q.shape[1] // s.shape[1])
        return out
    from ..formats.gguf import GGML_Q4_K, GGML_Q8_0, gguf_name_to_hf
    for name, (dims, t, _, _) in reader.tensors.items():
        hf = gguf_name_to_hf(name)
        if hf is None or not hf.endswith("_proj.weight"):
            continue
        n, k = dims[1], dims[0]
        raw = reader.raw(name).numpy()
        if t == GGML_Q8_0:
            out[hf] = Q.from_q8_0(raw, n, k)
        elif t == GGML_Q4_K:
            out[hf] = Q.from_q4_k(raw, n, k)
        else:
            return None
    return out


def load_model_dir(path: str, device="cuda", tp_rank: int = 0, tp_size: int = 1,
                   dtype=torch.bfloat16, keep_quantized: Optional[bool] = None):
    """``keep_quantized`` (default: on CUDA) keeps AWQ / GGUF Q4_K / Q8_0 projections in the
    dequant-fused GEMM layout instead of dequantizing them to bf16 at load."""
    fmt = detect_format(path)
    keep = (torch.device(device).type == "cuda") if keep_quantized is None else keep_quantized
    qlayers = None
    if fmt == "gguf":
        cfg, w, tok, reader = load_gguf_weights(path)
        if keep:
            qlayers = quantized_layers(cfg, fmt, path, reader=reader)
    elif fmt == "awq":
        cfg, w, quant, _ = load_awq_weights(path)
        if keep:
            qlayers = quantized_layers(cfg, fmt, path, quant=quant)
        tok = None
    else:
        cfg, w = load_hf_weights(path)
        tok = None
    if tok is None:
        if fmt == "gguf":
            tok = ByteTokenizer(cfg.vocab_size)
        else:
            with open(os.path.join(path, "config.json")) as f:
                tok = load_tokenizer(path, cfg.vocab_size, json.load(f))
    packed = pack_model(cfg, w, rank=tp_rank, world=tp_size, dtype=dtype, device=device)
    if qlayers:
        from .weights import pack_layer_quant
        for i in range(cfg.num_layers):
            lw = dict(qlayers)
            p = f"model.layers.{i}."
            for nm in ("input_layernorm.weight", "post_attention_layernorm.weight",
                       "self_attn.q_norm.weight", "self_attn.k_norm.weight"):
                if p + nm in w:
                    lw[p + nm] = w[p + nm]
            packed["layers"][i] = pack_layer_quant(cfg, lw, i, tp_rank, tp_size, device)
    return cfg, packed, tok
