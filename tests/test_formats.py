"""GGUF (C++ reader + dequant) and AWQ formats, and the checkpoint loaders."""
import os
import struct

import numpy as np
import pytest
import torch

from lightbulb_b200.config import get_preset
from lightbulb_b200.formats import awq as A
from lightbulb_b200.formats import gguf as G
from lightbulb_b200.models.weights import random_weights, save_checkpoint


def test_gguf_roundtrip_types(tmp_path):
    torch.manual_seed(0)
    x = torch.randn(4, 512) * 0.1
    tensors = {
        "a.f32": (G.GGML_F32, [4, 512], G.quantize(x, G.GGML_F32)),
        "a.f16": (G.GGML_F16, [4, 512], G.quantize(x, G.GGML_F16)),
        "a.bf16": (G.GGML_BF16, [4, 512], G.quantize(x, G.GGML_BF16)),
        "a.q8": (G.GGML_Q8_0, [4, 512], G.quantize(x, G.GGML_Q8_0)),
        "a.q4k": (G.GGML_Q4_K, [4, 512], G.quantize(x, G.GGML_Q4_K)),
    }
    md = {"general.architecture": "llama", "x.list": [1, 2, 3], "x.s": "hi", "x.f": 1.5,
          "x.b": True, "tokenizer.ggml.tokens": ["a", "b"]}
    p = str(tmp_path / "t.gguf")
    G.write_gguf(p, md, tensors)
    r = G.GGUFReader(p)
    assert r.version == 3
    assert r.metadata["x.list"] == [1, 2, 3] and r.metadata["x.s"] == "hi"
    assert r.metadata["x.b"] is True and abs(r.metadata["x.f"] - 1.5) < 1e-6
    assert r.shape("a.q4k") == [4, 512]
    assert torch.equal(r.dequantize("a.f32"), x)
    assert torch.allclose(r.dequantize("a.f16"), x, atol=1e-3)
    assert torch.allclose(r.dequantize("a.bf16"), x, atol=2e-3)
    q8 = r.dequantize("a.q8")
    assert (q8 - x).abs().max() < x.abs().max() / 127 * 0.51 + 1e-3
    q4 = r.dequantize("a.q4k")
    rel = ((q4 - x).norm() / x.norm()).item()
    assert rel < 0.12, rel


def test_q4k_reference_decoding_by_hand():
    # one super-block: check the packed 6-bit scale/min layout decodes as written
    x = torch.linspace(-1, 2, 256).reshape(1, 256)
    raw = np.frombuffer(G.quantize(x, G.GGML_Q4_K), dtype=np.uint8)
    assert raw.size == 144
    from lightbulb_b200 import _native
    y = _native.dequantize(G.GGML_Q4_K, torch.from_numpy(raw.copy()), 256)
    assert ((y - x.flatten()).abs().max() < 0.08)


def test_gguf_rejects_corrupt(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUF" + struct.pack("<I", 3) + b"\xff" * 8)
    with pytest.raises(Exception):
        G.GGUFReader(str(p))
    p.write_bytes(b"NOPE" + b"\0" * 40)
    with pytest.raises(Exception):
        G.GGUFReader(str(p))


def test_gguf_tokenizer_roundtrip():
    from lightbulb_b200.engine.tokenizer import GGUFTokenizer
    toks = ["<unk>", "<s>", "</s>", "▁hello", "▁world", "▁", "h", "e", "l", "o"] + \
        [f"<0x{i:02X}>" for i in range(256)]
    t = GGUFTokenizer({"tokenizer.ggml.tokens": toks, "tokenizer.ggml.bos_token_id": 1,
                       "tokenizer.ggml.eos_token_id": 2,
                       "tokenizer.ggml.token_type": [2, 3, 3] + [1] * (len(toks) - 3)})
    ids = t.encode("hello world")
    assert ids[0] == 1 and ids[1:] == [3, 4]
    assert t.decode(ids) == "hello world"


def test_awq_pack_unpack_both_layouts():
    g = torch.Generator().manual_seed(0)
    q, z, s = A.random_awq_linear(64, 256, 128, g)
    qw, qz, sc = A.awq_pack_gemm(q, z, s)
    assert qw.shape == (256, 8) and qz.shape == (2, 8) and sc.shape == (2, 64)
    q2, z2, s2 = A.awq_unpack(qw, qz, sc, 128)
    assert torch.equal(q2, q) and torch.equal(z2, z) and torch.equal(s2, s)
    # K-packed variant [in/8, out]
    kp = A.pack_int32_nibbles(q.view(64, 32, 8)).t().contiguous()
    q3, _, _ = A.awq_unpack(kp, qz, sc, 128)
    assert torch.equal(q3, q)
    w = A.awq_dequant(q, z, s, 128)
    assert torch.allclose(w[0, :128], (q[0, :128].float() - z[0, 0].float()) * s[0, 0].float())


def _greedy(cfg, packed, tok=None, n=6):
    from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=64, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                  max_model_len=256), use_cuda_graphs=False)
    eng = LLMEngine(ecfg, packed, tok)
    return eng.generate(prompt_token_ids=[[5, 6, 7, 8, 9]],
                        params=SamplingParams(temperature=0.0, max_tokens=n,
                                              ignore_eos=True))[0].output_token_ids


def test_loaders_safetensors_gguf_awq(tmp_path):
    from lightbulb_b200.models.loader import detect_format, load_model_dir
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=4, std=0.05)
    st = str(tmp_path / "st")
    save_checkpoint(st, cfg, w, max_shard_bytes=1 << 20)   # force several shards
    assert detect_format(st) == "safetensors"
    c1, p1, _ = load_model_dir(st, device="cpu")
    assert c1.hidden_size == cfg.hidden_size
    gg = str(tmp_path / "m.gguf")
    G.save_llama_gguf(gg, cfg, w, linear_type=G.GGML_Q8_0)
    assert detect_format(gg) == "gguf"
    c2, p2, _ = load_model_dir(gg, device="cpu")
    assert c2.num_layers == cfg.num_layers and c2.num_kv_heads == cfg.num_kv_heads
    a1 = _greedy(c1, p1)
    a2 = _greedy(c2, p2)
    assert a1[:2] == a2[:2]  # Q8_0 is close to the float weights
    aw = str(tmp_path / "awq")
    A.save_awq_checkpoint(aw, cfg, w, group=128)
    assert detect_format(aw) == "awq"
    c3, p3, _ = load_model_dir(aw, device="cpu")
    assert len(_greedy(c3, p3)) == 6


def test_awq_and_gguf_kept_quantized_match_dequantized(tmp_path):
    from lightbulb_b200.formats.quant import QuantWeight
    from lightbulb_b200.models.loader import load_model_dir
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=6, std=0.05)
    aw = str(tmp_path / "awq")
    A.save_awq_checkpoint(aw, cfg, w, group=128)
    gg = str(tmp_path / "m.gguf")
    G.save_llama_gguf(gg, cfg, w, linear_type=G.GGML_Q4_K)
    for path in (aw, gg):
        cq, pq, _ = load_model_dir(path, device="cpu", keep_quantized=True)
        cd, pd, _ = load_model_dir(path, device="cpu", keep_quantized=False)
        assert isinstance(pq["layers"][0]["qkv"], QuantWeight)
        assert _greedy(cq, pq)[:3] == _greedy(cd, pd)[:3]
