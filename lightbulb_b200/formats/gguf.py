"""GGUF: Python side of the C++ reader, a writer, and reference quantizers.

* :class:`GGUFReader` wraps ``_native.GGUFFile`` (mmap parser + CPU dequant in C++).
* :func:`write_gguf` writes GGUF v3 files (used to make random-init quantized checkpoints
  and test fixtures; the reference only reads GGUF).
* :func:`quantize_q8_0` / :func:`quantize_q4_k` produce ggml block layouts from float rows.
  The Q4_K quantizer here is a simple min/max fit per 32-element sub-block (not ggml's
  iterative search); the block FORMAT is the public one, so any reader decodes it.
* llama metadata keys with the reference's fallbacks (``src/gguf/mod.rs:36-283``,
  ``src/model/parallel_model_manager.rs:250-391``): ``llama.embedding_length`` /
  ``n_embd``, ``rope.freq_base`` default 1e4, etc.
"""
from __future__ import annotations

import struct
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from ..config import ModelConfig

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_BF16 = 0, 1, 2, 8, 12, 14, 30
TYPE_GEOM = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2), GGML_Q4_0: (32, 18),
             GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210)}
TYPE_NAMES = {"f32": GGML_F32, "f16": GGML_F16, "bf16": GGML_BF16, "q4_0": GGML_Q4_0,
              "q8_0": GGML_Q8_0, "q4_k": GGML_Q4_K, "q6_k": GGML_Q6_K}


class GGUFReader:
    def __init__(self, path: str):
        from .. import _native  # noqa: F401  (torch imported by the package)
        self.path = path
        self._f = _native.GGUFFile(path)
        self.metadata: dict = self._f.metadata()
        self.tensors: Dict[str, Tuple[List[int], int, int, int]] = {
            name: (dims, t, off, nb) for name, dims, t, off, nb in self._f.tensors()}

    @property
    def version(self) -> int:
        return self._f.version

    def raw(self, name: str) -> torch.Tensor:
        return self._f.raw(name)

    def dequantize(self, name: str) -> torch.Tensor:
        return self._f.dequantize(name)

    def type_of(self, name: str) -> int:
        return self.tensors[name][1]

    def shape(self, name: str) -> List[int]:
        return list(reversed(self.tensors[name][0]))


# ---------------------------------------------------------------------------------------
# Writer
# ---------------------------------------------------------------------------------------
def _w_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _w_value(v) -> Tuple[int, bytes]:
    if isinstance(v, bool):
        return 7, struct.pack("<B", int(v))
    if isinstance(v, int):
        return (4, struct.pack("<I", v)) if 0 <= v < 2**32 else (11, struct.pack("<q", v))
    if isinstance(v, float):
        return 6, struct.pack("<f", v)
    if isinstance(v, str):
        return 8, _w_str(v)
    if isinstance(v, (list, tuple)):
        if not v:
            return 9, struct.pack("<IQ", 8, 0)
        et, _ = _w_value(v[0])
        body = b"".join(_w_value(x)[1] for x in v)
        return 9, struct.pack("<IQ", et, len(v)) + body
    raise TypeError(type(v))


def write_gguf(path: str, metadata: dict, tensors: Dict[str, Tuple[int, List[int], bytes]],
               alignment: int = 32) -> None:
    """tensors: name -> (ggml type, torch-order shape, raw bytes)."""
    meta = dict(metadata)
    meta.setdefault("general.alignment", alignment)
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(meta))
    for k, v in meta.items():
        t, b = _w_value(v)
        head += _w_str(k) + struct.pack("<I", t) + b
    off = 0
    infos = b""
    order = list(tensors.items())
    offsets = []
    for name, (t, shape, raw) in order:
        offsets.append(off)
        dims = list(reversed(shape))
        infos += _w_str(name) + struct.pack("<I", len(dims)) + b"".join(
            struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", t, off)
        off += (len(raw) + alignment - 1) // alignment * alignment
    data_start = len(head) + len(infos)
    pad = (-data_start) % alignment
    with open(path, "wb") as f:
        f.write(head + infos + b"\0" * pad)
        for (name, (t, shape, raw)), o in zip(order, offsets):
            f.write(raw)
            f.write(b"\0" * ((-len(raw)) % alignment))


# ---------------------------------------------------------------------------------------
# Quantizers (float32 rows -> ggml block bytes)
# ---------------------------------------------------------------------------------------
def quantize_q8_0(x: np.ndarray) -> bytes:
    x = x.astype(np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = amax / 127.0
    inv = np.where(d > 0, 1.0 / np.maximum(d, 1e-30), 0.0)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    out = np.zeros((x.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def _pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """8 x 6-bit scales and mins -> 12 bytes (the Q4_K / Q5_K packing)."""
    out = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    for j in range(4):
        out[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        out[:, j + 4] = (mn[:, j] & 63) | ((mn[:, j + 4] >> 4) << 6)
        out[:, j + 8] = (sc[:, j + 4] & 0xF) | ((mn[:, j + 4] & 0xF) << 4)
    return out


def quantize_q4_k(x: np.ndarray) -> bytes:
    """y = d*sc*q - dmin*m per 32-element sub-block, q in 0..15, sc/m 6-bit."""
    x = x.astype(np.float32).reshape(-1, 8, 32)
    nb = x.shape[0]
    mins = np.minimum(x.min(axis=2), 0.0)            # <= 0
    maxs = x.max(axis=2)
    scale = np.maximum((maxs - mins) / 15.0, 1e-12)   # per sub-block step
    m = -mins                                          # >= 0
    d = np.maximum(scale.max(axis=1) / 63.0, 1e-12)
    dmin = np.maximum(m.max(axis=1) / 63.0, 1e-12)
    sc = np.clip(np.rint(scale / d[:, None]), 0, 63).astype(np.uint8)
    mn = np.clip(np.rint(m / dmin[:, None]), 0, 63).astype(np.uint8)
    d16 = d.astype(np.float16)
    dm16 = dmin.astype(np.float16)
    eff_s = d16.astype(np.float32)[:, None] * sc.astype(np.float32)
    eff_m = dm16.astype(np.float32)[:, None] * mn.astype(np.float32)
    q = np.clip(np.rint((x + eff_m[:, :, None]) / np.maximum(eff_s, 1e-12)[:, :, None]), 0, 15)
    q = q.astype(np.uint8)
    out = np.zeros((nb, 144), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(-1, 2)
    out[:, 4:16] = _pack_scale_min_k4(sc, mn)
    qs = np.zeros((nb, 128), dtype=np.uint8)
    for j in range(4):  # sub-blocks 2j (low nibble) and 2j+1 (high nibble) share 32 bytes
        qs[:, 32 * j:32 * (j + 1)] = q[:, 2 * j] | (q[:, 2 * j + 1] << 4)
    out[:, 16:] = qs
    return out.tobytes()


def quantize(t: torch.Tensor, ggml_type: int) -> bytes:
    a = t.detach().float().cpu().numpy()
    if ggml_type == GGML_F32:
        return a.astype(np.float32).tobytes()
    if ggml_type == GGML_F16:
        return a.astype(np.float16).tobytes()
    if ggml_type == GGML_BF16:
        return t.detach().to(torch.bfloat16).cpu().view(torch.int16).numpy().tobytes()
    if ggml_type == GGML_Q8_0:
        return quantize_q8_0(a)
    if ggml_type == GGML_Q4_K:
        return quantize_q4_k(a)
    raise ValueError(f"no quantizer for ggml type {ggml_type}")


# ---------------------------------------------------------------------------------------
# Llama mapping
# ---------------------------------------------------------------------------------------
HF_TO_GGUF = {
    "model.embed_tokens.weight": "token_embd.weight",
    "model.norm.weight": "output_norm.weight",
    "lm_head.weight": "output.weight",
}
LAYER_MAP = {
    "input_layernorm.weight": "attn_norm.weight",
    "post_attention_layernorm.weight": "ffn_norm.weight",
    "self_attn.q_proj.weight": "attn_q.weight",
    "self_attn.k_proj.weight": "attn_k.weight",
    "self_attn.v_proj.weight": "attn_v.weight",
    "self_attn.o_proj.weight": "attn_output.weight",
    "mlp.gate_proj.weight": "ffn_gate.weight",
    "mlp.up_proj.weight": "ffn_up.weight",
    "mlp.down_proj.weight": "ffn_down.weight",
    "self_attn.q_norm.weight": "attn_q_norm.weight",     # Qwen3
    "self_attn.k_norm.weight": "attn_k_norm.weight",
}


def hf_name_to_gguf(name: str) -> str:
    if name in HF_TO_GGUF:
        return HF_TO_GGUF[name]
    if name.startswith("model.layers."):
        rest = name[len("model.layers."):]
        i, sub = rest.split(".", 1)
        return f"blk.{i}.{LAYER_MAP[sub]}"
    raise KeyError(name)


def gguf_name_to_hf(name: str) -> Optional[str]:
    inv = {v: k for k, v in HF_TO_GGUF.items()}
    if name in inv:
        return inv[name]
    if name.startswith("blk."):
        _, i, sub = name.split(".", 2)
        for k, v in LAYER_MAP.items():
            if v == sub:
                return f"model.layers.{i}.{k}"
    return None


def _meta(md: dict, *keys, default=None):
    for k in keys:
        if k in md:
            return md[k]
    return default


def config_from_gguf(md: dict) -> ModelConfig:
    arch = md.get("general.architecture", "llama")
    p = f"{arch}."
    hs = int(_meta(md, p + "embedding_length", p + "n_embd"))
    nh = int(_meta(md, p + "attention.head_count", p + "n_head"))
    head_dim = int(_meta(md, p + "attention.key_length", default=0) or 0)
    toks = md.get("tokenizer.ggml.tokens")
    vocab = int(_meta(md, p + "vocab_size", default=len(toks) if toks else 32000))
    return ModelConfig(
        name=md.get("general.name", arch), vocab_size=vocab, hidden_size=hs,
        intermediate_size=int(_meta(md, p + "feed_forward_length", p + "n_ff")),
        num_layers=int(_meta(md, p + "block_count", p + "n_layer")), num_heads=nh,
        num_kv_heads=int(_meta(md, p + "attention.head_count_kv", default=nh)),
        rope_theta=float(_meta(md, p + "rope.freq_base", default=10000.0)),
        rms_norm_eps=float(_meta(md, p + "attention.layer_norm_rms_epsilon", default=1e-5)),
        max_position_embeddings=int(_meta(md, p + "context_length", default=4096)),
        bos_token_id=int(md.get("tokenizer.ggml.bos_token_id", 1)),
        eos_token_id=int(md.get("tokenizer.ggml.eos_token_id", 2)),
        tie_word_embeddings=False, head_dim=head_dim, qk_norm=arch == "qwen3")


def save_llama_gguf(path: str, cfg: ModelConfig, weights: Dict[str, torch.Tensor],
                    linear_type: int = GGML_Q4_K, other_type: int = GGML_F32,
                    extra_meta: Optional[dict] = None) -> None:
    md = {"general.architecture": "llama", "general.name": cfg.name,
          "llama.embedding_length": cfg.hidden_size, "llama.feed_forward_length":
          cfg.intermediate_size, "llama.block_count": cfg.num_layers,
          "llama.attention.head_count": cfg.num_heads,
          "llama.attention.head_count_kv": cfg.num_kv_heads,
          "llama.rope.freq_base": float(cfg.rope_theta),
          "llama.attention.layer_norm_rms_epsilon": float(cfg.rms_norm_eps),
          "llama.context_length": cfg.max_position_embeddings,
          "llama.vocab_size": cfg.vocab_size,
          "tokenizer.ggml.bos_token_id": cfg.bos_token_id,
          "tokenizer.ggml.eos_token_id": cfg.eos_ids()[0]}
    md.update(extra_meta or {})
    tensors = {}
    for name, t in weights.items():
        lin = name.endswith("proj.weight") or name == "lm_head.weight"
        typ = linear_type if lin and t.shape[-1] % TYPE_GEOM[linear_type][0] == 0 else other_type
        tensors[hf_name_to_gguf(name)] = (typ, list(t.shape), quantize(t, typ))
    write_gguf(path, md, tensors)
