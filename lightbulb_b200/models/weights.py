"""Weight creation, safetensors I/O and packing into the device layout.

Naming follows the HF Llama layout that the reference's loaders read
(``src/loaders/mod.rs:57-126``).  The device layout is this framework's own:

* ``qkv``  : [q rows | k rows | v rows] of this rank's heads, one GEMM per layer;
* ``gate_up``: gate and up rows interleaved in 64-row groups (rows 0..63 of every 128-row
  tile are gate features f..f+63, rows 64..127 the up rows of the same features) so that one
  128-row tensor-core tile holds both halves of SwiGLU and the GEMM epilogue writes
  ``silu(g) * u`` directly;
* tensor parallel: column split for qkv/gate_up (by heads / features), row split for
  o_proj/down_proj, vocab split for lm_head (the reference's ``ShardedLinear`` column/row
  modes, ``src/multi_gpu/tensor_parallel.rs:199-345``).
"""
from __future__ import annotations

import glob
import hashlib
import json
import os
from typing import Dict, Optional

import torch

from ..config import ModelConfig

SWIGLU_GROUP = 64  # gate/up interleave granularity (half of the 128-row MMA tile)


def _name_seed(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 62) - 1)


def weight_shapes(cfg: ModelConfig) -> Dict[str, tuple]:
    h, f = cfg.hidden_size, cfg.intermediate_size
    shapes = {"model.embed_tokens.weight": (cfg.vocab_size, h), "model.norm.weight": (h,)}
    if not cfg.tie_word_embeddings:
        shapes["lm_head.weight"] = (cfg.vocab_size, h)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        shapes[p + "input_layernorm.weight"] = (h,)
        shapes[p + "post_attention_layernorm.weight"] = (h,)
        shapes[p + "self_attn.q_proj.weight"] = (cfg.q_size, h)
        shapes[p + "self_attn.k_proj.weight"] = (cfg.kv_size, h)
        shapes[p + "self_attn.v_proj.weight"] = (cfg.kv_size, h)
        shapes[p + "self_attn.o_proj.weight"] = (h, cfg.q_size)
        shapes[p + "mlp.gate_proj.weight"] = (f, h)
        shapes[p + "mlp.up_proj.weight"] = (f, h)
        shapes[p + "mlp.down_proj.weight"] = (h, f)
        if cfg.qk_norm:
            shapes[p + "self_attn.q_norm.weight"] = (cfg.head_dim,)
            shapes[p + "self_attn.k_norm.weight"] = (cfg.head_dim,)
    return shapes


def pad_norm(w: torch.Tensor, d: int, dp: int) -> torch.Tensor:
    """Per-head norm weight [d] -> [dp] (padded lanes of q / k are zero, so their weight is
    irrelevant; zero keeps them zero)."""
    if dp == d:
        return w
    out = torch.zeros(dp, dtype=w.dtype, device=w.device)
    out[:d] = w
    return out


def qk_norm_weights(cfg: ModelConfig, w, p: str, dev) -> Dict[str, torch.Tensor]:
    if not cfg.qk_norm:
        return {}
    dp = cfg.head_dim_padded
    return {"q_norm": dev(pad_norm(w[p + "self_attn.q_norm.weight"], cfg.head_dim, dp)),
            "k_norm": dev(pad_norm(w[p + "self_attn.k_norm.weight"], cfg.head_dim, dp))}


def random_tensor(name: str, shape: tuple, seed: int, dtype: torch.dtype, device="cpu",
                  std: float = 0.02) -> torch.Tensor:
    if name.endswith("norm.weight"):
        g = torch.Generator(device="cpu").manual_seed(_name_seed(seed, name))
        return (1.0 + 0.1 * torch.randn(shape, generator=g)).to(dtype).to(device)
    g = torch.Generator(device=device).manual_seed(_name_seed(seed, name))
    t = torch.empty(shape, dtype=torch.float32 if device == "cpu" else dtype, device=device)
    t.normal_(0.0, std, generator=g)
    return t.to(dtype)


def random_weights(cfg: ModelConfig, seed: int = 0, dtype=torch.float32, device="cpu",
                   std: float = 0.02) -> Dict[str, torch.Tensor]:
    """Random-init N(0, std) weights (norm gains ~1) with HF names."""
    return {n: random_tensor(n, s, seed, dtype, device, std) for n, s in weight_shapes(cfg).items()}


def save_checkpoint(path: str, cfg: ModelConfig, weights: Dict[str, torch.Tensor],
                    max_shard_bytes: int = 4 << 30) -> None:
    """Write ``config.json`` + sharded ``model-XXXXX-of-YYYYY.safetensors``."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg.to_hf_dict(), f, indent=2)
    shards, cur, cur_bytes = [], {}, 0
    for name in sorted(weights):
        t = weights[name].contiguous().cpu()
        nb = t.numel() * t.element_size()
        if cur and cur_bytes + nb > max_shard_bytes:
            shards.append(cur)
            cur, cur_bytes = {}, 0
        cur[name] = t
        cur_bytes += nb
    if cur:
        shards.append(cur)
    index = {"metadata": {}, "weight_map": {}}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors" if len(shards) > 1 else \
            "model.safetensors"
        save_file(sh, os.path.join(path, fn), metadata={"format": "pt"})
        for n in sh:
            index["weight_map"][n] = fn
    if len(shards) > 1:
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump(index, f)


def load_safetensors_dir(path: str, device="cpu",
                         dtype: Optional[torch.dtype] = None) -> Dict[str, torch.Tensor]:
    """Load every ``*.safetensors`` file in ``path`` (sorted), as ``src/loaders/mod.rs:18-56``."""
    from safetensors.torch import load_file
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors under {path}")
    out: Dict[str, torch.Tensor] = {}
    for fn in files:
        for k, v in load_file(fn, device=str(device)).items():
            out[k] = v.to(dtype) if dtype is not None else v
    return out


# ----------------------------------------------------------------------------------------
# Device packing
# ----------------------------------------------------------------------------------------

def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = SWIGLU_GROUP):
    """[F, H] x2 -> [2F, H] with 64-row gate/up groups alternating."""
    f, h = gate.shape
    assert f % group == 0, f"intermediate size {f} must be a multiple of {group}"
    g = gate.view(f // group, group, h)
    u = up.view(f // group, group, h)
    return torch.stack([g, u], dim=1).reshape(2 * f, h)


def deinterleave_gate_up(w: torch.Tensor, group: int = SWIGLU_GROUP):
    f2, h = w.shape
    x = w.view(f2 // (2 * group), 2, group, h)
    return x[:, 0].reshape(-1, h), x[:, 1].reshape(-1, h)


def tp_head_ranges(cfg: ModelConfig, rank: int, world: int):
    """Query-head and KV-head slices owned by ``rank``.  KV heads are replicated when
    ``num_kv_heads < world`` (each rank keeps the one KV head its query heads use)."""
    assert cfg.num_heads % world == 0
    hq = cfg.num_heads // world
    q0 = rank * hq
    if cfg.num_kv_heads >= world:
        assert cfg.num_kv_heads % world == 0
        hk = cfg.num_kv_heads // world
        k0 = rank * hk
    else:
        hk = 1
        k0 = q0 // cfg.group_size
    return (q0, hq), (k0, hk)


def pad_head_rows(w: torch.Tensor, n_heads: int, d: int, dp: int) -> torch.Tensor:
    """[n_heads * d, K] -> [n_heads * dp, K] with zero rows after each head's d rows."""
    if d == dp:
        return w
    k = w.shape[1]
    out = torch.zeros(n_heads, dp, k, dtype=w.dtype, device=w.device)
    out[:, :d] = w.reshape(n_heads, d, k)
    return out.reshape(n_heads * dp, k)


def pad_head_cols(w: torch.Tensor, n_heads: int, d: int, dp: int) -> torch.Tensor:
    """[H, n_heads * d] -> [H, n_heads * dp] with zero columns after each head's d columns."""
    if d == dp:
        return w
    h = w.shape[0]
    out = torch.zeros(h, n_heads, dp, dtype=w.dtype, device=w.device)
    out[:, :, :d] = w.reshape(h, n_heads, d)
    return out.reshape(h, n_heads * dp)


def pack_layer(cfg: ModelConfig, w: Dict[str, torch.Tensor], i: int, rank: int = 0,
               world: int = 1, dtype=torch.bfloat16, device="cpu") -> Dict[str, torch.Tensor]:
    p = f"model.layers.{i}."
    d = cfg.head_dim
    (q0, hq), (k0, hk) = tp_head_ranges(cfg, rank, world)
    qw = w[p + "self_attn.q_proj.weight"][q0 * d:(q0 + hq) * d]
    kw = w[p + "self_attn.k_proj.weight"][k0 * d:(k0 + hk) * d]
    vw = w[p + "self_attn.v_proj.weight"][k0 * d:(k0 + hk) * d]
    ow = w[p + "self_attn.o_proj.weight"][:, q0 * d:(q0 + hq) * d]
    f = cfg.intermediate_size
    assert f % world == 0
    fl = f // world
    gw = w[p + "mlp.gate_proj.weight"][rank * fl:(rank + 1) * fl]
    uw = w[p + "mlp.up_proj.weight"][rank * fl:(rank + 1) * fl]
    dw = w[p + "mlp.down_proj.weight"][:, rank * fl:(rank + 1) * fl]

    def dev(t):
        return t.to(device=device, dtype=dtype).contiguous()

    dp = cfg.head_dim_padded
    qw, kw, vw = (pad_head_rows(qw, hq, d, dp), pad_head_rows(kw, hk, d, dp),
                  pad_head_rows(vw, hk, d, dp))
    ow = pad_head_cols(ow, hq, d, dp)
    return {
        "ln_in": dev(w[p + "input_layernorm.weight"]),
        "ln_post": dev(w[p + "post_attention_layernorm.weight"]),
        "qkv": dev(torch.cat([qw, kw, vw], 0)),
        "o": dev(ow),
        "gate_up": dev(interleave_gate_up(gw, uw)),
        "down": dev(dw),
        **qk_norm_weights(cfg, w, p, dev),
    }


def pack_model(cfg: ModelConfig, w: Dict[str, torch.Tensor], rank: int = 0, world: int = 1,
               dtype=torch.bfloat16, device="cpu") -> Dict[str, object]:
    v = cfg.vocab_size
    vl = (v + world - 1) // world
    lm = w.get("lm_head.weight", w["model.embed_tokens.weight"])
    lm_shard = lm[rank * vl:min(v, (rank + 1) * vl)]
    return {
        "embed": w["model.embed_tokens.weight"].to(device=device, dtype=dtype).contiguous(),
        "norm": w["model.norm.weight"].to(device=device, dtype=dtype).contiguous(),
        "lm_head": lm_shard.to(device=device, dtype=dtype).contiguous(),
        "layers": [pack_layer(cfg, w, i, rank, world, dtype, device)
                   for i in range(cfg.num_layers)],
    }


def random_packed_model(cfg: ModelConfig, seed: int = 0, rank: int = 0, world: int = 1,
                        dtype=torch.bfloat16, device="cuda", std: float = 0.02):
    """Random-init weights created layer by layer directly in device layout (the full-size
    benchmark models never exist as a whole on the host)."""
    layers = []
    for i in range(cfg.num_layers):
        names = [n for n in weight_shapes(cfg) if n.startswith(f"model.layers.{i}.")]
        shapes = weight_shapes(cfg)
        lw = {n: random_tensor(n, shapes[n], seed, torch.bfloat16, device, std) for n in names}
        layers.append(pack_layer(cfg, lw, i, rank, world, dtype, device))
        del lw
    shapes = weight_shapes(cfg)
    top = {n: random_tensor(n, shapes[n], seed, torch.bfloat16, device, std)
           for n in ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight")
           if n in shapes}
    v = cfg.vocab_size
    vl = (v + world - 1) // world
    lm = top.get("lm_head.weight", top["model.embed_tokens.weight"])
    return {
        "embed": top["model.embed_tokens.weight"].to(dtype).contiguous(),
        "norm": top["model.norm.weight"].to(dtype).contiguous(),
        "lm_head": lm[rank * vl:min(v, (rank + 1) * vl)].to(dtype).contiguous(),
        "layers": layers,
    }


# ----------------------------------------------------------------------------------------
# Quantized packing (AWQ int4 / GGUF Q4_K / Q8_0 -> dequant-fused GEMM layout)
# ----------------------------------------------------------------------------------------
def pack_layer_quant(cfg: ModelConfig, lw: Dict[str, object], i: int, rank: int = 0,
                     world: int = 1, device="cpu") -> Dict[str, object]:
    """``lw`` maps HF projection names to QuantWeight (norms as tensors)."""
    from ..formats.quant import cat_rows, interleave_rows
    p = f"model.layers.{i}."
    d = cfg.head_dim
    (q0, hq), (k0, hk) = tp_head_ranges(cfg, rank, world)
    fl = cfg.intermediate_size // world
    qw = lw[p + "self_attn.q_proj.weight"].rows(slice(q0 * d, (q0 + hq) * d))
    kw = lw[p + "self_attn.k_proj.weight"].rows(slice(k0 * d, (k0 + hk) * d))
    vw = lw[p + "self_attn.v_proj.weight"].rows(slice(k0 * d, (k0 + hk) * d))
    ow = lw[p + "self_attn.o_proj.weight"].cols(q0 * d, (q0 + hq) * d)
    gw = lw[p + "mlp.gate_proj.weight"].rows(slice(rank * fl, (rank + 1) * fl))
    uw = lw[p + "mlp.up_proj.weight"].rows(slice(rank * fl, (rank + 1) * fl))
    dw = lw[p + "mlp.down_proj.weight"].cols(rank * fl, (rank + 1) * fl)

    def dev(t):
        return t.contiguous().to(device)

    def nrm(name):
        return lw[p + name].to(device=device, dtype=torch.bfloat16).contiguous()

    dp = cfg.head_dim_padded
    if dp != d:
        # narrow heads: zero rows per head in q/k/v (exact); o_proj's input groups would not
        # line up with the padded head width, so it is kept dequantized (bf16)
        qw, kw, vw = (qw.pad_head_rows(hq, d, dp), kw.pad_head_rows(hk, d, dp),
                      vw.pad_head_rows(hk, d, dp))
        ow = pad_head_cols(ow.to(device).dequantize(torch.bfloat16), hq, d, dp)
    return {"ln_in": nrm("input_layernorm.weight"), "ln_post": nrm("post_attention_layernorm.weight"),
            "qkv": dev(cat_rows([qw, kw, vw])), "o": dev(ow),
            "gate_up": dev(interleave_rows(gw, uw)), "down": dev(dw),
            **qk_norm_weights(cfg, lw, p,
                              lambda t: t.to(device=device, dtype=torch.bfloat16).contiguous())}


def random_packed_awq_model(cfg: ModelConfig, seed: int = 0, rank: int = 0, world: int = 1,
                            device="cuda", group: int = 128):
    """Random AWQ int4 model (uint4 weights, fp16 scales U[0.001, 0.02], zeros U{0..15}),
    created shard by shard on the device; norms / embeddings random bf16."""
    from ..formats.quant import QuantWeight
    g = torch.Generator(device=device).manual_seed(seed)
    shapes = weight_shapes(cfg)
    layers = []

    def qlin(n, k):
        # random uint4 values: any byte pattern is a valid packing of 8 random nibbles
        qw = torch.randint(0, 256, (n, k // 2), generator=g, device=device, dtype=torch.int32)
        s = torch.empty(n, k // group, device=device).uniform_(0.001, 0.02, generator=g)
        z = torch.randint(0, 16, (n, k // group), generator=g, device=device).float()
        return QuantWeight(qw.to(torch.uint8), s.half(), (z * s).half(), 4, group, int_zero=True)

    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        lw = {}
        for name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                     "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            n_, k_ = shapes[p + name + ".weight"]
            lw[p + name + ".weight"] = qlin(n_, k_)
        for name in ("input_layernorm.weight", "post_attention_layernorm.weight",
                     "self_attn.q_norm.weight", "self_attn.k_norm.weight"):
            if p + name in shapes:
                lw[p + name] = random_tensor(p + name, shapes[p + name], seed, torch.bfloat16,
                                             device)
        layers.append(pack_layer_quant(cfg, lw, i, rank, world, device))
    top = {n: random_tensor(n, shapes[n], seed, torch.bfloat16, device)
           for n in ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight")
           if n in shapes}
    v = cfg.vocab_size
    vl = (v + world - 1) // world
    lm = top.get("lm_head.weight", top["model.embed_tokens.weight"])
    return {"embed": top["model.embed_tokens.weight"].contiguous(),
            "norm": top["model.norm.weight"].contiguous(),
            "lm_head": lm[rank * vl:min(v, (rank + 1) * vl)].contiguous(), "layers": layers}
