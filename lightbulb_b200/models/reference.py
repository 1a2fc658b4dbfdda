"""CPU fp32 reference Llama model: the numerical oracle and the ``local-llama-gen`` path.

This restates the math of the reference's candle Llama path in plain PyTorch fp32:
RMSNorm ``x * rsqrt(mean(x^2) + eps) * g`` (``src/model/fused_rmsnorm.rs:47-110``),
rotate-half RoPE over the full head dim (``src/model/custom_attention.rs:687-728``),
GQA attention with causal mask (``custom_attention.rs:741-858``), Qwen3's per-head q/k RMSNorm
(``src/model/awq_qwen3.rs:259-267``), SwiGLU MLP
(``src/model/mlp_wrapper.rs:154-199``) and greedy argmax with first-max tie-break
(``src/model_fuel/generate.rs:54-65``).  It is deliberately unoptimised and independent of
every CUDA kernel in this package so that kernel tests compare against it.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

from ..config import ModelConfig


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float):
    inv = rope_inv_freq(head_dim, theta)
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE.  ``x``: [T, H, D]; cos/sin: [T, D/2]."""
    d2 = x.shape[-1] // 2
    x1, x2 = x[..., :d2], x[..., d2:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor,
                  k_pos: Optional[torch.Tensor] = None, causal: bool = True,
                  scale: Optional[float] = None) -> torch.Tensor:
    """fp32 GQA attention.  q: [Tq, Hq, D]; k, v: [Tk, Hkv, D]; positions give the causal mask;
    scale defaults to 1 / sqrt(D)."""
    tq, hq, d = q.shape
    tk, hkv, _ = k.shape
    g = hq // hkv
    qf, kf, vf = q.float(), k.float(), v.float()
    kf = kf.repeat_interleave(g, dim=1)
    vf = vf.repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", qf, kf) * (scale if scale is not None else 1.0 / math.sqrt(d))
    if causal:
        if k_pos is None:
            k_pos = torch.arange(tk)
        mask = k_pos[None, :] > q_pos[:, None]
        s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vf)


class ReferenceLlama:
    """fp32 Llama forward with a dense per-sequence KV cache."""

    def __init__(self, cfg: ModelConfig, weights: Dict[str, torch.Tensor]):
        self.cfg = cfg
        self.w = {k: v.float().contiguous() for k, v in weights.items()}
        self.k_cache: List[torch.Tensor] = []
        self.v_cache: List[torch.Tensor] = []
        self.reset()

    def reset(self) -> None:
        c = self.cfg
        self.k_cache = [torch.zeros(0, c.num_kv_heads, c.head_dim) for _ in range(c.num_layers)]
        self.v_cache = [torch.zeros(0, c.num_kv_heads, c.head_dim) for _ in range(c.num_layers)]

    @property
    def seq_len(self) -> int:
        return self.k_cache[0].shape[0]

    def lm_head_weight(self) -> torch.Tensor:
        if "lm_head.weight" in self.w:
            return self.w["lm_head.weight"]
        return self.w["model.embed_tokens.weight"]

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """Append ``tokens`` ([T] int) to the cache and return logits [T, vocab] (fp32)."""
        c = self.cfg
        w = self.w
        start = self.seq_len
        t = tokens.shape[0]
        pos = torch.arange(start, start + t)
        cos, sin = rope_cos_sin(pos, c.head_dim, c.rope_theta)
        x = w["model.embed_tokens.weight"][tokens.long()]
        for i in range(c.num_layers):
            p = f"model.layers.{i}."
            h = rms_norm(x, w[p + "input_layernorm.weight"], c.rms_norm_eps)
            q = (h @ w[p + "self_attn.q_proj.weight"].T).view(t, c.num_heads, c.head_dim)
            k = (h @ w[p + "self_attn.k_proj.weight"].T).view(t, c.num_kv_heads, c.head_dim)
            v = (h @ w[p + "self_attn.v_proj.weight"].T).view(t, c.num_kv_heads, c.head_dim)
            if c.qk_norm:   # Qwen3 (src/model/awq_qwen3.rs:259-267): per-head norm, then RoPE
                q = rms_norm(q, w[p + "self_attn.q_norm.weight"], c.rms_norm_eps)
                k = rms_norm(k, w[p + "self_attn.k_norm.weight"], c.rms_norm_eps)
            q = apply_rope(q, cos, sin)
            k = apply_rope(k, cos, sin)
            self.k_cache[i] = torch.cat([self.k_cache[i], k], 0)
            self.v_cache[i] = torch.cat([self.v_cache[i], v], 0)
            a = attention_ref(q, self.k_cache[i], self.v_cache[i], pos)
            x = x + a.reshape(t, -1) @ w[p + "self_attn.o_proj.weight"].T
            h = rms_norm(x, w[p + "post_attention_layernorm.weight"], c.rms_norm_eps)
            g = h @ w[p + "mlp.gate_proj.weight"].T
            u = h @ w[p + "mlp.up_proj.weight"].T
            x = x + (torch.nn.functional.silu(g) * u) @ w[p + "mlp.down_proj.weight"].T
        x = rms_norm(x, w["model.norm.weight"], c.rms_norm_eps)
        return x @ self.lm_head_weight().T


def greedy_argmax(logits: torch.Tensor) -> int:
    """Argmax with first-max tie-break (``generate.rs:54-65``)."""
    m = logits.max()
    return int((logits == m).nonzero()[0].item())


@torch.no_grad()
def greedy_generate(model: ReferenceLlama, prompt: List[int], max_new_tokens: int,
                    eos_ids: Optional[List[int]] = None) -> List[int]:
    model.reset()
    out: List[int] = []
    logits = model.forward(torch.tensor(prompt))
    for _ in range(max_new_tokens):
        tok = greedy_argmax(logits[-1])
        out.append(tok)
        if eos_ids and tok in eos_ids:
            break
        logits = model.forward(torch.tensor([tok]))
    return out
