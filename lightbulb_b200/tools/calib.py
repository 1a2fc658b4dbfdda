"""Calibration forward passes that expose the activations the offline tools need.

Runs the fp32 oracle math (``models/reference.py``) over HF-named weight dicts and records, per
layer, the RMS-normalised hidden states *before* the gain (inputs of the attention and MLP
projections) and the inputs of every linear layer.  Used by norm tweaking (targets and inputs)
and Wanda pruning (input activation norms).
"""
from __future__ import annotations

from typing import Dict, List

import torch

from ..config import ModelConfig
from ..models.reference import apply_rope, attention_ref, rope_cos_sin


def _rms(x: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


@torch.no_grad()
def trace(cfg: ModelConfig, w: Dict[str, torch.Tensor], tokens: torch.Tensor,
          gains: Dict[str, torch.Tensor] = None) -> Dict[str, List[torch.Tensor]]:
    """One sequence ``tokens`` [T].  Returns, per HF norm / linear name, the captured tensors:
    ``<norm>.normed`` (pre-gain normalised input [T, H]), ``<norm>.out`` (after the gain),
    ``<linear>.in`` (linear input).  ``gains`` overrides norm weights (for re-tracing)."""
    c = cfg
    g = gains or {}
    rec: Dict[str, List[torch.Tensor]] = {}

    def put(k, v):
        rec.setdefault(k, []).append(v.detach().clone())

    t = tokens.shape[0]
    pos = torch.arange(t)
    cos, sin = rope_cos_sin(pos, c.head_dim, c.rope_theta)
    x = w["model.embed_tokens.weight"].float()[tokens.long()]
    for i in range(c.num_layers):
        p = f"model.layers.{i}."
        n1 = p + "input_layernorm.weight"
        nrm = _rms(x, c.rms_norm_eps)
        h = nrm * g.get(n1, w[n1]).float()
        put(n1 + ".normed", nrm)
        put(n1 + ".out", h)
        for lin in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
            put(p + lin + ".in", h)
        q = (h @ w[p + "self_attn.q_proj.weight"].float().T).view(t, c.num_heads, c.head_dim)
        k = (h @ w[p + "self_attn.k_proj.weight"].float().T).view(t, c.num_kv_heads, c.head_dim)
        v = (h @ w[p + "self_attn.v_proj.weight"].float().T).view(t, c.num_kv_heads, c.head_dim)
        a = attention_ref(apply_rope(q, cos, sin), apply_rope(k, cos, sin), v, pos).reshape(t, -1)
        put(p + "self_attn.o_proj.in", a)
        x = x + a @ w[p + "self_attn.o_proj.weight"].float().T
        n2 = p + "post_attention_layernorm.weight"
        nrm = _rms(x, c.rms_norm_eps)
        h = nrm * g.get(n2, w[n2]).float()
        put(n2 + ".normed", nrm)
        put(n2 + ".out", h)
        put(p + "mlp.gate_proj.in", h)
        put(p + "mlp.up_proj.in", h)
        act = torch.nn.functional.silu(h @ w[p + "mlp.gate_proj.weight"].float().T) * \
            (h @ w[p + "mlp.up_proj.weight"].float().T)
        put(p + "mlp.down_proj.in", act)
        x = x + act @ w[p + "mlp.down_proj.weight"].float().T
    return rec
