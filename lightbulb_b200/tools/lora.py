"""LoRA adapters: load (PEFT and plain layouts), map names, validate, merge into base weights.

Reference: ``src/lora/mod.rs:41-590`` -- load adapters in PEFT or other layouts, map their
tensor names onto the base model, validate shapes, merge ``W += scale * B @ A`` with
``scale = alpha / r``.  PEFT layout: ``adapter_config.json`` (``r``, ``lora_alpha``,
``target_modules``, ``fan_in_fan_out``) and ``adapter_model.safetensors`` with names like
``base_model.model.model.layers.0.self_attn.q_proj.lora_A.weight`` ([r, in]) and ``...lora_B.weight``
([out, r]).  Plain layout: ``<base name>.lora_A`` / ``.lora_B`` (optionally ``.alpha``).
"""
from __future__ import annotations

import json
import os
import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch


@dataclass
class LoraPair:
    a: torch.Tensor          # [r, in]
    b: torch.Tensor          # [out, r]
    alpha: float

    @property
    def r(self) -> int:
        return self.a.shape[0]

    @property
    def scale(self) -> float:
        return self.alpha / self.r


@dataclass
class LoraAdapter:
    pairs: Dict[str, LoraPair] = field(default_factory=dict)   # base weight name -> pair
    config: dict = field(default_factory=dict)


_PEFT = re.compile(r"^(?:base_model\.model\.)?(?P<base>.+?)\.lora_(?P<ab>[AB])(?:\.default)?\.weight$")
_PLAIN = re.compile(r"^(?P<base>.+?)\.lora_(?P<ab>[AB])$")


def map_name(base: str) -> str:
    """Adapter module name -> HF base weight name."""
    base = base[len("base_model.model."):] if base.startswith("base_model.model.") else base
    if not base.startswith("model.") and not base.startswith("lm_head"):
        base = "model." + base
    return base + ".weight"


def from_tensors(tensors: Dict[str, torch.Tensor], alpha: Optional[float] = None,
                 config: Optional[dict] = None) -> LoraAdapter:
    cfg = config or {}
    default_alpha = alpha if alpha is not None else cfg.get("lora_alpha")
    parts: Dict[str, dict] = {}
    for k, v in tensors.items():
        m = _PEFT.match(k) or _PLAIN.match(k)
        if m:
            parts.setdefault(map_name(m.group("base")), {})[m.group("ab")] = v
        elif k.endswith(".alpha"):
            parts.setdefault(map_name(k[:-len(".alpha")]), {})["alpha"] = float(v)
    ad = LoraAdapter(config=cfg)
    fan_in_fan_out = bool(cfg.get("fan_in_fan_out", False))
    for name, p in parts.items():
        if "A" not in p or "B" not in p:
            raise ValueError(f"{name}: lora_A and lora_B must both be present")
        a, b = p["A"], p["B"]
        if fan_in_fan_out:
            a, b = a.t(), b.t()
        al = p.get("alpha", default_alpha if default_alpha is not None else a.shape[0])
        ad.pairs[name] = LoraPair(a.contiguous(), b.contiguous(), float(al))
    return ad


def load_adapter(path: str) -> LoraAdapter:
    from safetensors.torch import load_file
    cfg = {}
    cp = os.path.join(path, "adapter_config.json")
    if os.path.exists(cp):
        with open(cp) as f:
            cfg = json.load(f)
    files = [f for f in os.listdir(path) if f.endswith(".safetensors")]
    if not files:
        raise FileNotFoundError(f"no adapter safetensors in {path}")
    tensors = {}
    for f in sorted(files):
        tensors.update(load_file(os.path.join(path, f)))
    return from_tensors(tensors, config=cfg)


def validate(adapter: LoraAdapter, base: Dict[str, torch.Tensor]) -> List[str]:
    errs = []
    for name, p in adapter.pairs.items():
        if name not in base:
            errs.append(f"{name}: not in the base model")
            continue
        out, inn = base[name].shape
        if p.a.shape[1] != inn or p.b.shape[0] != out or p.b.shape[1] != p.a.shape[0]:
            errs.append(f"{name}: A {tuple(p.a.shape)} / B {tuple(p.b.shape)} vs W {out}x{inn}")
    return errs


def merge(base: Dict[str, torch.Tensor], adapter: LoraAdapter, weight: float = 1.0,
          unmerge: bool = False) -> Dict[str, torch.Tensor]:
    """``W += weight * alpha / r * B @ A`` (fp32 math, result in W's dtype)."""
    errs = validate(adapter, base)
    if errs:
        raise ValueError("; ".join(errs))
    out = dict(base)
    sign = -1.0 if unmerge else 1.0
    for name, p in adapter.pairs.items():
        W = base[name]
        delta = (p.b.float() @ p.a.float()) * (p.scale * weight * sign)
        out[name] = (W.float() + delta).to(W.dtype)
    return out
