"""Norm tweaking: recalibrate RMSNorm gains after weight quantisation.

Reference: ``src/quantization/norm_tweaking.rs:18-270`` -- collect activation statistics of the
unquantised and the quantised model on calibration samples, then adjust each normalisation
layer's scale so the quantised model's post-norm activations match the unquantised ones
(learning rate and a few steps per layer), layer by layer.

Here each gain is solved in closed form per channel: with n the quantised model's normalised
(pre-gain) input and t the unquantised model's post-norm output at the same place,
g_c = sum(n_c * t_c) / sum(n_c^2) minimises ||n * g - t||^2.  ``lr`` < 1 blends the solution into
the current gain (the reference's update step); layers are processed in order and the quantised
model is re-traced after each layer so later layers see the tweaked earlier ones.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Sequence

import torch

from ..config import ModelConfig
from .calib import trace


@dataclass
class NormTweakingConfig:
    lr: float = 1.0
    steps: int = 1
    targets: Sequence[str] = ("input_layernorm", "post_attention_layernorm")


@dataclass
class NormStats:
    name: str
    mean_float: float
    std_float: float
    mean_quant: float
    std_quant: float

    def shift_magnitude(self) -> float:
        return abs(self.mean_float - self.mean_quant) + abs(self.std_float - self.std_quant)


def _norm_names(cfg: ModelConfig, targets) -> List[str]:
    out = []
    for i in range(cfg.num_layers):
        for t in ("input_layernorm", "post_attention_layernorm"):
            if t in targets:
                out.append(f"model.layers.{i}.{t}.weight")
    return out


def collect_statistics(cfg, w_float, w_quant, calib: List[torch.Tensor], targets=None):
    targets = targets or NormTweakingConfig.targets
    rf = [trace(cfg, w_float, t) for t in calib]
    rq = [trace(cfg, w_quant, t) for t in calib]
    stats = []
    for n in _norm_names(cfg, targets):
        a = torch.cat([torch.cat(r[n + ".out"]) for r in rf])
        b = torch.cat([torch.cat(r[n + ".out"]) for r in rq])
        stats.append(NormStats(n, a.mean().item(), a.std().item(), b.mean().item(),
                               b.std().item()))
    return stats


def tweak(cfg: ModelConfig, w_float: Dict[str, torch.Tensor], w_quant: Dict[str, torch.Tensor],
          calib: List[torch.Tensor], config: NormTweakingConfig = None) -> Dict[str, torch.Tensor]:
    """Returns new gains {norm weight name: tensor} for the quantised model."""
    c = config or NormTweakingConfig()
    targets = [n for n in _norm_names(cfg, c.targets)]
    rf = [trace(cfg, w_float, t) for t in calib]
    gains: Dict[str, torch.Tensor] = {}
    for name in targets:
        for _ in range(max(1, c.steps)):
            rq = [trace(cfg, w_quant, t, gains) for t in calib]
            n = torch.cat([torch.cat(r[name + ".normed"]) for r in rq])
            tgt = torch.cat([torch.cat(r[name + ".out"]) for r in rf])
            sol = (n * tgt).sum(0) / (n * n).sum(0).clamp_min(1e-12)
            cur = gains.get(name, w_quant[name].float())
            gains[name] = cur + c.lr * (sol - cur)
    return gains


def apply(w: Dict[str, torch.Tensor], gains: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    out = dict(w)
    for k, v in gains.items():
        out[k] = v.to(w[k].dtype)
    return out
