"""Weight pruning: Wanda (|W| x input activation norm), N:M structured (2:4), magnitude, with a
JSON manifest, applied to HF weight dicts or to GGUF quantised tensors (dequant -> mask ->
requant).

Reference: ``src/pruning/mod.rs:101-560`` (Wanda / structured / tail pruning, manifest) and
``src/pruning/gguf_application.rs:50-239`` (applying a mask to quantised GGUF tensors).
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

LINEARS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
           "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def wanda_scores(w: torch.Tensor, act_norm: torch.Tensor) -> torch.Tensor:
    """|W_ij| * ||X_j||_2 (W [out, in], act_norm [in])."""
    return w.float().abs() * act_norm.float()[None, :]


def mask_unstructured(scores: torch.Tensor, sparsity: float) -> torch.Tensor:
    """Per output row, drop the ``sparsity`` fraction with the lowest scores."""
    k = int(scores.shape[1] * sparsity)
    mask = torch.ones_like(scores, dtype=torch.bool)
    if k > 0:
        idx = torch.topk(scores, k, dim=1, largest=False).indices
        mask.scatter_(1, idx, False)
    return mask


def mask_nm(scores: torch.Tensor, n: int = 2, m: int = 4) -> torch.Tensor:
    """N:M: in every group of ``m`` consecutive inputs keep the ``n`` highest scores."""
    o, i = scores.shape
    assert i % m == 0
    g = scores.reshape(o, i // m, m)
    keep = torch.topk(g, n, dim=2).indices
    mask = torch.zeros_like(g, dtype=torch.bool)
    mask.scatter_(2, keep, True)
    return mask.reshape(o, i)


@dataclass
class PruneEntry:
    name: str
    method: str
    sparsity: float


@dataclass
class PruneManifest:
    entries: List[PruneEntry] = field(default_factory=list)

    def to_json(self) -> str:
        return json.dumps({"entries": [asdict(e) for e in self.entries]}, indent=1)

    @classmethod
    def from_json(cls, s: str) -> "PruneManifest":
        return cls([PruneEntry(**e) for e in json.loads(s)["entries"]])


def activation_norms(cfg, w, calib: List[torch.Tensor]) -> Dict[str, torch.Tensor]:
    from .calib import trace
    acc: Dict[str, torch.Tensor] = {}
    for t in calib:
        r = trace(cfg, w, t)
        for k, v in r.items():
            if k.endswith(".in"):
                sq = torch.cat(v).pow(2).sum(0)
                acc[k[:-3]] = acc.get(k[:-3], 0) + sq
    return {k: v.sqrt() for k, v in acc.items()}


def prune(cfg, w: Dict[str, torch.Tensor], method: str = "wanda", sparsity: float = 0.5,
          calib: Optional[List[torch.Tensor]] = None, skip_last: int = 0):
    """Returns (pruned weights, manifest).  method: wanda | nm24 | magnitude.  ``skip_last``
    keeps the last layers dense (tail protection)."""
    norms = activation_norms(cfg, w, calib) if method in ("wanda", "nm24") and calib else {}
    out = dict(w)
    man = PruneManifest()
    for i in range(cfg.num_layers - skip_last):
        for lin in LINEARS:
            name = f"model.layers.{i}.{lin}"
            W = w[name + ".weight"]
            an = norms.get(name, torch.ones(W.shape[1]))
            sc = wanda_scores(W, an) if method in ("wanda", "nm24") else W.float().abs()
            mask = mask_nm(sc) if method == "nm24" else mask_unstructured(sc, sparsity)
            out[name + ".weight"] = (W * mask).to(W.dtype)
            man.entries.append(PruneEntry(name + ".weight", method,
                                          1.0 - mask.float().mean().item()))
    return out, man


def map_manifest(man: PruneManifest, tensor_names) -> Dict[str, str]:
    """Manifest entries (HF layer names) -> the names the target checkpoint uses, whatever its
    family (GGUF llama.cpp names, GPT ``h.N`` names or HF names; detected from
    ``tensor_names``, reference ``src/pruning/name_mapping.rs:100-128``).  Entries with no
    counterpart in the checkpoint are left out."""
    from ..formats.name_map import MISTRAL, TensorNameMapper, translate
    names = list(tensor_names)
    dst = TensorNameMapper(names)
    src = TensorNameMapper([e.name for e in man.entries], MISTRAL)
    present = set(names)
    out = {}
    for e in man.entries:
        arch = dst.architecture if dst.architecture in ("llama", "gpt", "mistral") else "llama"
        t = translate(e.name, src, arch)
        if t is not None and t in present:
            out[e.name] = t
    return out


def apply_to_gguf(raw: np.ndarray, ggml_type: int, n: int, k: int, mask: torch.Tensor) -> bytes:
    """Dequantise a GGUF tensor, zero the masked weights and requantise to the same type."""
    from .. import _native as N
    from ..formats import gguf as G
    buf = torch.from_numpy(np.ascontiguousarray(raw).view(np.uint8).copy())
    x = N.dequantize(int(ggml_type), buf, n * k).reshape(n, k)
    return G.quantize(x.float() * mask.float(), ggml_type)
