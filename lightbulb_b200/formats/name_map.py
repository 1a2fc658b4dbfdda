"""Architecture detection and tensor-name mapping across checkpoint naming families.

Offline tools (pruning, LoRA, norm tweaking) address transformer weights abstractly --
"layer 5, attention query" -- while checkpoints name them per family.  This module detects the
family from a checkpoint's tensor names and maps between abstract components and concrete
names, as the reference's ``TensorNameMapper`` does (``src/pruning/name_mapping.rs:67-260``):

* LLaMA-style GGUF (``blk.N.attn_q.weight`` ...; also Qwen, Mistral and Qwen3 GGUF files,
  which use the same llama.cpp names, plus ``attn_q_norm`` / ``attn_k_norm`` for Qwen3);
* GPT-style (``h.N.attn.c_attn.weight``, fused q/k/v; ``h.N.mlp.c_fc`` / ``c_proj``);
* HF-style "Mistral" family (``model.layers.N.self_attn.q_proj.weight`` ...), which also covers
  HF Llama / Qwen2 / Qwen3 safetensors.

Detection order and the fallback follow the reference's observable behaviour: GGUF LLaMA
names first, then GPT, then HF layer names, else unknown (mapped with the LLaMA table).
Abstract names: ``layer_N`` (the layer's attention query) or ``layer_N.<component>`` with
components ``attention.query|key|value|output``, ``attn.q|k|v|output``, ``ffn.gate|up|down``,
and (an extension) ``attention.norm``, ``ffn.norm``, ``attention.q_norm|k_norm``.
"""
from __future__ import annotations

import re
from typing import Dict, Iterable, List, Optional, Tuple

LLAMA, GPT, MISTRAL, UNKNOWN = "llama", "gpt", "mistral", "unknown"

COMPONENTS = ("attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down",
              "attn_norm", "ffn_norm", "q_norm", "k_norm")

# Per family: layer-index pattern, and per component the name suffix after the layer prefix.
# GPT fuses q/k/v into one tensor, so the three components map to the same name.
_TABLES: Dict[str, Tuple[str, str, Dict[str, str]]] = {
    LLAMA: (r"^blk\.(\d+)\.", "blk.{i}.", {
        "attn_q": "attn_q.weight", "attn_k": "attn_k.weight", "attn_v": "attn_v.weight",
        "attn_o": "attn_output.weight", "ffn_gate": "ffn_gate.weight",
        "ffn_up": "ffn_up.weight", "ffn_down": "ffn_down.weight",
        "attn_norm": "attn_norm.weight", "ffn_norm": "ffn_norm.weight",
        "q_norm": "attn_q_norm.weight", "k_norm": "attn_k_norm.weight"}),
    GPT: (r"(?:^|\.)h\.(\d+)\.", "h.{i}.", {
        "attn_q": "attn.c_attn.weight", "attn_k": "attn.c_attn.weight",
        "attn_v": "attn.c_attn.weight", "attn_o": "attn.c_proj.weight",
        "ffn_up": "mlp.c_fc.weight", "ffn_down": "mlp.c_proj.weight",
        "attn_norm": "ln_1.weight", "ffn_norm": "ln_2.weight"}),
    MISTRAL: (r"(?:^|\.)layers\.(\d+)\.", "model.layers.{i}.", {
        "attn_q": "self_attn.q_proj.weight", "attn_k": "self_attn.k_proj.weight",
        "attn_v": "self_attn.v_proj.weight", "attn_o": "self_attn.o_proj.weight",
        "ffn_gate": "mlp.gate_proj.weight", "ffn_up": "mlp.up_proj.weight",
        "ffn_down": "mlp.down_proj.weight", "attn_norm": "input_layernorm.weight",
        "ffn_norm": "post_attention_layernorm.weight",
        "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight"}),
}

_ABSTRACT = {
    ("attention", "query"): "attn_q", ("attn", "q"): "attn_q",
    ("attention", "key"): "attn_k", ("attn", "k"): "attn_k",
    ("attention", "value"): "attn_v", ("attn", "v"): "attn_v",
    ("attention", "output"): "attn_o", ("attn", "output"): "attn_o",
    ("ffn", "gate"): "ffn_gate", ("ffn", "up"): "ffn_up", ("ffn", "down"): "ffn_down",
    ("attention", "norm"): "attn_norm", ("ffn", "norm"): "ffn_norm",
    ("attention", "q_norm"): "q_norm", ("attention", "k_norm"): "k_norm",
}


def detect_architecture(names: Iterable[str]) -> str:
    names = list(names)
    if any(n.startswith("blk.") and ".attn_q" in n for n in names):
        return LLAMA
    if any(re.search(r"(?:^|\.)h\.\d+\.attn\.c_attn", n) for n in names):
        return GPT
    if any(re.search(r"(?:^|\.)layers\.\d+\.self_attn\.", n) for n in names):
        return MISTRAL
    return UNKNOWN


def parse_abstract(name: str) -> Optional[Tuple[int, str]]:
    """``layer_N`` -> (N, attn_q); ``layer_N.a.b`` -> (N, component) or None."""
    head, _, rest = name.partition(".")
    if not head.startswith("layer_"):
        return None
    try:
        idx = int(head[len("layer_"):])
    except ValueError:
        return None
    if not rest:
        return idx, "attn_q"
    comp = _ABSTRACT.get(tuple(rest.split(".")))
    return (idx, comp) if comp else None


class TensorNameMapper:
    """Mapping (layer, component) <-> concrete tensor name for one checkpoint."""

    def __init__(self, names: Iterable[str], architecture: Optional[str] = None):
        names = list(names)
        self.architecture = architecture or detect_architecture(names)
        pat, self._prefix, self._suffix = _TABLES.get(self.architecture, _TABLES[LLAMA])
        self._layer_re = re.compile(pat)
        self.mappings: Dict[Tuple[int, str], str] = {}
        seen = set()
        for n in names:
            hit = self.parse_tensor_name(n)
            if hit is None:
                continue
            i, comps = hit
            for c in comps:
                self.mappings.setdefault((i, c), n)
            seen.add(i)
        self.layer_indices: List[int] = sorted(seen)

    def parse_tensor_name(self, name: str) -> Optional[Tuple[int, List[str]]]:
        """(layer index, components) of a concrete name (GPT's fused c_attn has three)."""
        m = self._layer_re.search(name)
        if m is None:
            return None
        rest = name[m.end():]
        comps = [c for c, suf in self._suffix.items() if rest == suf]
        return (int(m.group(1)), comps) if comps else None

    @staticmethod
    def from_tensor_names(names: Iterable[str]) -> "TensorNameMapper":
        return TensorNameMapper(names)

    def map_name(self, abstract: str) -> Optional[str]:
        hit = parse_abstract(abstract)
        return self.mappings.get(hit) if hit else None

    def concrete(self, layer: int, component: str) -> str:
        """The name this family gives (layer, component), whether or not it is present."""
        if component not in self._suffix:
            raise KeyError(f"{self.architecture} has no {component}")
        return self._prefix.format(i=layer) + self._suffix[component]

    def map_layer(self, layer: int) -> List[Tuple[str, str]]:
        """The projections of one layer present in the checkpoint, in a fixed order."""
        order = ("attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down")
        return [(c, self.mappings[(layer, c)]) for c in order if (layer, c) in self.mappings]

    def get_layer_tensors(self, layer: int) -> List[str]:
        return sorted({n for (i, _c), n in self.mappings.items() if i == layer})


def translate(name: str, src: TensorNameMapper, dst_architecture: str) -> Optional[str]:
    """Rename one layer tensor from ``src``'s family to another family (None when the
    destination has no such component or the name is not a layer tensor)."""
    hit = src.parse_tensor_name(name)
    if hit is None:
        return None
    i, comps = hit
    _pat, prefix, suffix = _TABLES[dst_architecture]
    for c in comps:
        if c in suffix:
            return prefix.format(i=i) + suffix[c]
    return None
