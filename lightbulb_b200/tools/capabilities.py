"""Model capability detection from tensor names and tokenizer metadata.

Reference: ``src/tools/mod.rs:38-310`` (tool registry: text / vision / function-calling
capabilities detected from a checkpoint's tensor names).
"""
from __future__ import annotations

from typing import Iterable, Optional, Set

VISION_MARKERS = ("vision_tower", "vision_model", "visual.", "image_newline", "mm_projector",
                  "multi_modal_projector", "patch_embed")
AUDIO_MARKERS = ("audio_tower", "audio_encoder", "whisper")
TOOL_TOKENS = ("<tool_call>", "[TOOL_CALLS]", "<|tool_call|>", "<|python_tag|>", "[TOOL_CALL]")


def detect(tensor_names: Iterable[str], chat_template: Optional[str] = None,
           added_tokens: Iterable[str] = ()) -> Set[str]:
    names = list(tensor_names)
    caps: Set[str] = set()
    if any(n.startswith(("model.embed_tokens", "token_embd")) or "lm_head" in n or
           n == "output.weight" for n in names):
        caps.add("text")
    if any(m in n for n in names for m in VISION_MARKERS):
        caps.add("vision")
    if any(m in n for n in names for m in AUDIO_MARKERS):
        caps.add("audio")
    toks = set(added_tokens)
    tmpl = chat_template or ""
    if any(t in toks or t in tmpl for t in TOOL_TOKENS) or "tools" in tmpl:
        caps.add("function_calling")
    if any(".experts." in n or "block_sparse_moe" in n for n in names):
        caps.add("mixture_of_experts")
    return caps
