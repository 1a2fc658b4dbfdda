"""Tool registry and tool-call detection.

* ``ToolRegistry``: tools registered over ``/v1/lightbulb/tools/*`` plus model capability
  detection from tensor names (reference ``src/tools/mod.rs:38-310``: text / vision /
  function-calling signatures in checkpoint tensor names).
* ``ToolCallDetector``: scans generated text for ``<tool_call>``, ``[TOOL_CALL]`` or
  ``<|tool_call|>`` markers (reference ``src/engine/tool_call.rs:30-320``); the engine pauses
  the request in ``AWAITING_TOOL`` and ``LLMEngine.inject_tool_result`` appends the tool's
  answer as a mini-prefill into the preserved KV.
"""
from __future__ import annotations

import json
import re
import threading
from typing import Dict, Iterable, List, Optional

TOOL_PATTERNS = [re.compile(r"<tool_call>(.*?)</tool_call>", re.S),
                 re.compile(r"\[TOOL_CALL\](.*?)\[/TOOL_CALL\]", re.S),
                 re.compile(r"<\|tool_call\|>(.*?)(?:<\|/tool_call\|>|$)", re.S)]


class ToolRegistry:
    def __init__(self):
        self.tools: Dict[str, dict] = {}
        self._lock = threading.Lock()

    def register(self, name: str, description: str = "", parameters: Optional[dict] = None):
        if not name or not re.match(r"^[A-Za-z_][A-Za-z0-9_.-]*$", name):
            raise ValueError("invalid tool name")
        with self._lock:
            self.tools[name] = {"name": name, "description": description,
                                "parameters": parameters or {}}
        return self.tools[name]

    def list(self) -> List[dict]:
        with self._lock:
            return list(self.tools.values())

    @staticmethod
    def detect_capabilities(tensor_names: Iterable[str]) -> List[str]:
        names = list(tensor_names)
        caps = ["text"] if any("embed" in n or "tok_embeddings" in n for n in names) else []
        if any(k in n for n in names for k in ("vision", "visual", "image", "patch_embed")):
            caps.append("vision")
        if any(k in n for n in names for k in ("tool", "function")):
            caps.append("function_calling")
        return caps


class ToolCallDetector:
    def find(self, text: str) -> Optional[dict]:
        for pat in TOOL_PATTERNS:
            m = pat.search(text)
            if m:
                body = m.group(1).strip()
                try:
                    return {"raw": body, "call": json.loads(body)}
                except Exception:
                    return {"raw": body, "call": None}
        return None
