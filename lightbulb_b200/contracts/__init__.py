"""Output contracts: constrain a chat answer to a parseable shape, re-prompting on failure.

Behaviour of the reference (``src/contracts/mod.rs:79-177``, ``executor.rs:60-300``,
``validation.rs:34-171``, ``enum_choice.rs``, ``tagged_fields.rs``, ``commit_block.rs``):

* four contract kinds: ``enum_choice`` (final line is one of N choices, optionally by
  1-based index), ``tagged_fields`` (``<tag>...</tag>`` fields, some required, some
  repeatable), ``commit_block`` (a sentinel-delimited block, optionally required to be the
  last thing in the answer) and ``json`` (the answer parses as a JSON value);
* the instruction is appended to the system message (or prepended as one);
* an answer that does not parse is retried with a tightening user message, up to
  ``max_attempts``; then the fallback contracts are tried in order;
* the result (type, attempts, parse success, model, latency, parsed output) is returned as
  ``lightbulb_result`` next to the normal chat completion; usage is summed over attempts.

The instruction wording here is this framework's own.
"""
from __future__ import annotations

import json
import re
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional


@dataclass
class ContractSpec:
    type: str
    choices: List[str] = field(default_factory=list)
    case_sensitive: bool = False
    allow_index: bool = True
    allowed_tags: List[str] = field(default_factory=list)
    required_tags: List[str] = field(default_factory=list)
    repeatable_tags: List[str] = field(default_factory=list)
    block_type: str = ""
    must_be_last: bool = True

    @classmethod
    def from_dict(cls, d: dict) -> "ContractSpec":
        t = d.get("type")
        if t not in ("enum_choice", "tagged_fields", "commit_block", "json"):
            raise ValueError(f"unknown output contract type {t!r}")
        kw = {k: d[k] for k in ("choices", "case_sensitive", "allow_index", "allowed_tags",
                                "required_tags", "repeatable_tags", "block_type", "must_be_last")
              if k in d}
        if t == "enum_choice" and not kw.get("choices"):
            raise ValueError("enum_choice needs non-empty choices")
        if t == "commit_block" and not kw.get("block_type"):
            raise ValueError("commit_block needs block_type")
        return cls(type=t, **kw)


# ---------------------------------------------------------------------------------------
# Instructions
# ---------------------------------------------------------------------------------------
def system_instruction(c: ContractSpec) -> str:
    if c.type == "enum_choice":
        opts = " | ".join(f"{i + 1}. {x.upper()}" if c.allow_index else x.upper()
                          for i, x in enumerate(c.choices))
        idx = " Answering with only the number is also accepted." if c.allow_index else ""
        return ("\n\nANSWER FORMAT: think as briefly as you like, then put exactly one of these "
                f"on the LAST line, alone: {opts}.{idx}")
    if c.type == "tagged_fields":
        tags = " ".join(f"<{t.upper()}>...</{t.upper()}>" for t in c.allowed_tags)
        req = f" Required: {', '.join(t.upper() for t in c.required_tags)}." \
            if c.required_tags else ""
        return f"\n\nANSWER FORMAT: give your answer in these tagged fields: {tags}.{req}"
    if c.type == "commit_block":
        u = c.block_type.upper()
        last = " Nothing may follow the block." if c.must_be_last else ""
        return (f"\n\nANSWER FORMAT: write your final result between the lines "
                f"<<<COMMIT:{u} v1>>> and <<<END:{u}>>>.{last}")
    return "\n\nANSWER FORMAT: reply with one valid JSON value and nothing else."


def tightening_message(attempt: int, c: ContractSpec) -> str:
    strict = attempt >= 2
    if c.type == "enum_choice":
        opts = ", ".join(f"{x.upper()} ({i + 1})" if c.allow_index else x.upper()
                         for i, x in enumerate(c.choices))
        return (f"Reply with ONLY one of: {opts}." if strict else
                f"The last line of your answer was not one of the allowed choices. Answer again; "
                f"the final line must be only one of: {opts}")
    if c.type == "tagged_fields":
        tags = " ".join(f"<{t.upper()}></{t.upper()}>" for t in c.allowed_tags)
        return (f"Reply with only the tagged fields {tags}." if strict else
                f"Your answer was missing required tagged fields. Answer again using {tags}.")
    if c.type == "commit_block":
        u = c.block_type.upper()
        return (f"Reply with only <<<COMMIT:{u} v1>>> ... <<<END:{u}>>>." if strict else
                f"Your answer did not contain a complete <<<COMMIT:{u} v1>>> block. Try again.")
    return "Reply with only valid JSON." if strict else "That was not valid JSON. Answer again."


# ---------------------------------------------------------------------------------------
# Parsers
# ---------------------------------------------------------------------------------------
def parse_enum_choice(text: str, c: ContractSpec) -> Optional[str]:
    norm = (lambda s: s) if c.case_sensitive else (lambda s: s.lower())
    table = {norm(x): x for x in c.choices}
    for line in reversed(text.splitlines()):
        cleaned = line.strip().strip("*_`\"'.,:;!()[]").strip()
        if not cleaned:
            continue
        if norm(cleaned) in table:
            return table[norm(cleaned)]
        if c.allow_index and cleaned.isdigit():
            i = int(cleaned)
            if 1 <= i <= len(c.choices):
                return c.choices[i - 1]
        m = re.match(r"^(\d+)[.)]\s*(.+)$", cleaned)
        if m and norm(m.group(2).strip()) in table:
            return table[norm(m.group(2).strip())]
        return None  # only the last non-empty line counts
    return None


def parse_tagged_fields(text: str, c: ContractSpec) -> Dict[str, List[str]]:
    out: Dict[str, List[str]] = {}
    low = text.lower()
    for tag in c.allowed_tags:
        t = tag.lower()
        vals = []
        pos = 0
        while True:
            a = low.find(f"<{t}>", pos)
            if a < 0:
                break
            b = low.find(f"</{t}>", a)
            if b < 0:
                break
            vals.append(text[a + len(t) + 2:b].strip())
            pos = b + len(t) + 3
        if vals:
            out[tag] = vals if tag in c.repeatable_tags else [vals[-1]]
    return out


def parse_commit_block(text: str, c: ContractSpec) -> Optional[str]:
    u = re.escape(c.block_type.upper())
    m = None
    for m in re.finditer(rf"<<<COMMIT:{u} v1>>>(.*?)<<<END:{u}>>>", text, re.S | re.I):
        pass
    if m is None:
        return None
    body = m.group(1).strip()
    if not body:
        return None
    if c.must_be_last and text[m.end():].strip():
        return None
    return body


def try_parse(text: str, c: ContractSpec) -> Optional[Dict[str, Any]]:
    if c.type == "enum_choice":
        ch = parse_enum_choice(text, c)
        return None if ch is None else {"type": "enum_choice", "choice": ch}
    if c.type == "tagged_fields":
        tags = parse_tagged_fields(text, c)
        if not tags or any(r not in tags for r in c.required_tags):
            return None
        return {"type": "tagged_fields", "tags": tags}
    if c.type == "commit_block":
        b = parse_commit_block(text, c)
        return None if b is None else {"type": "commit_block", "block_text": b}
    try:
        s = text.strip()
        if s.startswith("```"):
            s = s.strip("`")
            s = s[4:] if s.lower().startswith("json") else s
        json.loads(s)
        return {"type": "raw", "text": text.strip()}
    except Exception:
        return None


def inject_instruction(messages: List[dict], c: ContractSpec) -> List[dict]:
    msgs = [dict(m) for m in messages]
    ins = system_instruction(c)
    for m in msgs:
        if m.get("role") == "system":
            m["content"] = m.get("content", "") + ins
            return msgs
    return [{"role": "system", "content": ins.lstrip("\n")}] + msgs


@dataclass
class Completion:
    text: str
    finish_reason: str
    prompt_tokens: int = 0
    completion_tokens: int = 0


def execute_contract(messages: List[dict], spec: ContractSpec,
                     infer: Callable[[List[dict]], Completion], max_attempts: int = 3,
                     fallbacks: Optional[List[ContractSpec]] = None, model_id: str = ""):
    """Run the attempt loop.  Returns (final Completion, usage totals, result dict)."""
    t0 = time.perf_counter()
    usage = {"prompt_tokens": 0, "completion_tokens": 0}
    attempts = 0
    last: Optional[Completion] = None
    for c in [spec] + list(fallbacks or []):
        msgs = inject_instruction(messages, c)
        for attempt in range(max(1, max_attempts)):
            attempts += 1
            last = infer(msgs)
            usage["prompt_tokens"] += last.prompt_tokens
            usage["completion_tokens"] += last.completion_tokens
            parsed = try_parse(last.text, c)
            if parsed is not None:
                return last, usage, {
                    "contract_type": c.type, "attempts": attempts, "parse_success": True,
                    "model_id": model_id, "latency_ms": int((time.perf_counter() - t0) * 1e3),
                    "output": parsed}
            msgs = msgs + [{"role": "assistant", "content": last.text},
                           {"role": "user", "content": tightening_message(attempt + 1, c)}]
    return last, usage, {
        "contract_type": spec.type, "attempts": attempts, "parse_success": False,
        "model_id": model_id, "latency_ms": int((time.perf_counter() - t0) * 1e3),
        "output": {"type": "raw", "text": last.text if last else ""}}
