"""Chat-template resolution and rendering.

Resolution tiers, in order (reference ``src/api/chat_template.rs:759-860``):

1. sidecar ``lightbulb-chat-template.json`` beside the checkpoint (records provenance);
2. GGUF ``tokenizer.chat_template`` metadata;
3. ``tokenizer_config.json`` ``chat_template`` (string, or the list-of-named-templates form
   where the ``default`` entry wins);
4. vocabulary signature: added tokens ``<|im_start|>`` -> ChatML, ``[INST]`` -> Llama-2;
5. family registry by path component, leaf first (tinyllama+chat -> Zephyr, qwen/chatml ->
   ChatML, llama-2/llama2/mistral -> Llama-2);
6. none: the legacy ``"role: content"`` newline join, tokenized WITH special tokens.

Rendering uses jinja2's ``ImmutableSandboxedEnvironment(trim_blocks=True,
lstrip_blocks=True)`` - the dialect HF ``transformers`` compiles chat templates with - plus
``raise_exception`` and ``strftime_now`` (local time), ``add_generation_prompt=True`` and the
checkpoint's bos/eos strings.  A rendered template is tokenized with
``add_special_tokens=False`` (the template already carries them), the legacy join with
``True`` (``src/api/openai/chat.rs:235-271``).
"""
from __future__ import annotations

import datetime
import enum
import hashlib
import json
import os
from dataclasses import asdict, dataclass
from typing import Dict, List, Optional, Sequence

SIDECAR_NAME = "lightbulb-chat-template.json"


class Resolution(str, enum.Enum):
    SIDECAR = "sidecar"
    TOKENIZER_CONFIG = "tokenizer_config"
    GGUF_METADATA = "gguf_metadata"
    VOCAB_SIGNATURE = "vocab_signature"
    REGISTRY = "registry"
    PROBE = "probe"
    NONE = "none"


# Family registry formats (same renderings as the reference registry,
# src/api/chat_template/registry.rs, written as standard Jinja).
ZEPHYR = ("{% for message in messages %}{{ '<|' ~ message['role'] ~ '|>\n' ~ message['content'] "
          "~ eos_token ~ '\n' }}{% endfor %}{% if add_generation_prompt %}"
          "{{ '<|assistant|>\n' }}{% endif %}")
CHATML = ("{% for message in messages %}{{ '<|im_start|>' ~ message['role'] ~ '\n' ~ "
          "message['content'] ~ '<|im_end|>\n' }}{% endfor %}{% if add_generation_prompt %}"
          "{{ '<|im_start|>assistant\n' }}{% endif %}")
LLAMA2 = ("{% for message in messages %}{% if message['role'] == 'user' %}"
          "{{ '[INST] ' ~ message['content'] ~ ' [/INST]' }}{% else %}"
          "{{ message['content'] ~ eos_token }}{% endif %}{% endfor %}")

REGISTRY = {"zephyr": ZEPHYR, "chatml": CHATML, "llama2": LLAMA2}


class TemplateError(RuntimeError):
    pass


def _raise(msg):
    raise TemplateError(msg)


def _strftime_now(fmt: str) -> str:
    return datetime.datetime.now().strftime(fmt)


_env = None


def _jinja_env():
    global _env
    if _env is None:
        from jinja2.sandbox import ImmutableSandboxedEnvironment
        _env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
        _env.globals["raise_exception"] = _raise
        _env.globals["strftime_now"] = _strftime_now
    return _env


@dataclass
class ChatTemplate:
    source: str
    resolved_by: Resolution

    def is_usable(self) -> bool:
        return self.resolved_by != Resolution.NONE and bool(self.source.strip())

    def render(self, messages: Sequence[dict], bos_token: str = "", eos_token: str = "",
               add_generation_prompt: bool = True, **extra) -> str:
        tpl = _jinja_env().from_string(self.source)
        return tpl.render(messages=list(messages), bos_token=bos_token or "",
                          eos_token=eos_token or "", add_generation_prompt=add_generation_prompt,
                          **extra)


@dataclass
class Sidecar:
    template: str
    resolved_by: str
    evidence: str
    resolved_at: str
    model_fingerprint: str


def _digest(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()[:16]


def fingerprint(model_path: str) -> Optional[str]:
    """Identity of a checkpoint: for a single file its name + size + mtime; for a directory
    the digest of its config.json."""
    try:
        if os.path.isfile(model_path):
            st = os.stat(model_path)
            return f"file:{os.path.basename(model_path)}:{st.st_size}:{int(st.st_mtime)}"
        p = os.path.join(model_path, "config.json")
        with open(p, "rb") as f:
            return "config:" + _digest(f.read())
    except OSError:
        return None


def sidecar_path(model_path: str) -> str:
    if os.path.isfile(model_path):
        return model_path + "." + SIDECAR_NAME
    return os.path.join(model_path, SIDECAR_NAME)


def write_sidecar(model_path: str, sc: Sidecar) -> None:
    with open(sidecar_path(model_path), "w") as f:
        json.dump(asdict(sc), f, indent=2)


def read_sidecar(model_path: str) -> Optional[Sidecar]:
    p = sidecar_path(model_path)
    if not os.path.exists(p):
        return None
    try:
        with open(p) as f:
            d = json.load(f)
        sc = Sidecar(**{k: d[k] for k in ("template", "resolved_by", "evidence", "resolved_at",
                                          "model_fingerprint")})
    except Exception:
        return None
    fp = fingerprint(model_path)
    if fp is not None and sc.model_fingerprint and sc.model_fingerprint != fp:
        return None  # sidecar written for a different checkpoint at this path
    if not sc.template.strip():
        return None
    return sc


def _metadata_dir(model_path: str) -> str:
    return os.path.dirname(model_path) if os.path.isfile(model_path) else model_path


def chat_template_field(cfg: dict) -> Optional[str]:
    t = cfg.get("chat_template")
    if isinstance(t, str) and t.strip():
        return t
    if isinstance(t, list):  # [{"name": "default", "template": ...}, ...]
        named = {e.get("name"): e.get("template") for e in t if isinstance(e, dict)}
        d = named.get("default")
        if isinstance(d, str) and d.strip():
            return d
    return None


def from_vocab_signature(meta_dir: str) -> Optional[str]:
    p = os.path.join(meta_dir, "tokenizer.json")
    try:
        with open(p) as f:
            v = json.load(f)
    except Exception:
        return None
    added = [t.get("content") for t in v.get("added_tokens", []) if isinstance(t, dict)]
    if "<|im_start|>" in added:
        return CHATML
    if "[INST]" in added:
        return LLAMA2
    return None


def _from_component(name: str) -> Optional[str]:
    if "tinyllama" in name and "chat" in name:
        return ZEPHYR
    if "qwen" in name or "chatml" in name:
        return CHATML
    if "llama-2" in name or "llama2" in name or "mistral" in name:
        return LLAMA2
    return None


def from_family(model_path: str) -> Optional[str]:
    parts = os.path.normpath(os.path.abspath(model_path)).split(os.sep)
    for comp in reversed(parts):
        t = _from_component(comp.lower())
        if t:
            return t
    return None


def _gguf_template(model_path: str) -> Optional[str]:
    if not (os.path.isfile(model_path) and model_path.endswith(".gguf")):
        return None
    try:
        from ..formats.gguf import GGUFReader
        meta = GGUFReader(model_path).metadata
    except Exception:
        return None
    t = meta.get("tokenizer.chat_template")
    return t if isinstance(t, str) and t.strip() else None


def resolve(model_path: str) -> ChatTemplate:
    sc = read_sidecar(model_path)
    if sc is not None:
        return ChatTemplate(sc.template, Resolution(sc.resolved_by)
                            if sc.resolved_by in Resolution._value2member_map_ else Resolution.SIDECAR)
    g = _gguf_template(model_path)
    if g:
        return ChatTemplate(g, Resolution.GGUF_METADATA)
    meta = _metadata_dir(model_path)
    try:
        with open(os.path.join(meta, "tokenizer_config.json")) as f:
            t = chat_template_field(json.load(f))
        if t:
            return ChatTemplate(t, Resolution.TOKENIZER_CONFIG)
    except Exception:
        pass
    t = from_vocab_signature(meta)
    if t:
        return ChatTemplate(t, Resolution.VOCAB_SIGNATURE)
    t = from_family(model_path)
    if t:
        return ChatTemplate(t, Resolution.REGISTRY)
    return ChatTemplate("", Resolution.NONE)


def legacy_join(messages: Sequence[dict]) -> str:
    return "\n".join(f"{m['role']}: {m['content']}" for m in messages)


@dataclass
class BuiltPrompt:
    text: str
    add_special_tokens: bool


class ResolvedTemplate:
    """A template plus the checkpoint's bos/eos strings, ready for serving."""

    def __init__(self, tpl: ChatTemplate, bos_token: str = "", eos_token: str = ""):
        self.tpl = tpl
        self.bos_token = bos_token
        self.eos_token = eos_token

    @property
    def resolved_by(self) -> Resolution:
        return self.tpl.resolved_by

    def build_prompt(self, messages: Sequence[dict]) -> BuiltPrompt:
        if self.tpl.is_usable():
            try:
                return BuiltPrompt(self.tpl.render(messages, self.bos_token, self.eos_token),
                                   add_special_tokens=False)
            except TemplateError:
                raise
            except Exception:
                pass
        return BuiltPrompt(legacy_join(messages), add_special_tokens=True)


def resolve_for_model(model_path: Optional[str], tokenizer=None) -> ResolvedTemplate:
    tpl = resolve(model_path) if model_path else ChatTemplate("", Resolution.NONE)
    bos = getattr(tokenizer, "bos_token", None) or ""
    eos = getattr(tokenizer, "eos_token", None) or ""
    return ResolvedTemplate(tpl, bos, eos)
