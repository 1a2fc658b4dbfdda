"""Tokenizers.

* :class:`HFTokenizer` wraps the HF ``tokenizers`` Rust core (the same library the reference
  links, ``Cargo.toml:129``) loaded from ``tokenizer.json``; special tokens (bos/eos) come
  from the checkpoint's ``tokenizer_config.json`` / ``config.json``.
* :class:`GGUFTokenizer` builds a tokenizer from the ``tokenizer.ggml.*`` metadata of a GGUF
  file (reference: ``src/gguf/mod.rs`` tokenizer extraction).
* :class:`ByteTokenizer` is a dependency-free byte-level tokenizer used for random-init
  checkpoints that ship no vocabulary (ids 0..2 are specials, 3..258 are bytes).
"""
from __future__ import annotations

import json
import os
from typing import List, Optional


class BaseTokenizer:
    bos_token_id: Optional[int] = None
    eos_token_ids: List[int] = []
    bos_token: Optional[str] = None
    eos_token: Optional[str] = None
    added_tokens: List[str] = []

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        raise NotImplementedError

    def decode(self, ids: List[int], skip_special_tokens: bool = True) -> str:
        raise NotImplementedError

    @property
    def vocab_size(self) -> int:
        raise NotImplementedError


class ByteTokenizer(BaseTokenizer):
    PAD, BOS, EOS = 0, 1, 2
    OFFSET = 3

    def __init__(self, vocab_size: int = 512):
        self._v = vocab_size
        self.bos_token_id = self.BOS
        self.eos_token_ids = [self.EOS]
        self.bos_token = "<s>"
        self.eos_token = "</s>"

    @property
    def vocab_size(self) -> int:
        return self._v

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return ([self.BOS] if add_special_tokens else []) + ids

    def decode(self, ids: List[int], skip_special_tokens: bool = True) -> str:
        bs = bytes(i - self.OFFSET for i in ids if self.OFFSET <= i < 256 + self.OFFSET)
        return bs.decode("utf-8", errors="replace")


class HFTokenizer(BaseTokenizer):
    def __init__(self, path: str, config: Optional[dict] = None):
        from tokenizers import Tokenizer
        tj = path if path.endswith(".json") else os.path.join(path, "tokenizer.json")
        self.tok = Tokenizer.from_file(tj)
        d = os.path.dirname(tj)
        tcfg = {}
        p = os.path.join(d, "tokenizer_config.json")
        if os.path.exists(p):
            with open(p) as f:
                tcfg = json.load(f)
        self.config = tcfg

        def tok_str(v):
            if isinstance(v, dict):
                return v.get("content")
            return v

        self.bos_token = tok_str(tcfg.get("bos_token"))
        self.eos_token = tok_str(tcfg.get("eos_token"))
        self.bos_token_id = self.tok.token_to_id(self.bos_token) if self.bos_token else None
        eos = []
        if self.eos_token and self.tok.token_to_id(self.eos_token) is not None:
            eos.append(self.tok.token_to_id(self.eos_token))
        if config:
            e = config.get("eos_token_id")
            for x in (e if isinstance(e, list) else [e]):
                if isinstance(x, int) and x not in eos:
                    eos.append(x)
            if self.bos_token_id is None and isinstance(config.get("bos_token_id"), int):
                self.bos_token_id = config["bos_token_id"]
        self.eos_token_ids = eos
        self.added_tokens = [t.content for t in self.tok.get_added_tokens_decoder().values()] \
            if hasattr(self.tok, "get_added_tokens_decoder") else []

    @property
    def vocab_size(self) -> int:
        return self.tok.get_vocab_size()

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        return self.tok.encode(text, add_special_tokens=add_special_tokens).ids

    def decode(self, ids: List[int], skip_special_tokens: bool = True) -> str:
        return self.tok.decode(ids, skip_special_tokens=skip_special_tokens)


class GGUFTokenizer(BaseTokenizer):
    """Greedy longest-match tokenizer over a GGUF vocabulary (SentencePiece-style '▁')."""

    def __init__(self, meta: dict):
        self.tokens: List[str] = list(meta.get("tokenizer.ggml.tokens", []))
        self.index = {t: i for i, t in enumerate(self.tokens)}
        self.bos_token_id = meta.get("tokenizer.ggml.bos_token_id")
        eos = meta.get("tokenizer.ggml.eos_token_id")
        self.eos_token_ids = [eos] if eos is not None else []
        self.bos_token = self.tokens[self.bos_token_id] if self.bos_token_id is not None and \
            self.bos_token_id < len(self.tokens) else None
        self.eos_token = self.tokens[eos] if eos is not None and eos < len(self.tokens) else None
        types = meta.get("tokenizer.ggml.token_type", [])
        self.special = {i for i, t in enumerate(types) if t in (3, 4)}  # control / user-defined
        self.added_tokens = [self.tokens[i] for i in sorted(self.special)]
        self.maxlen = max((len(t) for t in self.tokens), default=1)
        self.chat_template = meta.get("tokenizer.chat_template")

    @property
    def vocab_size(self) -> int:
        return len(self.tokens)

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        s = "▁" + text.replace(" ", "▁")
        out = [self.bos_token_id] if add_special_tokens and self.bos_token_id is not None else []
        i = 0
        while i < len(s):
            for L in range(min(self.maxlen, len(s) - i), 0, -1):
                tid = self.index.get(s[i:i + L])
                if tid is not None:
                    out.append(tid)
                    i += L
                    break
            else:
                b = s[i].encode("utf-8")
                for byte in b:
                    tid = self.index.get(f"<0x{byte:02X}>")
                    if tid is not None:
                        out.append(tid)
                i += 1
        return out

    def decode(self, ids: List[int], skip_special_tokens: bool = True) -> str:
        parts = []
        bbuf = bytearray()
        for i in ids:
            if i < 0 or i >= len(self.tokens) or (skip_special_tokens and i in self.special):
                continue
            t = self.tokens[i]
            if t.startswith("<0x") and t.endswith(">") and len(t) == 6:
                bbuf.append(int(t[3:5], 16))
                continue
            if bbuf:
                parts.append(bbuf.decode("utf-8", errors="replace"))
                bbuf = bytearray()
            parts.append(t.replace("▁", " "))
        if bbuf:
            parts.append(bbuf.decode("utf-8", errors="replace"))
        s = "".join(parts)
        return s[1:] if s.startswith(" ") else s


def load_tokenizer(path: Optional[str], vocab_size: int = 512,
                   config: Optional[dict] = None) -> BaseTokenizer:
    if path and os.path.isdir(path) and os.path.exists(os.path.join(path, "tokenizer.json")):
        return HFTokenizer(path, config)
    if path and path.endswith(".json") and os.path.exists(path):
        return HFTokenizer(path, config)
    return ByteTokenizer(vocab_size)


class IncrementalDetokenizer:
    """Emits the newly decoded suffix after each token (streaming)."""

    def __init__(self, tok: BaseTokenizer):
        self.tok = tok
        self.ids: List[int] = []
        self.text = ""

    def push(self, token_id: int) -> str:
        self.ids.append(token_id)
        full = self.tok.decode(self.ids)
        if full.endswith("�"):  # incomplete UTF-8 sequence: wait for more bytes
            return ""
        delta = full[len(self.text):] if full.startswith(self.text) else full
        self.text = full
        return delta
