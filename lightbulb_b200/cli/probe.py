"""``lightbulb-probe``: determine a chat template empirically and persist it as a sidecar.

Reference: ``src/bin/lightbulb-probe.rs`` + ``src/api/chat_template.rs:1151-1430``.  For each
family-registry candidate the probe renders a short conversation, generates greedily, and
records whether generation stopped on EOS.  Exactly one candidate stopping on EOS wins and is
written to ``lightbulb-chat-template.json`` (resolved_by = probe, with the evidence); zero or
several winners write nothing.  The probe refuses when the checkpoint declares no EOS token,
and refuses to override a template the checkpoint itself declares (tokenizer_config / GGUF)
unless ``--force``.

    python -m lightbulb_b200.cli.probe MODEL_PATH [--force] [--max-tokens 48]
"""
from __future__ import annotations

import argparse
import datetime
import sys
from dataclasses import dataclass
from typing import Callable, List, Optional

from ..templates.chat_template import (REGISTRY, ChatTemplate, Resolution, Sidecar, fingerprint,
                                       resolve, write_sidecar)

PROBE_MESSAGES = [{"role": "user", "content": "Reply with one short sentence: what is 2 + 2?"}]


@dataclass
class ProbeRow:
    candidate: str
    stopped_on_eos: bool
    tokens_generated: int
    first_line: str


def first_line_of(text: str) -> str:
    for line in text.splitlines():
        if line.strip():
            return line.strip()[:120]
    return ""


def select_winner(rows: List[ProbeRow]) -> ProbeRow:
    fired = [r for r in rows if r.stopped_on_eos]
    if len(fired) == 1:
        return fired[0]
    if not fired:
        raise RuntimeError("no candidate stopped on EOS; nothing was written")
    raise RuntimeError(f"{len(fired)} candidates stopped on EOS "
                       f"({', '.join(r.candidate for r in fired)}); nothing was written")


def override_check(current: Resolution, force: bool) -> Optional[str]:
    """None = proceed; otherwise the refusal reason."""
    if current in (Resolution.TOKENIZER_CONFIG, Resolution.GGUF_METADATA) and not force:
        return (f"the checkpoint declares its own template ({current.value}); "
                "pass --force to override it with a probe result")
    return None


def run_probe(model_path: str, generate: Callable[[str], tuple], bos: str, eos: str,
              eos_ids: List[int], force: bool = False) -> dict:
    """generate(prompt_text) -> (text, stopped_on_eos, n_tokens)."""
    if not eos_ids:
        raise RuntimeError("checkpoint declares no EOS token: a probe cannot measure anything")
    reason = override_check(resolve(model_path).resolved_by, force)
    if reason:
        raise RuntimeError(reason)
    rows = []
    for name, src in REGISTRY.items():
        text = ChatTemplate(src, Resolution.PROBE).render(PROBE_MESSAGES, bos, eos)
        out, stopped, n = generate(text)
        rows.append(ProbeRow(name, stopped, n, first_line_of(out)))
    report = "\n".join(f"{r.candidate:8s} eos={'yes' if r.stopped_on_eos else 'no ':3s} "
                       f"tokens={r.tokens_generated:4d} | {r.first_line}" for r in rows)
    win = select_winner(rows)
    sc = Sidecar(template=REGISTRY[win.candidate], resolved_by=Resolution.PROBE.value,
                 evidence=f"probe: only '{win.candidate}' stopped on EOS "
                          f"({win.tokens_generated} tokens)",
                 resolved_at=datetime.datetime.now(datetime.timezone.utc).isoformat(),
                 model_fingerprint=fingerprint(model_path) or "")
    write_sidecar(model_path, sc)
    return {"winner": win.candidate, "report": report}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="lightbulb-probe")
    ap.add_argument("model_path")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--max-tokens", type=int, default=48)
    ap.add_argument("--device", default="cuda")
    a = ap.parse_args(argv)
    from ..config import EngineConfig, SchedulerConfig
    from ..engine.llm_engine import LLMEngine
    from ..engine.sampling import SamplingParams
    eng = LLMEngine.from_pretrained(a.model_path, EngineConfig(
        scheduler=SchedulerConfig(max_num_seqs=4, max_model_len=2048)), device=a.device)
    tok = eng.tokenizer

    def gen(text):
        s = eng.generate(prompt_token_ids=[tok.encode(text, False)],
                         params=SamplingParams(temperature=0.0, max_tokens=a.max_tokens))[0]
        return tok.decode(s.output_token_ids), s.finish_reason == "stop", len(s.output_token_ids)

    try:
        r = run_probe(a.model_path, gen, tok.bos_token or "", tok.eos_token or "",
                      sorted(eng.eos_ids), a.force)
    except RuntimeError as e:
        print(f"lightbulb-probe: {e}", file=sys.stderr)
        return 1
    print(r["report"])
    print(f"winner: {r['winner']} (sidecar written)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
