"""``local-llama-gen``: offline CPU generation, fp32 (reference ``src/lib.rs:48-130``
``local_llama_generate`` and the clap front-end ``src/main.rs.bak:33-98``).

    python -m lightbulb_b200.cli.local_gen --model-dir DIR --prompt "..." --sample-len 16 \
        [--temperature 0] [--top-p 0.9] [--seed 42]

Loads the checkpoint (safetensors / GGUF / AWQ) in fp32 on the CPU, encodes the prompt with
special tokens, runs the first step over the whole prompt and then one token at a time with a
KV cache, samples (argmax when temperature <= 0, else temperature / top-p with a seeded RNG),
stops on EOS and decodes token by token.  This is BASELINE config 1 and the CPU oracle.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from typing import List, Optional

import torch


def local_llama_generate(model_dir: str, prompt: str, sample_len: int = 16,
                         temperature: float = 0.0, top_p: Optional[float] = None,
                         seed: int = 42, prompt_ids: Optional[List[int]] = None,
                         stream=None):
    from ..engine.sampling import sample_row_reference, splitmix64
    from ..models.loader import detect_format, load_awq_weights, load_gguf_weights, load_hf_weights
    from ..models.reference import ReferenceLlama, greedy_argmax
    from ..engine.tokenizer import ByteTokenizer, load_tokenizer
    fmt = detect_format(model_dir)
    tok = None
    if fmt == "gguf":
        cfg, w, tok, _ = load_gguf_weights(model_dir)
    elif fmt == "awq":
        cfg, w, _, _ = load_awq_weights(model_dir)
    else:
        cfg, w = load_hf_weights(model_dir)
    if tok is None:
        cfgd = {}
        if os.path.isdir(model_dir):
            with open(os.path.join(model_dir, "config.json")) as f:
                cfgd = json.load(f)
        tok = load_tokenizer(model_dir if os.path.isdir(model_dir) else None, cfg.vocab_size, cfgd)
    model = ReferenceLlama(cfg, {k: v.float() for k, v in w.items()})
    ids = list(prompt_ids) if prompt_ids is not None else tok.encode(prompt, True)
    eos = set(cfg.eos_ids()) | set(tok.eos_token_ids or [])
    out: List[int] = []
    text = ""
    t0 = time.perf_counter()
    times = []
    logits = model.forward(torch.tensor(ids))
    for i in range(sample_len):
        ts = time.perf_counter()
        row = logits[-1]
        if temperature <= 0:
            nxt = greedy_argmax(row)
        else:
            nxt = sample_row_reference(row, temperature, 0, top_p if top_p else 1.0,
                                       splitmix64(seed + i))
        out.append(nxt)
        piece = tok.decode([nxt])
        text += piece
        if stream is not None:
            stream(piece)
        if nxt in eos:
            break
        logits = model.forward(torch.tensor([nxt]))
        times.append(time.perf_counter() - ts)
    return {"tokens": out, "text": text, "prompt_tokens": len(ids),
            "seconds": time.perf_counter() - t0,
            "ms_per_token": 1e3 * sum(times) / max(1, len(times))}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="local-llama-gen")
    ap.add_argument("--model-dir", required=True)
    ap.add_argument("--prompt", default="Hello")
    ap.add_argument("--sample-len", type=int, default=16)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-p", type=float, default=None)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--threads", type=int, default=0)
    a = ap.parse_args(argv)
    if a.threads:
        torch.set_num_threads(a.threads)
    r = local_llama_generate(a.model_dir, a.prompt, a.sample_len, a.temperature, a.top_p, a.seed,
                             stream=lambda s: (sys.stdout.write(s), sys.stdout.flush()))
    print()
    print(json.dumps({k: r[k] for k in ("tokens", "prompt_tokens", "seconds", "ms_per_token")}),
          file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
