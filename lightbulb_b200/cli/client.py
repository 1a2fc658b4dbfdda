"""``lightbulb-cli``: interactive chat client for the HTTP API (reference
``src/bin/lightbulb-cli.rs:15-349``: stream / non-stream, system prompt, temperature,
max tokens, API key).

    python -m lightbulb_b200.cli.client --url http://127.0.0.1:8080 [--stream] [--system S]
"""
from __future__ import annotations

import argparse
import json
import sys

import httpx


def chat_once(url, messages, model="default", stream=False, temperature=1.0, max_tokens=100,
              api_key=None, out=sys.stdout, client=None):
    h = {"Authorization": f"Bearer {api_key}"} if api_key else {}
    body = {"model": model, "messages": messages, "stream": stream,
            "temperature": temperature, "max_tokens": max_tokens}
    c = client or httpx.Client(timeout=600)
    if not stream:
        r = c.post(url.rstrip("/") + "/v1/chat/completions", json=body, headers=h)
        r.raise_for_status()
        text = r.json()["choices"][0]["message"]["content"]
        out.write(text + "\n")
        return text
    text = []
    with c.stream("POST", url.rstrip("/") + "/v1/chat/completions", json=body, headers=h) as r:
        for line in r.iter_lines():
            if not line.startswith("data: ") or line == "data: [DONE]":
                continue
            d = json.loads(line[6:])
            if "error" in d:
                raise RuntimeError(d["error"])
            piece = d["choices"][0]["delta"].get("content") or ""
            text.append(piece)
            out.write(piece)
            out.flush()
    out.write("\n")
    return "".join(text)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="lightbulb-cli")
    ap.add_argument("--url", default="http://127.0.0.1:8080")
    ap.add_argument("--model", default="default")
    ap.add_argument("--stream", action="store_true")
    ap.add_argument("--system", default=None)
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--max-tokens", type=int, default=256)
    ap.add_argument("--api-key", default=None)
    ap.add_argument("--once", default=None, help="send one message and exit")
    a = ap.parse_args(argv)
    msgs = [{"role": "system", "content": a.system}] if a.system else []
    if a.once is not None:
        msgs.append({"role": "user", "content": a.once})
        chat_once(a.url, msgs, a.model, a.stream, a.temperature, a.max_tokens, a.api_key)
        return 0
    while True:
        try:
            line = input("> ")
        except EOFError:
            return 0
        if line.strip() in ("/quit", "/exit"):
            return 0
        msgs.append({"role": "user", "content": line})
        reply = chat_once(a.url, msgs, a.model, a.stream, a.temperature, a.max_tokens, a.api_key)
        msgs.append({"role": "assistant", "content": reply})


if __name__ == "__main__":
    sys.exit(main())
