"""Chat-template tiers, rendering dialect, sidecar/probe logic, CLIs (CPU)."""
import json
import os

import pytest
import torch

from lightbulb_b200.templates import chat_template as T


MSGS = [{"role": "system", "content": "sys"}, {"role": "user", "content": "hi"}]


def test_registry_renderings():
    z = T.ChatTemplate(T.ZEPHYR, T.Resolution.REGISTRY).render(MSGS, "<s>", "</s>")
    assert z == "<|system|>\nsys</s>\n<|user|>\nhi</s>\n<|assistant|>\n"
    c = T.ChatTemplate(T.CHATML, T.Resolution.REGISTRY).render(MSGS)
    assert c == "<|im_start|>system\nsys<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n" \
                "<|im_start|>assistant\n"
    l2 = T.ChatTemplate(T.LLAMA2, T.Resolution.REGISTRY).render(
        [{"role": "user", "content": "a"}, {"role": "assistant", "content": "b"}], "", "</s>")
    assert l2 == "[INST] a [/INST]b</s>"


def test_trim_lstrip_blocks_and_helpers():
    # trim_blocks drops the newline after a block tag, lstrip_blocks the indent before one
    src = "{% for m in messages %}\n  {% if true %}{{ m['content'] }},{% endif %}\n{% endfor %}"
    assert T.ChatTemplate(src, T.Resolution.TOKENIZER_CONFIG).render(MSGS) == "sys,hi,"
    with pytest.raises(T.TemplateError):
        T.ChatTemplate("{{ raise_exception('bad role') }}", T.Resolution.PROBE).render(MSGS)
    out = T.ChatTemplate("{{ strftime_now('%Y') }}", T.Resolution.PROBE).render(MSGS)
    assert out.isdigit()


def test_tier_order(tmp_path):
    d = tmp_path / "TinyLlama-1.1B-Chat"
    d.mkdir()
    (d / "config.json").write_text("{}")
    assert T.resolve(str(d)).resolved_by == T.Resolution.REGISTRY
    (d / "tokenizer.json").write_text(json.dumps({"added_tokens": [{"content": "<|im_start|>"}]}))
    r = T.resolve(str(d))
    assert r.resolved_by == T.Resolution.VOCAB_SIGNATURE and r.source == T.CHATML
    (d / "tokenizer_config.json").write_text(json.dumps(
        {"chat_template": [{"name": "tool_use", "template": "x"},
                           {"name": "default", "template": "{{ 'D' }}"}]}))
    r = T.resolve(str(d))
    assert r.resolved_by == T.Resolution.TOKENIZER_CONFIG and r.render(MSGS) == "D"
    T.write_sidecar(str(d), T.Sidecar("{{ 'S' }}", "probe", "e", "now", T.fingerprint(str(d))))
    r = T.resolve(str(d))
    assert r.resolved_by == T.Resolution.PROBE and r.render(MSGS) == "S"
    (d / "config.json").write_text('{"changed": 1}')   # different checkpoint: sidecar ignored
    assert T.resolve(str(d)).resolved_by == T.Resolution.TOKENIZER_CONFIG


def test_build_prompt_special_token_rule(tmp_path):
    none = T.ResolvedTemplate(T.ChatTemplate("", T.Resolution.NONE))
    bp = none.build_prompt(MSGS)
    assert bp.text == "system: sys\nuser: hi" and bp.add_special_tokens is True
    rt = T.ResolvedTemplate(T.ChatTemplate(T.CHATML, T.Resolution.REGISTRY))
    assert rt.build_prompt(MSGS).add_special_tokens is False


def test_probe_selection_and_refusals(tmp_path):
    from lightbulb_b200.cli import probe as P
    d = tmp_path / "m"
    d.mkdir()
    (d / "config.json").write_text("{}")
    calls = []

    def gen(text):
        calls.append(text)
        stopped = text.startswith("<|im_start|>")
        return ("4\n", stopped, 3)

    r = P.run_probe(str(d), gen, "<s>", "</s>", [2])
    assert r["winner"] == "chatml" and len(calls) == 3
    assert T.resolve(str(d)).resolved_by == T.Resolution.PROBE
    with pytest.raises(RuntimeError):
        P.run_probe(str(d), gen, "<s>", "</s>", [])          # no EOS declared
    with pytest.raises(RuntimeError):
        P.run_probe(str(d), lambda t: ("x", True, 1), "", "", [2])  # several fire
    (d / "tokenizer_config.json").write_text(json.dumps({"chat_template": "{{ 'x' }}"}))
    os.remove(T.sidecar_path(str(d)))
    with pytest.raises(RuntimeError):
        P.run_probe(str(d), gen, "", "", [2])                 # checkpoint declares a template
    assert P.run_probe(str(d), gen, "", "", [2], force=True)["winner"] == "chatml"


def test_local_llama_gen_cpu(tmp_path):
    from lightbulb_b200.cli.local_gen import local_llama_generate
    from lightbulb_b200.config import get_preset
    from lightbulb_b200.models.reference import ReferenceLlama, greedy_generate
    from lightbulb_b200.models.weights import random_weights, save_checkpoint
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=9, std=0.05)
    save_checkpoint(str(tmp_path / "m"), cfg, w)
    r = local_llama_generate(str(tmp_path / "m"), "", sample_len=6, prompt_ids=[1, 2, 3, 4])
    ref = greedy_generate(ReferenceLlama(cfg, w), [1, 2, 3, 4], 6, eos_ids=cfg.eos_ids())
    assert r["tokens"] == ref
    r2 = local_llama_generate(str(tmp_path / "m"), "", sample_len=6, temperature=0.8,
                              top_p=0.9, seed=1, prompt_ids=[1, 2, 3, 4])
    r3 = local_llama_generate(str(tmp_path / "m"), "", sample_len=6, temperature=0.8,
                              top_p=0.9, seed=1, prompt_ids=[1, 2, 3, 4])
    assert r2["tokens"] == r3["tokens"]  # seeded


def test_contract_parsers():
    from lightbulb_b200.contracts import ContractSpec, try_parse, execute_contract, Completion
    e = ContractSpec.from_dict({"type": "enum_choice", "choices": ["yes", "no"]})
    assert try_parse("thinking...\n**NO**", e)["choice"] == "no"
    assert try_parse("2", e)["choice"] == "no"
    assert try_parse("yes\nand more", e) is None
    t = ContractSpec.from_dict({"type": "tagged_fields", "allowed_tags": ["a", "b"],
                                "required_tags": ["a"], "repeatable_tags": ["b"]})
    p = try_parse("<A>1</A><b>x</b><b>y</b>", t)
    assert p["tags"] == {"a": ["1"], "b": ["x", "y"]}
    assert try_parse("<b>x</b>", t) is None
    c = ContractSpec.from_dict({"type": "commit_block", "block_type": "plan"})
    assert try_parse("pre <<<COMMIT:PLAN v1>>>\nstep\n<<<END:PLAN>>>  ", c)["block_text"] == "step"
    assert try_parse("<<<COMMIT:PLAN v1>>>s<<<END:PLAN>>> trailing", c) is None
    j = ContractSpec.from_dict({"type": "json"})
    assert try_parse('{"a": 1}', j) is not None and try_parse("{a", j) is None
    answers = iter(["maybe", "YES"])
    last, usage, res = execute_contract([{"role": "user", "content": "q"}], e,
                                        lambda m: Completion(next(answers), "stop", 3, 2))
    assert res["parse_success"] and res["attempts"] == 2 and usage["completion_tokens"] == 4
    assert res["output"]["choice"] == "yes"
