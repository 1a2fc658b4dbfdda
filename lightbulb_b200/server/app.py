"""OpenAI-compatible HTTP server (FastAPI).

Routes and observable behaviour follow the reference (``src/api/mod.rs``,
``src/api/openai/{chat,completions,models}.rs``, ``src/api/admin.rs``, ``src/api/lightbulb.rs``):

* ``POST /v1/chat/completions``: messages -> chat template (``add_special_tokens=False``) or
  the legacy ``role: content`` join (``True``); ``stream`` -> SSE ``chat.completion.chunk``
  frames with the role in the first delta only and a final frame carrying ``finish_reason``
  and an empty delta; errors as ``{"error": {...}}`` frames; ``stream`` together with
  ``lightbulb.output_contract`` -> 400; without a model a canned answer with ``usage: null``;
  defaults ``temperature`` 1.0, ``max_tokens`` 100, ``n`` ignored.
* ``POST /v1/completions``: raw prompt (string or list joined by ``\\n``), ``echo`` prepends
  the prompt with no separator.
* ``/v1/models`` on GET and POST (the reference routes it as POST only): the loaded model.
* ``GET /health`` is never behind auth.  ``GET /metrics``: Prometheus text.
* ``/v1/lightbulb/admin/*`` and ``/v1/lightbulb/{knowledge,reasoning,state,tools}/*``.

Unlike the reference, many concurrent requests share one continuous batch
(:class:`~lightbulb_b200.engine.async_engine.AsyncEngine`).
"""
from __future__ import annotations

import asyncio
import json
import logging
import os
import time
import uuid
from typing import Any, List, Optional, Union

from fastapi import FastAPI, Request
from fastapi.middleware.cors import CORSMiddleware
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..contracts import Completion, ContractSpec, execute_contract
from ..engine.eos_monitor import EosMonitor
from ..engine.sampling import SamplingParams
from ..extras.knowledge import KnowledgeBase
from ..extras.reasoning import ReasoningControls
from ..extras.state import (CheckpointManager, engine_snapshot, restore_engine_state,
                             save_engine_state)
from ..extras.tools import ToolRegistry
from ..templates.chat_template import BuiltPrompt, ResolvedTemplate, legacy_join
from .auth import AuthStore
from .metrics import Metrics

log = logging.getLogger("lightbulb_b200.server")

STREAM_CONTRACT_REJECTION = (
    "`stream: true` cannot be combined with `lightbulb.output_contract`: the contract is "
    "validated (and retried) against the complete answer, so nothing can be streamed before "
    "generation ends. Send `stream: false` to use the contract, or drop the contract to stream.")

PRIORITY = {"low": 0, "normal": 1, "high": 2, "critical": 3}


class AppState:
    def __init__(self, engine=None, template: Optional[ResolvedTemplate] = None,
                 model_name: str = "lightbulb-default", database_url: Optional[str] = None,
                 state_dir: Optional[str] = None):
        self.engine = engine          # AsyncEngine or None
        self.template = template
        self.model_name = model_name
        self.eos = EosMonitor()
        self.metrics = Metrics()
        self.auth = AuthStore(database_url)
        self.kb = KnowledgeBase()
        self.reasoning = ReasoningControls()
        self.tools = ToolRegistry()
        self.ckpt = CheckpointManager(state_dir or os.path.join(
            os.environ.get("TMPDIR", "/tmp"), f"lb_state_{os.getpid()}"))
        self.created = int(time.time())


def _err(status: int, msg: str, typ: str = "invalid_request_error"):
    return JSONResponse(status_code=status, content={"error": {"message": msg, "type": typ}})


def build_prompt(state: AppState, messages: List[dict]) -> BuiltPrompt:
    if state.template is not None:
        return state.template.build_prompt(messages)
    return BuiltPrompt(legacy_join(messages), add_special_tokens=True)


def _sampling(body: dict, default_max: int = 100) -> SamplingParams:
    stop = body.get("stop")
    if isinstance(stop, str):
        stop = [stop]
    return SamplingParams(temperature=float(body.get("temperature", 1.0)),
                          top_p=float(body.get("top_p", 1.0) or 1.0),
                          top_k=int(body.get("top_k", 0) or 0),
                          max_tokens=int(body.get("max_tokens") or default_max),
                          stop=list(stop or []), seed=body.get("seed"))


def create_app(state: Optional[AppState] = None) -> FastAPI:
    state = state or AppState()
    app = FastAPI(title="lightbulb_b200", version="0.1.0")
    app.state.lb = state
    app.add_middleware(CORSMiddleware, allow_origins=["*"], allow_methods=["*"],
                       allow_headers=["*"])

    @app.middleware("http")
    async def auth_rate_audit(request: Request, call_next):
        t0 = time.perf_counter()
        path = request.url.path
        key_hash = None
        open_path = path == "/health" or path.startswith("/.well-known/acme-challenge/")
        if state.auth.enabled and not open_path:
            h = request.headers.get("authorization", "")
            if not h.lower().startswith("bearer "):
                return _err(401, "missing bearer API key", "authentication_error")
            row = state.auth.lookup(h.split(None, 1)[1].strip())
            if row is None:
                return _err(401, "invalid API key", "authentication_error")
            key_hash, role, limit = row
            if path.startswith("/v1/lightbulb/admin") and role != "admin":
                return _err(403, "admin role required", "permission_error")
            if not state.auth.hit(key_hash, limit):
                return _err(429, "rate limit exceeded", "rate_limit_error")
        resp = await call_next(request)
        if state.auth.enabled and not open_path:
            state.auth.audit(key_hash, request.method, path, resp.status_code,
                             (time.perf_counter() - t0) * 1e3)
        return resp

    # ------------------------------------------------------------------------------
    @app.get("/health")
    async def health():
        ok = state.engine is None or state.engine.healthy
        return JSONResponse(status_code=200 if ok else 503,
                            content={"status": "ok" if ok else "unhealthy",
                                     "model_loaded": state.engine is not None,
                                     "error": None if ok else state.engine.last_error})

    @app.get("/.well-known/acme-challenge/{token}")
    async def acme_challenge(token: str):
        from .tls import CHALLENGES
        ka = CHALLENGES.get(token)
        if ka is None:
            return PlainTextResponse("Challenge not found", status_code=404)
        return PlainTextResponse(ka)

    @app.get("/metrics")
    async def metrics():
        eng = state.engine.engine if state.engine is not None else None
        return PlainTextResponse(state.metrics.prometheus(eng))

    async def list_models():
        return {"object": "list", "data": [{"id": state.model_name, "object": "model",
                                            "created": state.created, "owned_by": "lightbulb"}]}

    app.add_api_route("/v1/models", list_models, methods=["GET", "POST"])

    # ------------------------------------------------------------------------------
    async def _run_once(prompt: BuiltPrompt, sp: SamplingParams, priority: int):
        return await state.engine.complete(prompt=prompt.text, params=sp,
                                           add_special_tokens=prompt.add_special_tokens,
                                           priority=priority)

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        state.metrics.count("chat")
        try:
            body = await request.json()
        except Exception:
            return _err(400, "invalid JSON body")
        messages = body.get("messages")
        if not isinstance(messages, list) or not all(isinstance(m, dict) for m in messages):
            return _err(400, "`messages` must be a list of {role, content} objects")
        messages = [{"role": str(m.get("role", "user")), "content": str(m.get("content", ""))}
                    for m in messages]
        lb = body.get("lightbulb") or {}
        contract = lb.get("output_contract")
        stream = bool(body.get("stream", False))
        if stream and contract:
            return JSONResponse(status_code=400, content={"error": STREAM_CONTRACT_REJECTION})
        model = body.get("model", state.model_name)
        sp = _sampling(body, default_max=200 if contract else 100)
        sp.max_tokens = state.reasoning.clamp_max_tokens(sp.max_tokens)
        prio = PRIORITY.get(str((lb.get("metadata") or {}).get("priority", "normal")).lower(), 1)
        if lb.get("use_knowledge_base") and messages:
            facts = state.kb.query(messages[-1]["content"], top_k=3)
            if facts:
                ctx = "\n".join(f"- {f['content']}" for f in facts)
                messages = [{"role": "system", "content": f"Known facts:\n{ctx}"}] + messages
        created = int(time.time())
        cid = f"chatcmpl-{uuid.uuid4()}"

        if state.engine is not None and not state.engine.healthy:
            return _err(503, f"engine unavailable: {state.engine.last_error}", "unavailable")
        if state.engine is None:
            text = f"Received request for model '{model}'. No model available on the server."
            if stream:
                async def canned():
                    words = ["No ", "model ", "runner ", "available. ", "Please ", "configure ",
                             "model ", "path."]
                    for i, w in enumerate(words):
                        d = {"id": cid, "object": "chat.completion.chunk", "created": created,
                             "model": model, "choices": [{"index": 0, "delta": {"content": w},
                                                          "finish_reason": "stop" if i == 7 else None}]}
                        yield f"data: {json.dumps(d)}\n\n"
                    yield "data: [DONE]\n\n"
                return StreamingResponse(canned(), media_type="text/event-stream")
            return {"id": cid, "object": "chat.completion", "created": created, "model": model,
                    "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                                 "finish_reason": "stop"}], "usage": None}

        if contract:
            try:
                spec = ContractSpec.from_dict(contract)
                fallbacks = [ContractSpec.from_dict(f) for f in lb.get("fallback_contracts") or []]
            except ValueError as e:
                return _err(400, str(e))
            import asyncio
            loop = asyncio.get_running_loop()

            def infer(msgs):
                fut = asyncio.run_coroutine_threadsafe(
                    _run_once(build_prompt(state, msgs), sp, prio), loop)
                r = fut.result()
                return Completion(r.text, r.finish_reason, r.prompt_tokens, r.completion_tokens)

            last, usage, result = await loop.run_in_executor(
                None, lambda: execute_contract(messages, spec, infer,
                                               int(lb.get("max_attempts") or 3), fallbacks, model))
            state.eos.record(last.finish_reason, state.template and state.template.resolved_by)
            return {"id": cid, "object": "chat.completion", "created": created, "model": model,
                    "choices": [{"index": 0, "message": {"role": "assistant", "content": last.text},
                                 "finish_reason": last.finish_reason}],
                    "usage": {"prompt_tokens": usage["prompt_tokens"],
                              "completion_tokens": usage["completion_tokens"],
                              "total_tokens": usage["prompt_tokens"] + usage["completion_tokens"]},
                    "lightbulb_result": result}

        prompt = build_prompt(state, messages)
        if not stream:
            try:
                r = await _run_once(prompt, sp, prio)
            except Exception as e:
                state.metrics.errors += 1
                return _err(500, str(e), "internal_error")
            state.eos.record(r.finish_reason, state.template and state.template.resolved_by)
            return {"id": cid, "object": "chat.completion", "created": created, "model": model,
                    "choices": [{"index": 0, "message": {"role": "assistant", "content": r.text},
                                 "finish_reason": r.finish_reason}],
                    "usage": {"prompt_tokens": r.prompt_tokens,
                              "completion_tokens": r.completion_tokens,
                              "total_tokens": r.prompt_tokens + r.completion_tokens,
                              "prompt_tokens_details": {"cached_tokens": r.cached_tokens}}}

        async def sse():
            first = True
            try:
                async for it in state.engine.generate(prompt=prompt.text, params=sp,
                                                      add_special_tokens=prompt.add_special_tokens,
                                                      priority=prio):
                    if it.error:
                        yield "data: " + json.dumps({"error": {"message": it.error,
                                                               "type": "inference_error"}}) + "\n\n"
                        return
                    if it.text or first:
                        delta = {"content": it.text}
                        if first:
                            delta = {"role": "assistant", "content": it.text}
                        first = False
                        d = {"id": cid, "object": "chat.completion.chunk", "created": created,
                             "model": model, "choices": [{"index": 0, "delta": delta,
                                                          "finish_reason": None}]}
                        yield f"data: {json.dumps(d)}\n\n"
                    if it.finished:
                        state.eos.record(it.finish_reason, state.template and
                                         state.template.resolved_by)
                        d = {"id": cid, "object": "chat.completion.chunk", "created": created,
                             "model": model, "choices": [{"index": 0, "delta": {},
                                                          "finish_reason": it.finish_reason}]}
                        yield f"data: {json.dumps(d)}\n\n"
                yield "data: [DONE]\n\n"
            except Exception as e:  # pragma: no cover
                yield "data: " + json.dumps({"error": {"message": str(e),
                                                       "type": "inference_error"}}) + "\n\n"

        return StreamingResponse(sse(), media_type="text/event-stream")

    @app.post("/v1/completions")
    async def completions(request: Request):
        state.metrics.count("completions")
        try:
            body = await request.json()
        except Exception:
            return _err(400, "invalid JSON body")
        p = body.get("prompt", "")
        prompt_text = "\n".join(p) if isinstance(p, list) else str(p)
        model = body.get("model", state.model_name)
        created = int(time.time())
        if state.engine is not None and not state.engine.healthy:
            return _err(503, f"engine unavailable: {state.engine.last_error}", "unavailable")
        if state.engine is None:
            return {"id": f"cmpl-{uuid.uuid4()}", "object": "text_completion", "created": created,
                    "model": model, "choices": [{"text": "No model available on the server.",
                                                 "index": 0, "logprobs": None,
                                                 "finish_reason": "stop"}], "usage": None}
        sp = _sampling(body)
        try:
            r = await _run_once(BuiltPrompt(prompt_text, True), sp, 1)
        except Exception as e:
            return _err(500, str(e), "internal_error")
        text = prompt_text + r.text if body.get("echo") else r.text
        return {"id": f"cmpl-{uuid.uuid4()}", "object": "text_completion", "created": created,
                "model": model, "choices": [{"text": text, "index": 0, "logprobs": None,
                                             "finish_reason": r.finish_reason}],
                "usage": {"prompt_tokens": r.prompt_tokens, "completion_tokens": r.completion_tokens,
                          "total_tokens": r.prompt_tokens + r.completion_tokens}}

    # ------------------------------------------------------------------------------
    # Admin (/v1/lightbulb/admin/*)
    def _eng():
        return state.engine.engine if state.engine is not None else None

    @app.get("/v1/lightbulb/admin/cache/stats")
    async def cache_stats():
        e = _eng()
        if e is None:
            return {"kv_blocks_total": 0, "kv_blocks_free": 0, "prefix_cached_blocks": 0,
                    "prefix_hit_rate": 0.0}
        return {"kv_blocks_total": e.blocks.num_blocks, "kv_blocks_free": e.blocks.num_free_blocks(),
                "prefix_cached_blocks": e.blocks.num_cached_blocks(),
                "prefix_hit_rate": e.blocks.prefix_hit_rate(), "block_size": e.blocks.block_size}

    @app.post("/v1/lightbulb/admin/cache/clear")
    async def cache_clear():
        e = _eng()
        if e is not None:
            e.blocks.reset_prefix_cache()
        return {"cleared": True}

    @app.get("/v1/lightbulb/admin/scheduler/queue")
    async def sched_queue():
        e = _eng()
        if e is None:
            return {"waiting": [], "running": []}
        return {"waiting": [s.request_id for s in list(e.scheduler.waiting)],
                "running": [s.request_id for s in list(e.scheduler.running)]}

    @app.get("/v1/lightbulb/admin/scheduler/stats")
    async def sched_stats():
        e = _eng()
        return state.metrics.snapshot(e)

    @app.get("/v1/lightbulb/admin/metrics")
    async def sys_metrics():
        snap = state.metrics.snapshot(_eng())
        snap["eos_monitor"] = state.eos.snapshot()
        try:
            import torch
            if torch.cuda.is_available():
                free, total = torch.cuda.mem_get_info()
                snap["gpu_memory_used_bytes"] = total - free
                snap["gpu_memory_total_bytes"] = total
        except Exception:
            pass
        return snap

    @app.post("/v1/lightbulb/admin/api-keys")
    async def create_key(request: Request):
        if not state.auth.enabled:
            return _err(503, "API keys need DATABASE_URL (sqlite:///path)", "unavailable")
        body = await request.json()
        key = state.auth.create_key(body.get("name", "key"), body.get("role", "user"),
                                    int(body.get("rate_limit_per_minute", 60)))
        return {"api_key": key}

    # ------------------------------------------------------------------------------
    # Extensions (/v1/lightbulb/*)
    @app.post("/v1/lightbulb/knowledge/query")
    async def kb_query(request: Request):
        b = await request.json()
        return {"results": state.kb.query(b.get("query", ""), int(b.get("top_k", 5)))}

    @app.post("/v1/lightbulb/knowledge/add")
    async def kb_add(request: Request):
        b = await request.json()
        f = state.kb.add(b.get("content", ""), b.get("source", "user"),
                         float(b.get("confidence", 1.0)))
        return {"id": f.id, "added": True}

    @app.post("/v1/lightbulb/knowledge/validate")
    async def kb_validate(request: Request):
        b = await request.json()
        return state.kb.validate(b.get("claim", ""))

    @app.post("/v1/lightbulb/reasoning/budget")
    async def reasoning_budget(request: Request):
        return state.reasoning.set_budget(**(await request.json()))

    @app.get("/v1/lightbulb/reasoning/convergence")
    async def reasoning_convergence(key: str = "default"):
        return state.reasoning.convergence(key)

    @app.get("/v1/lightbulb/reasoning/stats")
    async def reasoning_stats():
        return state.reasoning.stats()

    @app.post("/v1/lightbulb/state/save")
    async def state_save(request: Request):
        b = await request.json()
        e = _eng()
        payload = engine_snapshot(e) if e is not None else {"requests": []}
        payload["knowledge"] = [f.__dict__ for f in state.kb.facts]
        name = b.get("name") or f"ckpt-{int(time.time())}"
        res = state.ckpt.save(name, payload)
        if b.get("include_kv") and state.engine is not None:
            # requests + KV rows of their cached positions, written on the engine thread
            path = state.ckpt.kv_path(name)
            try:
                info = await asyncio.wrap_future(state.engine.call(
                    lambda eng: save_engine_state(eng, path)))
            except NotImplementedError as ex:
                return _err(501, str(ex), "not_implemented")
            res = dict(res, kv=info)
        return res

    @app.post("/v1/lightbulb/state/restore")
    async def state_restore(request: Request):
        b = await request.json()
        try:
            m = state.ckpt.restore(b.get("name", ""))
        except (OSError, ValueError) as ex:
            return _err(404, f"no checkpoint: {ex}")
        for f in m["payload"].get("knowledge", []):
            state.kb.add(f.get("content", ""), f.get("source", "user"), f.get("confidence", 1.0))
        out = {"restored": m["name"], "requests": len(m["payload"].get("requests", []))}
        path = state.ckpt.kv_path(m["name"])
        if b.get("kv") and state.engine is not None and os.path.exists(path):
            try:
                ids = await asyncio.wrap_future(state.engine.call(
                    lambda eng: restore_engine_state(eng, path)))
            except ValueError as ex:
                return _err(409, str(ex))
            except NotImplementedError as ex:
                return _err(501, str(ex), "not_implemented")
            out["resumed"] = ids
        return out

    @app.post("/v1/lightbulb/state/branch")
    async def state_branch(request: Request):
        b = await request.json()
        try:
            return state.ckpt.branch(b.get("source", ""), b.get("name", ""))
        except (OSError, ValueError) as ex:
            return _err(404, f"cannot branch: {ex}")

    @app.get("/v1/lightbulb/state/list")
    async def state_list():
        return {"checkpoints": state.ckpt.list()}

    @app.get("/v1/lightbulb/tools/list")
    async def tools_list():
        return {"tools": state.tools.list()}

    @app.post("/v1/lightbulb/tools/register")
    async def tools_register(request: Request):
        b = await request.json()
        try:
            return state.tools.register(b.get("name", ""), b.get("description", ""),
                                        b.get("parameters"))
        except ValueError as ex:
            return _err(400, str(ex))

    return app
