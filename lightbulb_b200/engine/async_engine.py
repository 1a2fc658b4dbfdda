"""Asynchronous front of the engine for the HTTP server.

The reference hands each HTTP request to one model-runner thread over an mpsc channel and
that thread serves ONE request at a time (``src/engine/model_runner.rs:383-398``).  Here one
background thread runs ``LLMEngine.step()`` continuously; every request submitted from any
asyncio task joins the same continuous batch, and its tokens are streamed back through a
per-request ``asyncio.Queue`` (``loop.call_soon_threadsafe``).

Failure behaviour kept from the reference: a load failure fails every queued request; a
client that disconnects (stream consumer gone) aborts its request and frees its KV blocks.
"""
from __future__ import annotations

import asyncio
import logging
import queue
import threading
import time
import uuid
from dataclasses import dataclass, field
from typing import AsyncIterator, Dict, List, Optional

from .sampling import SamplingParams

log = logging.getLogger("lightbulb_b200.async_engine")


@dataclass
class StreamItem:
    text: str = ""
    token_ids: List[int] = field(default_factory=list)
    finished: bool = False
    finish_reason: Optional[str] = None
    prompt_tokens: int = 0
    completion_tokens: int = 0
    cached_tokens: int = 0
    error: Optional[str] = None


@dataclass
class CompletionResult:
    text: str
    finish_reason: str
    prompt_tokens: int
    completion_tokens: int
    cached_tokens: int = 0


class AsyncEngine:
    def __init__(self, engine, idle_sleep: float = 0.001):
        self.engine = engine
        self._submit: "queue.Queue" = queue.Queue()
        self._streams: Dict[str, tuple] = {}
        self._stop = threading.Event()
        self._idle = idle_sleep
        self.healthy = True
        self.last_error: Optional[str] = None
        self.steps = 0
        self._thread = threading.Thread(target=self._loop, name="lb-engine", daemon=True)
        self._thread.start()

    def call(self, fn):
        """Run ``fn(engine)`` on the engine thread between steps; returns a
        ``concurrent.futures.Future`` (``asyncio.wrap_future`` it from coroutines)."""
        import concurrent.futures
        fut = concurrent.futures.Future()
        if getattr(self, "_plane", None) is not None:
            # would run on rank 0 only: the ranks' engines would diverge (or see one KV shard)
            fut.set_exception(NotImplementedError(
                "engine-thread calls are not available under tensor-parallel serving"))
            return fut
        self._submit.put(("call", (fn, fut)))
        return fut

    def _emit_outputs(self, outs) -> None:
        for o in outs:
            self._emit(o.request_id, StreamItem(o.new_text, o.new_token_ids, o.finished,
                                                o.finish_reason, o.prompt_tokens,
                                                o.completion_tokens, o.cached_tokens))
            if o.finished:
                self.engine.release(o.request_id)     # keep the request table bounded

    def fail(self, reason: str) -> None:
        """Orderly stop after an external failure (e.g. a peer rank died): no further steps;
        every in-flight request finishes with an error; the server reports 503."""
        self.healthy = False
        self.last_error = reason
        self._submit.put(("fail", reason))

    # ---- engine thread ----------------------------------------------------------------
    def attach_control_plane(self, plane) -> None:
        """Tensor-parallel serving: mirror every add / abort to the worker ranks (see
        :mod:`lightbulb_b200.parallel.serving`) so that all ranks step in lockstep."""
        self._plane = plane

    def _loop(self):
        eng = self.engine
        while not self._stop.is_set():
            drained = False
            mirror = []
            while True:
                try:
                    kind, payload = self._submit.get_nowait()
                except queue.Empty:
                    break
                drained = True
                if kind in ("add", "abort"):
                    mirror.append((kind, payload))
                if kind == "add":
                    rid, kw = payload
                    try:
                        eng.add_request(request_id=rid, **kw)
                    except Exception as e:  # invalid request: fail only this one
                        self._emit(rid, StreamItem(finished=True, finish_reason="error",
                                                   error=str(e)))
                elif kind == "abort":
                    eng.abort(payload)
                    eng.release(payload)
                    self._streams.pop(payload, None)
                elif kind == "call":
                    fn, fut = payload
                    try:
                        res = fn(eng)
                        if isinstance(res, dict) and "drained" in res:
                            self._emit_outputs(res.pop("drained"))
                        fut.set_result(res)
                    except Exception as e:
                        fut.set_exception(e)
                elif kind == "fail":
                    for rid in list(self._streams):
                        self._emit(rid, StreamItem(finished=True, finish_reason="error",
                                                   error=payload))
                        eng.abort(rid)
                        eng.release(rid)
            plane = getattr(self, "_plane", None)
            if plane is not None:
                if not self.healthy:
                    plane.publish(None)            # workers stop: nobody steps again
                    self._plane = None
                elif mirror or eng.has_unfinished():
                    # the workers apply the same submissions and step iff this rank steps
                    plane.publish(mirror)
            if not self.healthy:
                # failed: keep draining submissions (each fails at once), never step again
                for rid in list(self._streams):
                    self._emit(rid, StreamItem(finished=True, finish_reason="error",
                                               error=self.last_error))
                    eng.abort(rid)
                    eng.release(rid)
                if not drained:
                    time.sleep(self._idle)
                continue
            if not eng.has_unfinished():
                if not drained:
                    time.sleep(self._idle)
                continue
            try:
                outs = eng.step()
                self.steps += 1
            except Exception as e:  # engine failure: fail every in-flight request
                log.exception("engine step failed")
                self.healthy = False
                self.last_error = repr(e)
                for rid in list(self._streams):
                    self._emit(rid, StreamItem(finished=True, finish_reason="error", error=repr(e)))
                    eng.abort(rid)
                continue
            self._emit_outputs(outs)

    def _emit(self, rid: str, item: StreamItem):
        st = self._streams.get(rid)
        if st is None:
            return
        loop, q = st
        try:
            loop.call_soon_threadsafe(q.put_nowait, item)
        except RuntimeError:  # event loop closed: consumer is gone
            self._streams.pop(rid, None)
            self._submit.put(("abort", rid))
            return
        if item.finished:
            self._streams.pop(rid, None)

    # ---- asyncio side ---------------------------------------------------------------
    async def generate(self, prompt: Optional[str] = None,
                       params: Optional[SamplingParams] = None,
                       prompt_token_ids: Optional[List[int]] = None,
                       add_special_tokens: bool = True, priority: int = 1,
                       request_id: Optional[str] = None) -> AsyncIterator[StreamItem]:
        rid = request_id or uuid.uuid4().hex
        q: asyncio.Queue = asyncio.Queue()
        self._streams[rid] = (asyncio.get_running_loop(), q)
        self._submit.put(("add", (rid, dict(prompt=prompt, params=params,
                                            prompt_token_ids=prompt_token_ids,
                                            add_special_tokens=add_special_tokens,
                                            priority=priority))))
        try:
            while True:
                item = await q.get()
                yield item
                if item.finished:
                    return
        finally:
            if rid in self._streams:  # consumer left early (client disconnect)
                self._streams.pop(rid, None)
                self._submit.put(("abort", rid))

    async def complete(self, **kw) -> CompletionResult:
        text, reason, pt, ct, cached = [], "length", 0, 0, 0
        async for it in self.generate(**kw):
            if it.error:
                raise RuntimeError(it.error)
            text.append(it.text)
            pt, ct, cached = it.prompt_tokens, it.completion_tokens, it.cached_tokens
            if it.finished:
                reason = it.finish_reason or reason
        return CompletionResult("".join(text), reason, pt, ct, cached)

    def shutdown(self):
        self._stop.set()
        self._thread.join(timeout=10)
        plane = getattr(self, "_plane", None)
        if plane is not None:
            plane.publish(None)
            self._plane = None
