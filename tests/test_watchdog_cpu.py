"""Rank failure detection on the host: heartbeats through a TCP store among spawned processes
(a rank that exits, a rank that stops beating, no failure), and the engine / server side of a
detected failure (in-flight requests fail, the API answers 503).  No GPU involved."""
import asyncio
import datetime
import multiprocessing as mp
import socket
import time

import httpx
import pytest
import torch

from lightbulb_b200.parallel.watchdog import STORE_FAILURE, Watchdog, attach


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, scenario, q):
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=20), wait_for_workers=False)
    store.set(f"ready/{rank}", "1")                 # start together: spawn times differ
    store.wait([f"ready/{r}" for r in range(world)], datetime.timedelta(seconds=60))
    seen = []
    wd = Watchdog(store, rank, world, interval_s=0.1, timeout_s=1.0, startup_timeout_s=30.0,
                  on_failure=lambda dead: seen.append((sorted(dead), time.monotonic())))
    wd.start()
    t0 = time.monotonic()
    if scenario == "exit" and rank == 2:
        time.sleep(0.5)
        wd.stop()
        q.put((rank, "exited", None))
        return
    if scenario == "pause" and rank == 1:
        time.sleep(0.5)
        wd.pause()
    time.sleep(3.5)
    wd.stop()
    first = seen[0] if seen else None
    q.put((rank, first[0] if first else [], round(first[1] - t0, 2) if first else None))
    if rank == 0:
        time.sleep(1.0)          # keep the store up until every other rank has reported


def _run(scenario, world=3):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        r, dead, t = q.get(timeout=60)
        out[r] = (dead, t)
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_rank_exit_is_detected_by_every_survivor():
    out = _run("exit")
    for r in (0, 1):
        dead, t = out[r]
        assert dead == [2], out
        assert 1.0 <= t <= 6.0, out


def test_silent_rank_is_detected():
    out = _run("pause")
    assert out[0][0] == [1] and out[2][0] == [1], out
    assert out[1][0] == [], out          # the paused rank still sees its peers beating


def test_no_failure_no_report():
    out = _run("none")
    assert all(v[0] == [] for v in out.values()), out


def test_peer_that_never_starts_uses_startup_limit():
    class Store:
        def __init__(self):
            self.d = {}

        def add(self, k, v):
            self.d[k] = self.d.get(k, 0) + v
            return self.d[k]
    got = []
    wd = Watchdog(Store(), 0, 2, interval_s=0.05, timeout_s=0.2, startup_timeout_s=0.8,
                  on_failure=got.append).start()
    time.sleep(0.5)
    assert not got                       # not yet: the peer may still be starting
    time.sleep(0.8)
    wd.stop()
    assert got and got[0] == {1}


def test_unreachable_store_counts_as_failure():
    class Dead:
        def add(self, k, v):
            raise ConnectionError("store gone")
    got = []
    wd = Watchdog(Dead(), 1, 2, interval_s=0.05, timeout_s=0.5, on_failure=got.append).start()
    time.sleep(0.3)
    wd.stop()
    assert got and got[0] == {STORE_FAILURE} and not wd.healthy


def test_engine_fail_stops_requests_and_server_503():
    from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
    from lightbulb_b200.engine.async_engine import AsyncEngine
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.models.weights import pack_model, random_weights
    from lightbulb_b200.server.app import AppState, create_app

    cfg = get_preset("tiny-test")
    packed = pack_model(cfg, random_weights(cfg, seed=4, std=0.05), dtype=torch.bfloat16,
                        device="cpu")
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=64, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                  chunk_size=32, max_model_len=512),
                        use_cuda_graphs=False)
    ae = AsyncEngine(LLMEngine(ecfg, packed))

    class Store:                          # in-process store: the peer never beats
        def __init__(self):
            self.d = {}

        def add(self, k, v):
            self.d[k] = self.d.get(k, 0) + v
            return self.d[k]
    wd = attach(ae, Watchdog(Store(), 0, 2, interval_s=0.05, timeout_s=0.3,
                             startup_timeout_s=0.3))

    async def scenario():
        items = []

        async def consume():
            async for it in ae.generate(prompt_token_ids=[5, 6, 7],
                                        params=SamplingParams(max_tokens=10_000,
                                                              ignore_eos=True)):
                items.append(it)
        task = asyncio.ensure_future(consume())
        await asyncio.sleep(0.2)
        wd.start()
        await asyncio.wait_for(task, timeout=20)
        app = create_app(AppState(engine=ae))
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app),
                                     base_url="http://t") as c:
            h = await c.get("/health")
            r = await c.post("/v1/chat/completions",
                             json={"messages": [{"role": "user", "content": "hi"}]})
            r2 = await c.post("/v1/completions", json={"prompt": "hi"})
        return items, h, r, r2

    try:
        items, h, r, r2 = asyncio.new_event_loop().run_until_complete(scenario())
    finally:
        wd.stop()
        ae.shutdown()
    assert items[-1].finished and items[-1].finish_reason == "error"
    assert "rank(s) [1] stopped heartbeating" in (items[-1].error or "")
    assert h.status_code == 503 and r.status_code == 503 and r2.status_code == 503
