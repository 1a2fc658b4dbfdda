"""HTTP API tests without a socket (httpx ASGI transport) over a tiny CPU engine."""
import asyncio
import json
import os

import httpx
import pytest
import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.async_engine import AsyncEngine
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.models.weights import pack_model, random_weights
from lightbulb_b200.server.app import AppState, create_app
from lightbulb_b200.templates.chat_template import ChatTemplate, CHATML, Resolution, ResolvedTemplate


@pytest.fixture(scope="module")
def engine():
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=2, std=0.05)
    packed = pack_model(cfg, w, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=128, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=128,
                                                  chunk_size=64, max_model_len=512),
                        use_cuda_graphs=False)
    ae = AsyncEngine(LLMEngine(ecfg, packed))
    yield ae
    ae.shutdown()


def _client(state):
    app = create_app(state)
    return httpx.AsyncClient(transport=httpx.ASGITransport(app=app), base_url="http://t")


def run(coro):
    return asyncio.new_event_loop().run_until_complete(coro)


def test_health_and_models_without_model():
    async def go():
        async with _client(AppState()) as c:
            r = await c.get("/health")
            assert r.status_code == 200 and r.json()["model_loaded"] is False
            for m in ("GET", "POST"):
                r = await c.request(m, "/v1/models")
                assert r.json()["object"] == "list"
            r = await c.post("/v1/chat/completions", json={"model": "x", "messages": [
                {"role": "user", "content": "hi"}]})
            j = r.json()
            assert j["usage"] is None and j["choices"][0]["finish_reason"] == "stop"
            r = await c.post("/v1/completions", json={"model": "x", "prompt": "hi"})
            assert r.json()["usage"] is None
    run(go())


def test_chat_nonstream_and_stream(engine):
    tpl = ResolvedTemplate(ChatTemplate(CHATML, Resolution.REGISTRY), "<s>", "</s>")
    state = AppState(engine, tpl, model_name="tiny")

    async def go():
        async with _client(state) as c:
            body = {"model": "tiny", "messages": [{"role": "user", "content": "hello"}],
                    "max_tokens": 5, "temperature": 0}
            r = await c.post("/v1/chat/completions", json=body)
            j = r.json()
            assert r.status_code == 200
            assert j["object"] == "chat.completion"
            assert j["usage"]["completion_tokens"] <= 5
            assert j["choices"][0]["finish_reason"] in ("stop", "length")
            body["stream"] = True
            r = await c.post("/v1/chat/completions", json=body)
            frames = [l[6:] for l in r.text.splitlines() if l.startswith("data: ")]
            assert frames[-1] == "[DONE]"
            chunks = [json.loads(f) for f in frames[:-1]]
            assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
            assert all("role" not in ch["choices"][0]["delta"] for ch in chunks[1:])
            assert chunks[-1]["choices"][0]["delta"] == {}
            assert chunks[-1]["choices"][0]["finish_reason"] in ("stop", "length")
            assert all(ch["object"] == "chat.completion.chunk" for ch in chunks)
    run(go())


def test_stream_with_contract_is_400(engine):
    async def go():
        async with _client(AppState(engine)) as c:
            r = await c.post("/v1/chat/completions", json={
                "model": "m", "stream": True, "messages": [{"role": "user", "content": "x"}],
                "lightbulb": {"output_contract": {"type": "json"}}})
            assert r.status_code == 400 and "output_contract" in r.json()["error"]
    run(go())


def test_completions_echo_and_list_prompt(engine):
    async def go():
        async with _client(AppState(engine)) as c:
            r = await c.post("/v1/completions", json={"model": "m", "prompt": ["ab", "cd"],
                                                      "max_tokens": 3, "echo": True,
                                                      "temperature": 0})
            j = r.json()
            assert j["choices"][0]["text"].startswith("ab\ncd")
            assert j["usage"]["completion_tokens"] <= 3
    run(go())


def test_concurrent_requests_share_batch(engine):
    async def go():
        async with _client(AppState(engine)) as c:
            reqs = [c.post("/v1/completions", json={"model": "m", "prompt": f"p{i}",
                                                    "max_tokens": 8, "temperature": 0})
                    for i in range(6)]
            rs = await asyncio.gather(*reqs)
            assert all(r.status_code == 200 for r in rs)
    run(go())


def test_contract_enum_choice_roundtrip(engine):
    async def go():
        async with _client(AppState(engine)) as c:
            r = await c.post("/v1/chat/completions", json={
                "model": "m", "messages": [{"role": "user", "content": "yes or no?"}],
                "max_tokens": 4, "temperature": 0,
                "lightbulb": {"output_contract": {"type": "enum_choice", "choices": ["yes", "no"]},
                              "max_attempts": 2}})
            j = r.json()
            res = j["lightbulb_result"]
            assert res["contract_type"] == "enum_choice" and res["attempts"] == 2
            assert res["parse_success"] is False  # random weights cannot follow it
            assert j["usage"]["completion_tokens"] > 0
    run(go())


def test_auth_rate_limit_and_admin(tmp_path, engine):
    state = AppState(engine, database_url=f"sqlite:///{tmp_path}/auth.db")
    key = state.auth.create_key("t", role="admin", rate_limit=3)

    async def go():
        async with _client(state) as c:
            assert (await c.get("/health")).status_code == 200
            assert (await c.get("/v1/models")).status_code == 401
            h = {"Authorization": f"Bearer {key}"}
            assert (await c.get("/v1/lightbulb/admin/cache/stats", headers=h)).status_code == 200
            assert (await c.get("/v1/models", headers=h)).status_code == 200
            assert (await c.get("/v1/models", headers=h)).status_code == 200
            assert (await c.get("/v1/models", headers=h)).status_code == 429
    run(go())


def test_extension_routes(tmp_path, engine):
    state = AppState(engine, state_dir=str(tmp_path / "ckpt"))

    async def go():
        async with _client(state) as c:
            await c.post("/v1/lightbulb/knowledge/add", json={"content": "paris is in france"})
            r = await c.post("/v1/lightbulb/knowledge/query", json={"query": "where is paris"})
            assert r.json()["results"]
            assert (await c.post("/v1/lightbulb/knowledge/validate",
                                 json={"claim": "paris is in france"})).json()["supported"]
            assert (await c.post("/v1/lightbulb/reasoning/budget",
                                 json={"max_tokens": 7})).json()["max_tokens"] == 7
            assert "budget" in (await c.get("/v1/lightbulb/reasoning/stats")).json()
            assert (await c.post("/v1/lightbulb/state/save", json={"name": "a"})).status_code == 200
            assert (await c.post("/v1/lightbulb/state/branch",
                                 json={"source": "a", "name": "b"})).json()["parent"] == "a"
            names = [m["name"] for m in (await c.get("/v1/lightbulb/state/list")).json()["checkpoints"]]
            assert names == ["a", "b"]
            assert (await c.post("/v1/lightbulb/state/restore", json={"name": "b"})).status_code == 200
            await c.post("/v1/lightbulb/tools/register", json={"name": "calc", "description": "x"})
            assert (await c.get("/v1/lightbulb/tools/list")).json()["tools"][0]["name"] == "calc"
            m = await c.get("/metrics")
            assert "lb_kv_blocks_total" in m.text
            assert 'lb_ttft_seconds_bucket{le="+Inf"}' in m.text and "lb_itl_seconds_count" in m.text
    run(go())


def test_metrics_histograms_are_cumulative():
    from lightbulb_b200.server.metrics import ITL_BUCKETS, _histogram
    lines = _histogram("lb_itl_seconds", [0.0005, 0.003, 0.003, 0.07, 2.0], ITL_BUCKETS)
    assert lines[0] == "# TYPE lb_itl_seconds histogram"
    buckets = [int(l.rsplit(" ", 1)[1]) for l in lines if "_bucket" in l]
    assert buckets == sorted(buckets) and buckets[0] == 1 and buckets[-1] == 5
    assert 'lb_itl_seconds_bucket{le="0.005"} 3' in lines
    assert "lb_itl_seconds_count 5" in lines


def test_latency_samples_bounded_window_cumulative_counts():
    from lightbulb_b200.engine.llm_engine import ITL_BUCKETS, LatencySamples
    from lightbulb_b200.server.metrics import _histogram_cumulative
    st = LatencySamples(ITL_BUCKETS, window=100)
    for i in range(1000):
        st.append(0.003 if i % 2 else 0.07)
    assert len(st) == 100 and st.total == 1000          # memory bounded, counts are not
    lines = _histogram_cumulative("lb_itl_seconds", st)
    assert 'lb_itl_seconds_bucket{le="0.005"} 500' in lines
    assert 'lb_itl_seconds_bucket{le="+Inf"} 1000' in lines
    assert sorted(st)[0] == 0.003                         # quantiles over the window still work


def test_async_engine_releases_finished_requests(engine):
    from lightbulb_b200.engine.sampling import SamplingParams

    async def go():
        for i in range(3):
            async for _ in engine.generate(prompt_token_ids=[5, 6, 7 + i],
                                           params=SamplingParams(max_tokens=3,
                                                                 ignore_eos=True)):
                pass
    run(go())
    import time
    time.sleep(0.2)
    assert not [r for r, s in engine.engine.seqs.items() if s.finished]


def test_acme_config_cached_certificate_fallback_and_challenge(tmp_path, monkeypatch):
    """ACME (reference src/tls.rs:252-300,387-450): configuration from the environment, a valid
    cached pair is used as is, otherwise a self-signed fallback for the first domain; HTTP-01
    challenge tokens are served without authentication."""
    from cryptography import x509
    from cryptography.x509.oid import NameOID
    from lightbulb_b200.config import ServerConfig
    from lightbulb_b200.server import tls
    monkeypatch.setenv("LIGHTBULB_TLS_ACME_DOMAINS", "example.test, www.example.test")
    monkeypatch.setenv("LIGHTBULB_TLS_ACME_EMAIL", "ops@example.test")
    monkeypatch.setenv("LIGHTBULB_TLS_ACME_CERT_DIR", str(tmp_path / "acme"))
    sc = ServerConfig.from_env()
    assert sc.tls_acme.domains == ["example.test", "www.example.test"]
    kw = tls.ssl_kwargs(sc)
    with open(kw["ssl_certfile"], "rb") as f:
        c = x509.load_pem_x509_certificate(f.read())
    assert c.subject.get_attributes_for_oid(NameOID.COMMON_NAME)[0].value == "example.test"
    # a valid cached ACME pair takes precedence over the fallback
    cert, key = tls.self_signed(str(tmp_path / "issued"), common_name="example.test")
    os.makedirs(tmp_path / "acme", exist_ok=True)
    os.replace(cert, tmp_path / "acme" / "acme_cert.pem")
    os.replace(key, tmp_path / "acme" / "acme_key.pem")
    assert tls.ssl_kwargs(sc)["ssl_certfile"] == str(tmp_path / "acme" / "acme_cert.pem")
    st = AppState(database_url="sqlite://:memory:")      # auth on: challenges stay open
    assert st.auth.enabled
    tls.CHALLENGES.add("tok123", "tok123.thumbprint")

    async def go():
        async with _client(st) as c:
            r = await c.get("/.well-known/acme-challenge/tok123")
            assert r.status_code == 200 and r.text == "tok123.thumbprint"
            r = await c.get("/.well-known/acme-challenge/other")
            assert r.status_code == 404
    try:
        run(go())
    finally:
        tls.CHALLENGES.remove("tok123")
