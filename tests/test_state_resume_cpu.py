"""Engine state with KV: save mid-generation, restore into a fresh engine, finish; the tokens
must equal an uninterrupted run (greedy, same weights)."""
import pytest
import torch

from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig, get_preset
from lightbulb_b200.engine.llm_engine import LLMEngine
from lightbulb_b200.engine.sampling import SamplingParams
from lightbulb_b200.extras.state import restore_engine_state, save_engine_state
from lightbulb_b200.models.weights import pack_model, random_weights

CFG = get_preset("tiny-test")
W = random_weights(CFG, seed=9, std=0.05)
PROMPTS = [list(range(3, 40)), [7, 8, 9], [100] * 25]


def _engine(overlap=True):
    packed = pack_model(CFG, W, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=CFG, cache=CacheConfig(num_blocks=96, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=64,
                                                  chunk_size=32, max_model_len=256),
                        use_cuda_graphs=False, overlap_decode=overlap)
    return LLMEngine(ecfg, packed)


def _finish(eng):
    while eng.has_unfinished():
        eng.step()


@pytest.mark.parametrize("include_kv", [True, False])
def test_save_restore_resumes_identically(tmp_path, include_kv):
    sp = [SamplingParams(temperature=0.0, max_tokens=m, ignore_eos=True) for m in (20, 12, 30)]
    ref = _engine()
    rs = [ref.add_request(f"r{i}", prompt_token_ids=p, params=s)
          for i, (p, s) in enumerate(zip(PROMPTS, sp))]
    _finish(ref)

    a = _engine()
    for i, (p, s) in enumerate(zip(PROMPTS, sp)):
        a.add_request(f"r{i}", prompt_token_ids=p, params=s)
    for _ in range(8):
        a.step()                                   # mid-decode, overlapped step in flight
    info = save_engine_state(a, str(tmp_path / "snap.lbkv"), include_kv=include_kv)
    assert info["requests"] == 3 and (info["kv_tensors"] == 3) == include_kv
    partial = {rid: list(s.output_token_ids) for rid, s in a.seqs.items()}
    assert all(0 < len(v) < 30 for v in partial.values())

    b = _engine()
    ids = restore_engine_state(b, str(tmp_path / "snap.lbkv"))
    assert sorted(ids) == ["r0", "r1", "r2"]
    if include_kv:
        assert all(b.seqs[r].num_computed_tokens > 0 for r in ids)
        assert not b.scheduler.waiting
    _finish(b)
    for i, s in enumerate(rs):
        got = b.seqs[f"r{i}"]
        assert got.output_token_ids == s.output_token_ids, i
        assert got.finish_reason == "length"
    b.blocks.check_invariants()


def test_restore_rejects_other_model_shape(tmp_path):
    a = _engine()
    a.add_request("x", prompt_token_ids=[1, 2, 3], params=SamplingParams(max_tokens=5))
    a.step()
    save_engine_state(a, str(tmp_path / "s.lbkv"))
    other = get_preset("tiny-test", num_layers=3)
    packed = pack_model(other, random_weights(other, seed=1), dtype=torch.bfloat16, device="cpu")
    b = LLMEngine(EngineConfig(model=other, cache=CacheConfig(num_blocks=32, block_size=16),
                               scheduler=SchedulerConfig(max_model_len=128),
                               use_cuda_graphs=False), packed)
    with pytest.raises(ValueError, match="different model shape"):
        restore_engine_state(b, str(tmp_path / "s.lbkv"))


def test_state_routes_save_and_resume_with_kv(tmp_path):
    import asyncio

    import httpx

    from lightbulb_b200.engine.async_engine import AsyncEngine
    from lightbulb_b200.server.app import AppState, create_app

    a = _engine()
    a.add_request("keep", prompt_token_ids=PROMPTS[0],
                  params=SamplingParams(temperature=0.0, max_tokens=200, ignore_eos=True))
    for _ in range(4):
        a.step()
    ae = AsyncEngine(a)
    b = AsyncEngine(_engine())
    try:
        async def go():
            app = create_app(AppState(engine=ae, state_dir=str(tmp_path)))
            app2 = create_app(AppState(engine=b, state_dir=str(tmp_path)))
            async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app),
                                         base_url="http://t") as c:
                r = await c.post("/v1/lightbulb/state/save",
                                 json={"name": "snap1", "include_kv": True})
            async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app2),
                                         base_url="http://t") as c:
                r2 = await c.post("/v1/lightbulb/state/restore", json={"name": "snap1", "kv": True})
            return r, r2
        r, r2 = asyncio.new_event_loop().run_until_complete(go())
    finally:
        ae.shutdown()
        b.shutdown()
    assert r.status_code == 200 and r.json()["kv"]["kv_tensors"] == 1
    assert r2.status_code == 200 and r2.json()["resumed"] == ["keep"]


def test_engine_calls_refused_under_tp_serving():
    from lightbulb_b200.engine.async_engine import AsyncEngine
    ae = AsyncEngine(_engine())

    class Plane:                       # stands in for the control plane
        def publish(self, msgs):
            pass
    ae.attach_control_plane(Plane())
    try:
        fut = ae.call(lambda eng: 1)
        with pytest.raises(NotImplementedError):
            fut.result(timeout=5)
    finally:
        ae.shutdown()
