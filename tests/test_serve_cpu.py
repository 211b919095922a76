"""HTTP serving on CPU: OpenAI-compatible completions/chat/streaming against the engine's own output,
sleep/wake, metrics, and the least-in-flight proxy with park/unpark over two in-process replicas."""
import json

import httpx
import pytest
import torch
from starlette.testclient import TestClient

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import greedy_generate
from phung5_b200.models.llama import pack_weights
from phung5_b200.models.reference import RefModel
from phung5_b200.serve.router import LoadBalancedClient, affinity_key, build_proxy
from phung5_b200.serve.server import AsyncEngine, build_app
from phung5_b200.serve.tokenizer import ByteTokenizer
from phung5_b200.weights.init import random_weights


def _engine():
    tcfg, dcfg = preset("tiny"), preset("tiny-draft")
    tw, dw = random_weights(tcfg, seed=0, std=0.05), random_weights(dcfg, seed=1, std=0.05)
    cfg = EngineConfig(model=tcfg, spec=SpecConfig(mode="chain", num_draft=3), draft=DraftConfig(kind="model"),
                       cache=CacheConfig(page_size=16, num_pages=256))
    eng = LLMEngine(cfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", dtype=torch.float32),
                    drafter=pack_weights(dcfg, dw, "cpu", dtype=torch.float32), dtype=torch.float32, max_context=1024)
    return eng, RefModel(tcfg, tw)


@pytest.fixture(scope="module")
def served():
    eng, ref = _engine()
    aeng = AsyncEngine(eng)
    app = build_app(aeng, ByteTokenizer(), "tiny")
    with TestClient(app) as c:
        yield c, ref, aeng
    aeng.shutdown()


def test_completion_token_ids_match_greedy(served):
    c, ref, _ = served
    prompt = list(range(10, 50))
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 12, "temperature": 0, "ignore_eos": True})
    assert r.status_code == 200
    out = r.json()["choices"][0]["token_ids"]
    assert out == greedy_generate(ref, prompt, 12)
    assert r.json()["usage"]["completion_tokens"] == 12


def test_stream_equals_non_stream(served):
    c, _, _ = served
    body = {"prompt": list(range(60, 90)), "max_tokens": 10, "temperature": 0, "ignore_eos": True}
    full = c.post("/v1/completions", json=body).json()["choices"][0]["token_ids"]
    toks = []
    with c.stream("POST", "/v1/completions", json={**body, "stream": True}) as r:
        for line in r.iter_lines():
            if line.startswith("data: ") and line != "data: [DONE]":
                toks += json.loads(line[6:])["choices"][0]["token_ids"]
    assert toks == full


def test_chat_health_load_metrics(served):
    c, _, _ = served
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 5})
    assert r.status_code == 200 and r.json()["choices"][0]["message"]["role"] == "assistant"
    assert c.get("/health").status_code == 200
    assert set(c.get("/get_load").json()) == {"num_running", "num_waiting"}
    assert "phx_generated_tokens_total" in c.get("/metrics").text
    assert c.get("/v1/models").json()["data"][0]["id"] == "tiny"


def test_sleep_wake_roundtrip(served):
    c, ref, aeng = served
    assert c.post("/sleep").json()["sleeping"] is True
    assert c.get("/health").status_code == 503
    assert c.post("/wake_up").json()["sleeping"] is False
    assert c.get("/health").status_code == 200
    prompt = list(range(100, 140))
    out = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 8}).json()["choices"][0]["token_ids"]
    assert out == greedy_generate(ref, prompt, 8)


def test_proxy_least_inflight_and_park():
    apps, aengs = [], []
    for _ in range(2):
        eng, _ = _engine()
        a = AsyncEngine(eng)
        aengs.append(a)
        apps.append(build_app(a, ByteTokenizer(), "tiny"))
    mounts = {f"http://up{i}": httpx.ASGITransport(app=apps[i]) for i in range(2)}
    inner = httpx.AsyncClient(mounts=mounts, timeout=60)
    proxy = build_proxy(["http://up0", "http://up1"], client=inner)
    with TestClient(proxy) as c:
        for _ in range(4):
            assert c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 2}).status_code == 200
        st = c.get("/lb_stats").json()
        assert st["sent"]["http://up0"] == 2 and st["sent"]["http://up1"] == 2   # ties alternate
        assert c.post("/park", json={"upstreams": ["http://up1"]}).json()["ok"]
        assert aengs[1].engine.sleeping
        for _ in range(3):
            assert c.post("/v1/completions", json={"prompt": [4, 5], "max_tokens": 2}).status_code == 200
        assert c.get("/lb_stats").json()["sent"]["http://up1"] == 2
        assert c.post("/unpark", json={"upstreams": ["http://up1"]}).json()["ok"]
        assert not aengs[1].engine.sleeping
    for a in aengs:
        a.shutdown()


def test_load_balanced_client_affinity_and_migration():
    lb = LoadBalancedClient(["http://a", "http://b"], weights=[1, 1], migrate_margin=2)
    tok = affinity_key.set("task-1")
    i = lb.pick_index()
    assert lb.pick_index() == i           # sticky
    lb.inflight[i] = 5                    # its replica gets busy -> migrate
    j = lb.pick_index()
    assert j != i and lb.pick_index() == j
    affinity_key.reset(tok)
    lb.set_active([j], False)
    assert lb.pick_index() == i


def test_stop_tokens_stop_strings_and_finish_reasons(served):
    c, ref, aeng = served
    prompt = list(range(10, 50))
    want = greedy_generate(ref, prompt, 12)
    stop_tok = want[5]
    k = want.index(stop_tok)
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 12, "temperature": 0, "ignore_eos": True,
                                        "stop_token_ids": [stop_tok]}).json()["choices"][0]
    assert r["token_ids"] == want[:k] and r["finish_reason"] == "stop"
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 12, "temperature": 0,
                                        "ignore_eos": True}).json()["choices"][0]
    assert r["finish_reason"] == "length"
    text = ByteTokenizer().decode(want)
    stop = text[3:5] if len(text) >= 5 else None
    if stop:
        r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 12, "temperature": 0,
                                            "ignore_eos": True, "stop": [stop]}).json()["choices"][0]
        assert r["finish_reason"] == "stop" and r["text"] == text[:text.find(stop)]


def test_engine_abort_releases_the_request():
    eng, _ = _engine()
    free0 = eng.pool.alloc.available() + len(eng.pool.prefix.lru)
    rid = eng.add_request(list(range(5, 60)), __import__("phung5_b200.engine.oracle", fromlist=["x"]).SamplingParams(
        max_new_tokens=50))
    eng.step()
    eng.step()
    assert eng.reqs[rid].pages
    assert eng.abort(rid) and eng.reqs[rid].finish_reason == "abort" and not eng.abort(rid)
    assert not eng.has_work()
    assert eng.pool.alloc.available() + len(eng.pool.prefix.lru) == free0
    queued = eng.add_request(list(range(5, 20)), None)
    assert eng.abort(queued) and not eng.waiting


def test_client_going_away_aborts_its_request(served):
    """A caller that stops reading the stream (the HTTP handler's generator is closed when its client goes
    away) aborts the engine request."""
    import asyncio
    import time as _t

    from phung5_b200.engine.oracle import SamplingParams
    _, _, aeng = served
    n0 = len(aeng.engine.reqs)

    async def go():
        gen = aeng.generate(list(range(20, 60)), SamplingParams(max_new_tokens=400))
        await gen.__anext__()
        await gen.aclose()
    asyncio.run(go())
    t0 = _t.time()
    while _t.time() - t0 < 10:
        reqs = list(aeng.engine.reqs.values())[n0:]
        if reqs and reqs[-1].finished:
            break
        _t.sleep(0.02)
    r = list(aeng.engine.reqs.values())[n0:][-1]
    assert r.finished and r.finish_reason == "abort" and len(r.out) < 400
