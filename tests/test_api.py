"""HTTP API contract tests (FastAPI TestClient over the CPU engine)."""
import json

import pytest
from fastapi.testclient import TestClient

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.server.app import create_app
from gollek_b200.server.async_engine import AsyncEngine
from gollek_b200.utils.tokenizer import ByteTokenizer


@pytest.fixture(scope="module")
def client(tiny_weights):
    cfg = preset("tiny-llama")
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=8, max_num_batched_tokens=256, max_model_len=512,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=tiny_weights.__getitem__, tokenizer=ByteTokenizer(cfg.vocab_size),
                    num_blocks=256)
    ae = AsyncEngine(eng).start()
    app = create_app(ae, model_name="tiny")
    with TestClient(app) as c:
        yield c
    ae.shutdown()


def test_health_models_metrics(client):
    assert client.get("/health").json()["status"] == "UP"
    assert client.get("/q/health/ready").status_code == 200
    m = client.get("/v1/models").json()
    assert m["data"][0]["id"] == "tiny"
    assert client.get("/v1/models/nope").status_code == 404
    assert "gollek_steps" in client.get("/metrics").text


def test_completions(client):
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "hello", "max_tokens": 5,
                                             "temperature": 0, "ignore_eos": True})
    assert r.status_code == 200, r.text
    j = r.json()
    assert j["object"] == "text_completion"
    assert j["usage"]["completion_tokens"] == 5
    assert j["usage"]["prompt_tokens"] == len("hello")
    # token-id prompt, batch of two
    r = client.post("/v1/completions", json={"prompt": [[5, 6, 7], [8, 9]], "max_tokens": 3, "temperature": 0,
                                             "ignore_eos": True})
    assert len(r.json()["choices"]) == 2


def test_chat_and_stream(client):
    body = {"model": "tiny", "messages": [{"role": "user", "content": "hi"}], "max_tokens": 4, "temperature": 0}
    j = client.post("/v1/chat/completions", json=body).json()
    assert j["object"] == "chat.completion" and j["choices"][0]["message"]["role"] == "assistant"
    with client.stream("POST", "/v1/chat/completions", json={**body, "stream": True}) as r:
        lines = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[6:]) for l in lines[:-1]]
    assert chunks[0]["object"] == "chat.completion.chunk"
    assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
    assert chunks[-1]["usage"]["completion_tokens"] >= 1


def test_gollek_routes(client):
    req = {"model": "tiny", "messages": [{"role": "user", "content": "abc"}],
           "parameters": {"max_tokens": 3, "temperature": 0.0, "ignore_eos": True}}
    for path in ("/v1/infer/completions", "/v1/inference/completions", "/api/v1/inference"):
        j = client.post(path, json=req, headers={"X-Request-ID": "rid-1" + path}).json()
        assert set(j) >= {"requestId", "content", "model", "tokensUsed", "durationMs", "timestamp"}
    a = client.post("/v1/infer/async", json=req).json()
    import time
    for _ in range(200):
        s = client.get(f"/v1/infer/async/{a['jobId']}").json()
        if s["status"] in ("COMPLETED", "FAILED"):
            break
        time.sleep(0.02)
    assert s["status"] == "COMPLETED", s
    b = client.post("/v1/infer/batch", json=[req, req]).json()
    assert len(b) == 2
    with client.stream("POST", "/v1/infer/stream", json=req) as r:
        frames = [json.loads(l[6:]) for l in r.iter_lines() if l.startswith("data: ")]
    assert frames[-1]["isFinal"] and all("content" in f for f in frames)
    assert client.delete("/v1/infer/some-id").json()["status"] == "CANCELLED"


def test_embeddings(client):
    j = client.post("/v1/embeddings", json={"input": ["abc", "abd"]}).json()
    assert len(j["data"]) == 2 and len(j["data"][0]["embedding"]) == 256
    j = client.post("/v1/infer/embeddings", json={"messages": [{"content": "x"}]}).json()
    assert len(j["embeddings"]) == 1


def test_validation_errors(client):
    assert client.post("/v1/completions", json={"prompt": "x", "temperature": -1}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": "x", "n": 2}).status_code == 400


def test_api_keys(tiny_weights):
    cfg = preset("tiny-llama")
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=tiny_weights.__getitem__, tokenizer=ByteTokenizer(), num_blocks=32)
    ae = AsyncEngine(eng).start()
    app = create_app(ae, api_keys=["secret"])
    with TestClient(app) as c:
        assert c.get("/v1/models").status_code == 401
        assert c.get("/v1/models", headers={"Authorization": "Bearer secret"}).status_code == 200
        assert c.get("/health").status_code == 200
    ae.shutdown()


def test_error_payloads_admin_and_tenants(tiny_cfg, tiny_weights, monkeypatch):
    """Errors carry catalogue codes; admin routes create/revoke keys bound to tenants; a tenant at
    its running-request quota waits while another tenant's request is admitted."""
    from fastapi.testclient import TestClient

    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    monkeypatch.setenv("GOLLEK_ADMIN_KEY", "admin")
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False, tenant_quotas={"t1": {"max_running": 1}})
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=32)
    ae = AsyncEngine(eng).start()
    try:
        app = create_app(ae, api_keys={"k1": "t1", "k2": "t2"})
        with TestClient(app) as c:
            r = c.get("/v1/models")
            assert r.status_code == 401 and r.json()["error"]["code"] == "AUTH_101"
            r = c.get("/v1/models/nope", headers={"x-api-key": "k1"})
            assert r.status_code == 404 and r.json()["error"]["code"] == "MODEL_001"
            r = c.post("/v1/completions", json={"prompt": [1, 2, 3], "temperature": -1}, headers={"x-api-key": "k1"})
            assert r.status_code == 400 and r.json()["error"]["type"] == "VALIDATION"
            assert c.get("/v1/admin/api-keys", headers={"x-api-key": "k1"}).status_code == 403
            nk = c.post("/v1/admin/api-keys", json={"tenant": "t3"}, headers={"x-api-key": "admin"}).json()["key"]
            assert c.get("/v1/models", headers={"x-api-key": nk}).status_code == 200
            assert c.delete(f"/v1/admin/api-keys/{nk}", headers={"x-api-key": "admin"}).json()["revoked"]
            assert c.get("/v1/models", headers={"x-api-key": nk}).status_code == 401
            codes = c.get("/v1/admin/errors", headers={"x-api-key": "admin"}).json()["codes"]
            assert any(x["code"] == "QUOTA_101" for x in codes)
            assert c.get("/v1/admin/tenants", headers={"x-api-key": "admin"}).json()["quotas"] == {"t1": {"max_running": 1}}
    finally:
        ae.shutdown(drain=False)


def test_tenant_quota_scheduling(tiny_cfg, tiny_weights):
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=8, max_num_batched_tokens=256, max_model_len=128,
                      use_cuda_graphs=False, tenant_quotas={"a": {"max_running": 1}})
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=64)
    sp = SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True)
    for i in range(3):
        eng.add_request(f"a{i}", [1 + i, 2, 3], SamplingParams(**vars(sp)), tenant="a")
    eng.add_request("b0", [4, 5, 6], SamplingParams(**vars(sp)), tenant="b")
    eng.step()
    running = {s.request_id for s in eng.scheduler.running}
    assert "b0" in running and len([r for r in running if r.startswith("a")]) == 1
    while eng.has_unfinished():
        eng.step()
