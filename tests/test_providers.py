"""Provider registry, scored routing with fallback, and forwarding to OpenAI-compatible upstreams
(fake upstream HTTP servers on 127.0.0.1; CPU engine)."""
import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest
from fastapi.testclient import TestClient

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.server.app import create_app
from gollek_b200.server.async_engine import AsyncEngine
from gollek_b200.server.resilience import CircuitOpen
from gollek_b200.server.providers import (Capabilities, NoProvider, Provider, ProviderError, ProviderRegistry,
                                          ProviderRouter)
from gollek_b200.utils.tokenizer import ByteTokenizer


class Fake(Provider):
    def __init__(self, pid, models, fail=False, caps=None):
        super().__init__(pid, caps)
        self._m, self.fail, self.seen = list(models), fail, []

    def models(self):
        return self._m

    def _call(self, route, body):
        self.seen.append((route, body))
        if self.fail:
            raise ConnectionError("down")
        return {"id": "x", "by": self.id}


def test_router_pins_scores_and_fails_over():
    reg = ProviderRegistry()
    a, b = Fake("a", ["m"]), Fake("b", ["m"], caps=Capabilities(streaming=False))
    c = Fake("c", ["other"], caps=Capabilities(formats=("gguf",)))
    for p in (a, b, c):
        reg.register(p)
    r = ProviderRouter(reg)
    assert r.route("m", preferred="B").provider == "b" and r.route("m", preferred="B").score == 10_000
    d = r.route("m", streaming=True)
    assert d.provider == "a" and d.fallbacks == ["b"]  # streaming capability wins
    a.latency_ewma = 2.5  # a slow provider loses the non-streaming tie
    assert r.route("m").provider == "b"
    with pytest.raises(NoProvider):
        r.route("nope")
    assert r.route("other", fmt="safetensors").provider == "c"  # GGUF-capable fallback
    # a failing winner fails over, and enough failures open its circuit
    a.latency_ewma, a.fail = 0.0, True
    assert r.execute("chat/completions", {"model": "m", "stream": True})["by"] == "b"
    assert a.failures == 1 and r.route("m", streaming=True).provider == "b"  # its failure ratio now costs it
    a.calls = a.failures = 0
    for _ in range(6):  # failures until the breaker opens; then it rejects without calling
        with pytest.raises((ConnectionError, CircuitOpen)):
            a.call("completions", {"model": "m"})
    assert a.breaker.state == "open" and 0 < a.failures < 6
    a.calls = a.failures = 0  # only the open circuit counts against it now
    assert r.route("m", streaming=True).provider == "b"  # the open circuit outweighs streaming
    b.fail = True
    with pytest.raises(ProviderError):
        r.execute("completions", {"model": "m"})


class _Upstream(BaseHTTPRequestHandler):
    name = "up"

    def log_message(self, *a):
        pass

    def _send(self, code, obj):
        data = json.dumps(obj).encode()
        self.send_response(code)
        self.send_header("Content-Type", "application/json")
        self.send_header("Content-Length", str(len(data)))
        self.end_headers()
        self.wfile.write(data)

    def do_GET(self):
        if self.path == "/v1/models":
            self._send(200, {"object": "list", "data": [{"id": "remote-model", "object": "model"}]})
        else:
            self._send(404, {})

    def do_POST(self):
        body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
        if body.get("model") != "remote-model":
            return self._send(400, {"error": {"message": "unknown model"}})
        if body.get("stream"):
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.end_headers()
            for w in ("hel", "lo"):
                self.wfile.write(b"data: " + json.dumps({"choices": [{"delta": {"content": w}}]}).encode() + b"\n\n")
            self.wfile.write(b"data: [DONE]\n\n")
            return
        self._send(200, {"object": "chat.completion", "model": "remote-model", "upstream": self.server.tag,
                         "auth": self.headers.get("Authorization", ""),
                         "choices": [{"message": {"role": "assistant", "content": "hello from " + self.server.tag}}]})


def _serve(tag):
    srv = ThreadingHTTPServer(("127.0.0.1", 0), _Upstream)
    srv.tag = tag
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


@pytest.fixture(scope="module")
def client(tiny_weights):
    cfg = preset("tiny-llama")
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=128, max_model_len=256,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=tiny_weights.__getitem__, tokenizer=ByteTokenizer(cfg.vocab_size),
                    num_blocks=64)
    ae = AsyncEngine(eng).start()
    with TestClient(create_app(ae, model_name="tiny")) as c:
        yield c
    ae.shutdown()


def test_forwarding_streaming_and_failover(client):
    up1, up2 = _serve("one"), _serve("two")
    try:
        for pid, srv, key in (("p1", up1, "k1"), ("p2", up2, "")):
            r = client.post("/v1/admin/providers", json={"id": pid, "api_key": key,
                                                         "base_url": f"http://127.0.0.1:{srv.server_port}/v1"})
            assert r.status_code == 200, r.text
        ids = {m["id"]: m["owned_by"] for m in client.get("/v1/models").json()["data"]}
        assert ids["tiny"] == "gollek-b200" and ids["remote-model"] in ("p1", "p2")
        msg = {"model": "remote-model", "messages": [{"role": "user", "content": "hi"}]}
        j = client.post("/v1/chat/completions", json=msg).json()
        first = j["provider"]
        assert j["choices"][0]["message"]["content"] == "hello from " + j["upstream"]
        assert j["auth"] == ("Bearer k1" if first == "p1" else "")
        s = client.post("/v1/chat/completions", json={**msg, "stream": True})
        assert s.status_code == 200 and "text/event-stream" in s.headers["content-type"]
        deltas = [json.loads(ln[6:])["choices"][0]["delta"]["content"] for ln in s.text.splitlines()
                  if ln.startswith("data: {")]
        assert "".join(deltas) == "hello" and "[DONE]" in s.text
        # the local model is still served locally
        loc = client.post("/v1/completions", json={"model": "tiny", "prompt": "ab", "max_tokens": 2,
                                                   "temperature": 0, "ignore_eos": True}).json()
        assert loc["usage"]["completion_tokens"] == 2 and "provider" not in loc
        # the routed upstream goes away while it still ranks first: the request fails over
        other = "p2" if first == "p1" else "p1"
        client.app.state.server.providers.get(other).latency_ewma = 1.0
        assert client.get("/v1/admin/providers/route", params={"model": "remote-model"}).json()["provider"] == first
        (up1 if first == "p1" else up2).shutdown()
        (up1 if first == "p1" else up2).server_close()
        j2 = client.post("/v1/chat/completions", json=msg).json()
        assert j2["provider"] != first and j2["upstream"] != j["upstream"]
        st = {p["id"]: p for p in client.get("/v1/admin/providers").json()["providers"]}
        assert st[first]["failures"] == 1 and st[other]["calls"] >= 1
        assert client.get("/v1/admin/providers/route", params={"model": "nope"}).status_code == 404
        assert client.delete("/v1/admin/providers/p1").status_code == 200
        assert client.delete("/v1/admin/providers/p1").status_code == 404
    finally:
        for srv in (up1, up2):
            try:
                srv.shutdown()
                srv.server_close()
            except Exception:
                pass
        client.delete("/v1/admin/providers/p2")


def test_server_provider_flag():
    from gollek_b200.server.__main__ import parse_providers
    reg = parse_providers(["a=http://h:1/v1,sk-1", "b=http://h:2/v1"])
    a, b = reg.get("a"), reg.get("b")
    assert (a.base, a.key, b.base, b.key) == ("http://h:1/v1", "sk-1", "http://h:2/v1", "")
    with pytest.raises(SystemExit):
        parse_providers(["nourl"])
