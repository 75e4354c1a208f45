"""The remote SDK client (``GollekClient``) against the HTTP server, through a requests-shaped
adapter over FastAPI's TestClient (CPU engine)."""
import pytest
from fastapi.testclient import TestClient

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.sdk import GenerationRequest, GollekClient
from gollek_b200.server.app import create_app
from gollek_b200.server.async_engine import AsyncEngine
from gollek_b200.utils.tokenizer import ByteTokenizer


class _Resp:
    def __init__(self, r):
        self._r = r

    def __getattr__(self, k):
        return getattr(self._r, k)

    def iter_lines(self, decode_unicode=True):
        return self._r.iter_lines()


class _Session:
    """requests.Session surface over a TestClient (``stream`` is implied: bodies are buffered)."""

    def __init__(self, c):
        self.c, self.headers = c, c.headers

    def post(self, url, stream=False, **kw):
        return _Resp(self.c.post(url, **kw))

    def get(self, url, **kw):
        return _Resp(self.c.get(url, **kw))


@pytest.fixture(scope="module")
def sdk(tiny_weights):
    cfg = preset("tiny-llama")
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=128, max_model_len=256,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=tiny_weights.__getitem__, tokenizer=ByteTokenizer(cfg.vocab_size),
                    num_blocks=64)
    ae = AsyncEngine(eng).start()
    with TestClient(create_app(ae, model_name="tiny")) as c:
        yield GollekClient("http://testserver", session=_Session(c))
    ae.shutdown()


def test_remote_client_surface(sdk):
    assert sdk.health() and sdk.list_models() == ["tiny"]
    req = GenerationRequest("hello", model="tiny", max_tokens=4, temperature=0.0)
    r = sdk.generate(req)
    assert r.model == "tiny" and r.usage.completion_tokens == 4 and isinstance(r.text, str)
    assert "".join(sdk.stream(req)) == r.text  # greedy: the stream spells the same text
    c = sdk.complete("ab", model="tiny", max_tokens=3, temperature=0, ignore_eos=True)
    assert c["usage"]["completion_tokens"] == 3
    ch = sdk.chat([{"role": "user", "content": "hi"}], model="tiny", max_tokens=2, temperature=0, ignore_eos=True)
    assert ch["object"] == "chat.completion" and ch["usage"]["completion_tokens"] == 2
    assert len(sdk.embed(["a", "bc"])) == 2
    jid = sdk.submit(req)
    j = sdk.wait(jid, timeout=60)
    assert j["status"] == "COMPLETED" and j["result"]["content"] == r.text
    with pytest.raises(RuntimeError):
        sdk.job("no-such-job")
    # providers: registered through the SDK, listed back
    out = sdk.add_provider("up", "http://127.0.0.1:9/v1", models=["elsewhere"])
    assert out["registered"] == "up" and [p["id"] for p in sdk.providers()] == ["up"]
    assert "elsewhere" in sdk.list_models()
    # audio routes answer with an error when the server has no audio model; the client raises
    with pytest.raises(RuntimeError):
        sdk.speech("hello")
    with pytest.raises(RuntimeError):
        sdk.transcribe(b"RIFF0000WAVE", "a.wav")
