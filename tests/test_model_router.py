"""Model router: one server, several engines, each request served by the engine its ``model`` names
(the primary one for an unknown or missing name); routed models added and removed at run time."""
from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.models.reference import init_random_weights
from gollek_b200.utils.tokenizer import ByteTokenizer


def _engine(seed):
    cfg = preset("tiny-llama")
    w = init_random_weights(cfg, seed=seed)
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=256, max_model_len=512,
                      use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


def test_requests_go_to_the_named_engine():
    from fastapi.testclient import TestClient

    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    a, b = AsyncEngine(_engine(0)).start(), AsyncEngine(_engine(1)).start()
    app = create_app(a, model_name="base", routes={"other": b}, engine_builder=lambda m: _engine(2))
    body = {"prompt": "hello there", "max_tokens": 4, "temperature": 0.0, "ignore_eos": True, "logprobs": 1}
    try:
        with TestClient(app) as c:
            assert [m["id"] for m in c.get("/v1/models").json()["data"]] == ["base", "other"]
            ra = c.post("/v1/completions", json={**body, "model": "base"}).json()
            rb = c.post("/v1/completions", json={**body, "model": "other"}).json()
            ru = c.post("/v1/completions", json={**body, "model": "unknown"}).json()
            assert rb["model"] == "other" and ra["model"] == "base" and ru["model"] == "base"
            lp = lambda r: r["choices"][0]["logprobs"]["token_logprobs"]  # noqa: E731 (engines differ in weights)
            assert lp(ra) == lp(ru) and lp(ra) != lp(rb)
            # added at run time through the builder, removed again
            r = c.post("/v1/admin/models", json={"name": "third", "model": "tiny-llama"}).json()
            assert r["served"] == ["base", "other", "third"]
            rc = c.post("/v1/completions", json={**body, "model": "third"}).json()
            assert rc["model"] == "third"
            assert c.delete("/v1/admin/models/third").status_code == 204
            assert c.post("/v1/completions", json={**body, "model": "third"}).json()["model"] == "base"
    finally:
        for e in list(app.state.server.routes.values()) + [a]:
            e.shutdown()
