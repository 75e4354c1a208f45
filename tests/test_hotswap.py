"""Zero-downtime model hot-swap: the new model serves new requests after promotion, a request
in flight on the old model finishes there, lifecycle phases, refusals."""
import json
import threading
import time

import pytest
import torch
from fastapi.testclient import TestClient

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.models.reference import init_random_weights
from gollek_b200.server.app import create_app
from gollek_b200.server.async_engine import AsyncEngine
from gollek_b200.utils.tokenizer import ByteTokenizer


def _engine(seed):
    cfg = preset("tiny-llama")
    w = init_random_weights(cfg, seed=seed)
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=512,
                      use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


def _tokens(c, prompt=(5, 6, 7)):
    """Greedy log-probabilities of a short completion (they identify the serving weights)."""
    r = c.post("/v1/completions", json={"prompt": list(prompt), "max_tokens": 6, "temperature": 0,
                                        "ignore_eos": True, "logprobs": 1})
    assert r.status_code == 200, r.text
    return [round(v, 4) for v in r.json()["choices"][0]["logprobs"]["token_logprobs"]]


def test_hot_swap_promotes_and_drains():
    built = []

    def build(model):
        assert model == "tiny-v2"
        eng = _engine(seed=11)
        built.append(eng)
        return eng

    ae = AsyncEngine(_engine(seed=0)).start()
    app = create_app(ae, model_name="tiny-v1", engine_builder=build, drain_timeout_s=20)
    with TestClient(app) as c:
        before = _tokens(c)
        # a long request in flight on the old engine while the swap runs
        box = {}

        def long_request():
            r = c.post("/v1/completions", json={"prompt": [9, 9, 9], "max_tokens": 200, "temperature": 0,
                                                "ignore_eos": True})
            box["r"] = r

        th = threading.Thread(target=long_request)
        th.start()
        time.sleep(0.2)
        r = c.post("/v1/admin/models/swap", json={"model": "tiny-v2", "name": "tiny-v2"})
        assert r.status_code == 202, r.text
        sid = r.json()["swapId"]
        assert c.post("/v1/admin/models/swap", json={"model": "tiny-v2"}).status_code in (409, 202)
        for _ in range(600):
            st = c.get(f"/v1/admin/models/swap/{sid}").json()
            if st["done"]:
                break
            time.sleep(0.05)
        th.join(timeout=60)
        assert st["phase"] == "COMPLETE", st
        assert [e["phase"] for e in st["events"]] == ["LOADING", "WARMING_UP", "PROMOTED", "DRAINING", "UNLOADED",
                                                    "COMPLETE"]
        assert box["r"].status_code == 200 and box["r"].json()["usage"]["completion_tokens"] == 200
        after = _tokens(c)
        assert after != before                      # the new weights answer now
        assert c.get("/v1/models").json()["data"][0]["id"] == "tiny-v2"
        assert len(built) == 1 and app.state.server.engine is built[0]
        assert c.get("/v1/admin/models/swap").json()["active"] is None
    app.state.server.ae.shutdown(drain=False)


def test_hot_swap_failure_keeps_old_model():
    def build(model):
        raise FileNotFoundError(model)

    ae = AsyncEngine(_engine(seed=0)).start()
    app = create_app(ae, model_name="tiny-v1", engine_builder=build)
    with TestClient(app) as c:
        before = _tokens(c)
        sid = c.post("/v1/admin/models/swap", json={"model": "missing"}).json()["swapId"]
        for _ in range(200):
            st = c.get(f"/v1/admin/models/swap/{sid}").json()
            if st["done"]:
                break
            time.sleep(0.05)
        assert st["failed"] and st["phase"] == "FAILED"
        assert _tokens(c) == before
        assert c.post("/v1/admin/models/swap", json={}).status_code == 400
        assert c.get("/v1/admin/models/swap/nope").status_code == 404
    ae.shutdown(drain=False)
