"""The GGUF converter service and its ``/v1/converter/gguf/*`` routes."""
import json
import os

import pytest
from fastapi import FastAPI
from fastapi.testclient import TestClient

from gollek_b200.config import preset
from gollek_b200.loaders.safetensors import save_file
from gollek_b200.models.reference import init_random_weights
from gollek_b200.server.converter import ConverterService, recommend, register_converter_routes


@pytest.fixture()
def conv(tmp_path):
    inp, out = tmp_path / "in", tmp_path / "out"
    ck = inp / "tiny"
    ck.mkdir(parents=True)
    out.mkdir()
    cfg = preset("tiny-llama", intermediate_size=768, num_hidden_layers=2)
    w = init_random_weights(cfg, seed=5)
    save_file({k: v.contiguous() for k, v in w.items()}, str(ck / "model.safetensors"))
    (ck / "config.json").write_text(json.dumps(cfg.to_hf()))
    app = FastAPI()
    svc = register_converter_routes(app, ConverterService(str(inp), str(out)))
    with TestClient(app) as c:
        yield c, svc, cfg, w


def test_catalogue_health_and_recommendation(conv):
    c, svc, _, _ = conv
    assert c.get("/v1/converter/gguf/health").json()["status"] == "UP"
    q = c.get("/v1/converter/gguf/quantizations").json()["quantizations"]
    names = {x["name"] for x in q}
    assert {"Q4_K_M", "Q6_K", "Q8_0", "F16", "Q2_K", "Q5_0"} <= names
    r = c.get("/v1/converter/gguf/recommend-quantization", params={"modelSizeGb": 16}).json()
    assert r["name"] == recommend(16) == "Q4_K_M" and "balanced" in r["reason"]
    assert c.get("/v1/converter/gguf/recommend-quantization",
                 params={"modelSizeGb": 16, "prioritizeQuality": True}).json()["name"] == "Q8_0"


def test_convert_verify_info_and_requantize(conv):
    import gguf
    c, svc, cfg, _ = conv
    assert c.get("/v1/converter/gguf/detect-format", params={"path": "tiny"}).json()["format"] == "safetensors"
    prev = c.post("/v1/converter/gguf/convert/preview", json={"inputPath": "tiny", "quantization": "Q4_K_M"}).json()
    assert prev["derivedOutputName"] == "tiny-q4_k_m.gguf" and prev["dryRun"]
    r = c.post("/v1/converter/gguf/convert", json={"inputPath": "tiny", "quantization": "Q4_K_M"})
    assert r.status_code == 200, r.text
    res = r.json()
    assert res["success"] and res["status"] == "COMPLETED" and res["compressionRatio"] > 3
    assert os.path.exists(res["outputPath"])
    types = {t.name: t.tensor_type.name for t in gguf.GGUFReader(res["outputPath"]).tensors}
    assert types["output.weight"] == "Q6_K" and types["blk.1.ffn_up.weight"] == "Q4_K"
    v = c.get("/v1/converter/gguf/verify", params={"path": "tiny-q4_k_m.gguf"}).json()
    assert v["valid"] and v["tensorsChecked"] == len(types)
    info = c.get("/v1/converter/gguf/model-info", params={"path": "tiny-q4_k_m.gguf"}).json()
    assert info["format"] == "gguf" and info["tensorTypes"]["Q6_K"] >= 1 and info["architecture"] == "llama"
    # the same output again: refused unless overwriteExisting
    assert c.post("/v1/converter/gguf/convert", json={"inputPath": "tiny", "quantization": "Q4_K_M"}).status_code == 409
    # GGUF -> GGUF requantization (input read from the output directory's file copied to the input side)
    os.replace(res["outputPath"], os.path.join(svc.input_base, "m.gguf"))
    r2 = c.post("/v1/converter/gguf/convert", json={"inputPath": "m.gguf", "quantization": "Q8_0"}).json()
    assert r2["success"], r2
    t2 = {t.tensor_type.name for t in gguf.GGUFReader(r2["outputPath"]).tensors if len(t.shape) == 2}
    assert t2 == {"Q8_0"}


def test_stream_progress_cancel_and_path_safety(conv):
    c, svc, _, _ = conv
    with c.stream("POST", "/v1/converter/gguf/convert/stream", json={"inputPath": "tiny", "quantization": "Q8_0"}) as r:
        lines = [ln for ln in r.iter_lines() if ln.startswith("data: ")]
    evs = [json.loads(ln[6:]) for ln in lines[:-1]]
    assert lines[-1] == "data: [DONE]"
    assert evs[0]["type"] == "started" and any(e["type"] == "progress" for e in evs)
    assert evs[-1]["type"] == "done" and evs[-1]["success"]
    cid = evs[-1]["conversionId"]
    assert c.get(f"/v1/converter/gguf/convert/{cid}").json()["status"] == "COMPLETED"
    assert c.post("/v1/converter/gguf/convert/999/cancel").status_code == 404
    # a cancelled job stops at its next tensor and leaves no partial file
    job = svc.start({"inputPath": "tiny", "quantization": "F32", "outputPath": "x.gguf"})
    job.cancel.set()
    svc.wait(job, 60)
    assert job.status in ("CANCELLED", "COMPLETED")
    assert not os.path.exists(job.output_path + ".part")
    # paths outside the base directories are refused
    assert c.post("/v1/converter/gguf/convert", json={"inputPath": "../../etc", "quantization": "F16"}).status_code == 400
    assert c.get("/v1/converter/gguf/detect-format", params={"path": "/etc/passwd"}).status_code == 400
    assert c.post("/v1/converter/gguf/convert", json={"inputPath": "tiny", "quantization": "Q9_Z"}).status_code == 400
