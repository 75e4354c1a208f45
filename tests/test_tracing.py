"""Tracing hooks: NVTX toggling, torch.profiler capture of engine steps, request spans, roofline."""
import json

import torch

from gollek_b200.config import EngineConfig
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.utils import roofline, tracing


def test_profile_and_spans(tiny_cfg, tiny_weights, tmp_path):
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=32)
    tracing.set_nvtx(True)  # no CUDA here: ranges are no-ops but the code paths run
    try:
        eng.add_request("a", list(range(1, 30)), SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))
        seq = eng.seqs["a"]
        path = tracing.profile_steps(eng, 3, str(tmp_path / "trace.json"))
        assert json.load(open(path))["traceEvents"]
        while eng.has_unfinished():
            eng.step()
    finally:
        tracing.set_nvtx(False)
    spans = tracing.request_spans([seq])
    sp = spans[0]
    assert sp["attributes"]["gollek.output_tokens"] == 4 and sp["attributes"]["gollek.status"] == "length"
    assert sp["start_time_unix_nano"] <= sp["end_time_unix_nano"]
    assert {e["name"] for e in sp["events"]} == {"admitted", "first_token"}
    tracing.write_spans(spans, str(tmp_path / "spans.jsonl"))


def test_roofline_arithmetic():
    pk = {"hbm_gbs": 1000.0, "bf16_tflops": 100.0, "source": "test"}
    r = roofline.analyse(flops=1e12, nbytes=1e9, ms=20.0, pk=pk)  # compute 10 ms, memory 1 ms
    assert r.bound == "compute" and abs(r.frac_roofline - 0.5) < 1e-9 and abs(r.tflops - 50.0) < 1e-6
    r = roofline.analyse(flops=1e9, nbytes=1e10, ms=10.0, nvlink_bytes=0, pk=pk)
    assert r.bound == "hbm" and abs(r.frac_hbm - 1.0) < 1e-9
