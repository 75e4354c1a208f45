"""Typical and mirostat-v2 sampling, logprobs, through the engine and the OpenAI API."""
import math

import torch

from gollek_b200.config import EngineConfig
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sampling_modes import sample_row
from gollek_b200.engine.sequence import SamplingParams, Sequence


def test_typical_keeps_the_typical_set():
    # p0 ~ 0.3 next to 1000 tail tokens: the entropy (~5.4 nats) is close to the tail's surprise
    # (~7.3) and far from the mode's (~1.2), so typical sampling at mass 0.5 excludes the mode
    logits = torch.tensor([6.06] + [0.0] * 1000)
    seq = Sequence("s", [1], SamplingParams(temperature=1.0, typical_p=0.5, seed=1))
    picks = set()
    for i in range(40):
        seq.output_token_ids = [0] * i
        picks.add(sample_row(logits.clone(), logits, seq, 0))
    assert 0 not in picks and len(picks) > 1


def test_mirostat_tracks_target_surprise():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(2000, generator=g) * 3
    seq = Sequence("s", [1], SamplingParams(temperature=1.0, mirostat=2, mirostat_tau=3.0, mirostat_eta=0.2, seed=3))
    probs = torch.softmax(logits, -1)
    surprises = []
    for i in range(300):
        seq.output_token_ids = [0] * i
        t = sample_row(logits.clone(), logits, seq, 0)
        surprises.append(-math.log2(float(probs[t])))
    assert seq.mirostat_mu is not None
    assert abs(sum(surprises[100:]) / 200 - 3.0) < 1.5  # hovers around tau


def test_logprobs_through_engine_and_api(tiny_cfg, tiny_weights):
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=32)
    out = eng.generate([[5, 6, 7, 8]], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True, logprobs=3))[0]
    assert out.logprobs is not None and len(out.logprobs) == 4
    for tok, e in zip(out.output_token_ids, out.logprobs):
        assert e["token"] == tok and e["logprob"] <= 0 and len(e["top"]) == 3
        assert max(e["top"].values()) == e["logprob"]  # greedy: the chosen token is the most likely
    from fastapi.testclient import TestClient

    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    ae = AsyncEngine(eng).start()
    try:
        with TestClient(create_app(ae)) as c:
            r = c.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 3, "temperature": 0,
                                                "logprobs": 2, "ignore_eos": True}).json()
            lp = r["choices"][0]["logprobs"]
            assert len(lp["token_logprobs"]) == 3 and all(len(t) == 2 for t in lp["top_logprobs"])
            r = c.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 3, "temperature": 0.8,
                                                "typical_p": 0.5, "ignore_eos": True, "seed": 2})
            assert r.status_code == 200
    finally:
        ae.shutdown(drain=False)
