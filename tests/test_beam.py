"""Beam search: the engine-driven search against an exhaustive-vocabulary search on the fp32 oracle,
length penalty / early stopping / stop tokens, and the completions API."""
import math

import pytest
import torch

from gollek_b200.config import EngineConfig
from gollek_b200.engine.beam import BeamParams, BeamSearch
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.models.reference import ReferenceDecoder
from gollek_b200.utils.tokenizer import ByteTokenizer


def _engine(cfg, weights):
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=16, max_num_batched_tokens=256, max_model_len=256,
                      use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=weights.__getitem__, num_blocks=256,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


def _oracle_beam(ref, prompt, bp, eos):
    """The same selection rule over the full vocabulary with dense fp32 logits."""
    bs = BeamSearch(list(prompt), bp, eos)
    while not bs.done:
        tops = []
        for p in bs.prefixes():
            lp = torch.log_softmax(ref.forward(torch.tensor(p))[-1].double(), -1)
            v, i = lp.topk(bs.expansion_k)
            tops.append({int(a): float(b) for a, b in zip(i, v)})
        bs.update(tops)
    return bs.results()


@pytest.mark.parametrize("width,alpha", [(1, 1.0), (3, 1.0), (4, 0.0), (4, 2.0)])
def test_beam_matches_oracle(tiny_cfg, tiny_weights, width, alpha):
    eng = _engine(tiny_cfg, tiny_weights)
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    prompt = [5, 9, 13, 21, 40, 7, 3, 100, 77]
    bp = BeamParams(beam_width=width, max_tokens=12, length_penalty=alpha, num_return=width)
    got = eng.beam_search(prompt, bp)
    want = _oracle_beam(ref, prompt, bp, tiny_cfg.eos_token_id)
    assert [h.tokens for h in got] == [h.tokens for h in want]
    for g, w in zip(got, want):
        assert math.isclose(g.logprob, w.logprob, rel_tol=1e-3, abs_tol=1e-3)
    # width 1 is greedy decoding
    if width == 1:
        greedy, _ = ref.greedy(prompt, 12)
        assert got[0].tokens == list(greedy)[:12]


def test_beam_state_machine_rules():
    bp = BeamParams(beam_width=2, max_tokens=5, num_return=2, stop_token_ids=(9,))
    bs = BeamSearch([1], bp, eos_token_id=0)
    # step 1: EOS ranked first ends a hypothesis; the next two non-stop tokens become the beams
    bs.update([{0: -0.1, 4: -0.5, 5: -0.7, 6: -3.0}])
    assert [h.tokens for h in bs.finished] == [[]] and [h.tokens for h in bs.live] == [[4], [5]]
    # a stop token ranked below the K best candidates is ignored
    bs.update([{7: -0.1, 8: -0.2, 9: -5.0}, {7: -0.1, 9: -9.0}])
    assert len(bs.finished) == 1 and [h.tokens for h in bs.live] == [[4, 7], [4, 8]]
    # early stopping once K hypotheses finished
    bs2 = BeamSearch([1], BeamParams(beam_width=1, max_tokens=9, early_stopping=True), eos_token_id=0)
    bs2.update([{0: -0.1, 3: -0.2}])
    assert bs2.done and bs2.results()[0].finish_reason == "stop"
    with pytest.raises(ValueError):
        BeamParams(beam_width=2, num_return=3)


def test_beam_api(tiny_cfg, tiny_weights):
    from fastapi.testclient import TestClient

    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    eng = _engine(tiny_cfg, tiny_weights)
    want = eng.beam_search([5, 6, 7, 8], BeamParams(beam_width=3, max_tokens=6, num_return=2, ignore_eos=True))
    ae = AsyncEngine(_engine(tiny_cfg, tiny_weights)).start()
    try:
        with TestClient(create_app(ae)) as c:
            j = c.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "use_beam_search": True, "best_of": 3, "n": 2,
                                                "max_tokens": 6, "ignore_eos": True}).json()
            assert len(j["choices"]) == 2
            tok = ByteTokenizer(tiny_cfg.vocab_size, tiny_cfg.eos_token_id)
            assert [ch["text"] for ch in j["choices"]] == [tok.decode(h.tokens) for h in want]
            assert j["choices"][0]["score"] >= j["choices"][1]["score"]
            assert c.post("/v1/completions", json={"prompt": "x", "n": 2}).status_code == 400
    finally:
        ae.shutdown(drain=False)
