"""Constrained decoding: JSON objects and regular expressions through the engine and the API."""
import json
import re

import pytest
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import init_random_weights
from gollek_b200.native import host_ext
from gollek_b200.utils.tokenizer import ByteTokenizer, _gpt2_byte_decoder, _piece_bytes


def _engine():
    cfg = preset("tiny-llama")
    w = init_random_weights(cfg, seed=0)
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256,
                      use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


@pytest.mark.parametrize("pattern", [r'\{"ok": (true|false), "n": [0-9]{1,3}\}', r"(cat|dog)s?-\d{2}",
                                     r"[A-Z][a-z]{2,5}( [A-Z][a-z]{2,5})?"])
@pytest.mark.parametrize("temperature", [0.0, 1.0])
def test_regex_outputs_match(pattern, temperature):
    eng = _engine()
    outs = eng.generate([[5, 6, 7]] * 3, SamplingParams(temperature=temperature, max_tokens=60, guided_regex=pattern,
                                                        seed=3))
    for o in outs:
        text = eng.tokenizer.decode(o.output_token_ids)
        assert o.finish_reason == "stop", (o.finish_reason, text)
        assert re.fullmatch(pattern, text), (pattern, text)


def test_json_mode_every_prefix_valid():
    eng = _engine()
    outs = eng.generate([[9, 10]] * 2, SamplingParams(temperature=1.0, max_tokens=120, guided_json=True, seed=1))
    comp = host_ext().GrammarCompiler(eng.tokenizer.token_bytes(), eng.eos_token_id)
    for o in outs:
        m = comp.json(True)
        for t in o.output_token_ids:
            assert m.advance(t), o.output_token_ids
        text = eng.tokenizer.decode(o.output_token_ids)
        if o.finish_reason == "stop":
            assert isinstance(json.loads(text), dict)


def test_grammar_masks_and_byte_level_vocab():
    dec = _gpt2_byte_decoder()
    assert len(dec) == 256 and _piece_bytes("Ġhello", True, dec) == b" hello"
    assert _piece_bytes("▁the", False, dec) == b" the" and _piece_bytes("<0x0A>", False, dec) == b"\n"
    toks = [b"", b"", b"<eos>"] + [b'{"a"', b":", b" 1", b"}", b"x", b"[", b'"', b"1e5", b"-"]
    comp = host_ext().GrammarCompiler(toks, 2)
    m = comp.json(True)
    allowed = {toks[i] for i, a in enumerate(m.mask().tolist()) if a}
    assert allowed == {b'{"a"'}  # top-level object only
    for t in (b'{"a"', b":", b" 1", b"}"):
        assert m.advance(toks.index(t))
    assert m.accepting() and m.mask()[2]  # EOS allowed once complete
    with pytest.raises(ValueError):
        _engine().add_request("bad", [1, 2], SamplingParams(guided_regex="(unclosed"))


def test_api_response_format_json():
    from fastapi.testclient import TestClient

    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    ae = AsyncEngine(_engine()).start()
    try:
        with TestClient(create_app(ae)) as c:
            r = c.post("/v1/completions", json={"prompt": "x", "max_tokens": 40, "temperature": 0,
                                                "guided_regex": "[0-9]{3}-[0-9]{4}"}).json()
            assert re.fullmatch("[0-9]{3}-[0-9]{4}", r["choices"][0]["text"])
            r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                     "max_tokens": 30, "response_format": {"type": "json_object"}})
            assert r.status_code == 200
            txt = r.json()["choices"][0]["message"]["content"]
            assert txt.lstrip().startswith("{")
    finally:
        ae.shutdown(drain=False)


def test_mask_cache_separates_patterns():
    """Masks are cached per matcher state; NFA states of two patterns must not share entries."""
    toks = [b"", b"", b"<eos>", b"a", b"b", b"c"]
    comp = host_ext().GrammarCompiler(toks, 2)
    ma, mb = comp.regex("a+"), comp.regex("b+")
    assert ma.mask().tolist() == [False, False, False, True, False, False]
    assert mb.mask().tolist() == [False, False, False, False, True, False]
    assert comp.regex("a+").mask().tolist() == ma.mask().tolist()
