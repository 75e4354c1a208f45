"""SpeechT5 text-to-speech and the HiFi-GAN vocoder against transformers' implementation (random
init, CPU): the same spectrogram frame for frame, the same stopping step, the same waveform."""
import pytest
import torch

transformers = pytest.importorskip("transformers")


def _tiny():
    from transformers import SpeechT5Config, SpeechT5ForTextToSpeech
    cfg = SpeechT5Config(hidden_size=64, encoder_layers=2, decoder_layers=2, encoder_attention_heads=4,
                         decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=128,
                         speech_decoder_prenet_units=32, speaker_embedding_dim=16, speech_decoder_postnet_units=32,
                         vocab_size=40, encoder_max_relative_position=8)
    torch.manual_seed(0)
    m = SpeechT5ForTextToSpeech(cfg).eval()
    # non-trivial batch-norm statistics in the postnet
    for layer in m.speech_decoder_postnet.layers:
        layer.batch_norm.running_mean.normal_(0, 0.1)
        layer.batch_norm.running_var.uniform_(0.5, 1.5)
    return cfg, m


def test_speecht5_spectrogram_matches_transformers(monkeypatch):
    from gollek_b200.models.speecht5 import SpeechT5TTS
    from transformers.models.speecht5 import modeling_speecht5 as M
    cfg, m = _tiny()
    # the reference keeps the prenet dropout on at inference; compare the deterministic model
    monkeypatch.setattr(M.SpeechT5SpeechDecoderPrenet, "_consistent_dropout", lambda self, x, p: x)
    ids = torch.randint(3, 40, (1, 23), generator=torch.Generator().manual_seed(1))
    spk = torch.randn(1, 16, generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = m.generate_speech(ids, spk, threshold=0.5, maxlenratio=3.0)
    sd = m.state_dict()
    d = cfg.to_dict()
    d["speech_decoder_prenet_dropout"] = 0.0
    ours = SpeechT5TTS(d, sd.__getitem__).generate(ids[0], spk[0], threshold=0.5, maxlenratio=3.0)
    assert ours.shape == ref.shape, (ours.shape, ref.shape)
    torch.testing.assert_close(ours, ref, rtol=1e-3, atol=1e-3)


def test_speecht5_prenet_dropout_is_seeded():
    from gollek_b200.models.speecht5 import SpeechT5TTS
    cfg, m = _tiny()
    tts = SpeechT5TTS(cfg.to_dict(), m.state_dict().__getitem__)
    ids, spk = torch.arange(3, 20), torch.ones(16)
    # at least 4 steps: frames after the first (all-zero) one make the dropout masks matter
    a = tts.generate(ids, spk, minlenratio=0.5, maxlenratio=2.0, seed=5)
    b = tts.generate(ids, spk, minlenratio=0.5, maxlenratio=2.0, seed=5)
    c = tts.generate(ids, spk, minlenratio=0.5, maxlenratio=2.0, seed=6)
    assert a.shape[0] >= 8
    assert torch.equal(a, b) and (a.shape != c.shape or not torch.equal(a, c))


def test_hifigan_matches_transformers():
    from transformers import SpeechT5HifiGan, SpeechT5HifiGanConfig
    from gollek_b200.models.speecht5 import HiFiGan
    cfg = SpeechT5HifiGanConfig(upsample_initial_channel=32, model_in_dim=80)
    torch.manual_seed(3)
    v = SpeechT5HifiGan(cfg).eval()
    v.mean.normal_(0, 0.5)
    v.scale.uniform_(0.5, 2.0)
    spec = torch.randn(37, 80, generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        ref = v(spec)
    ours = HiFiGan(cfg.to_dict(), v.state_dict().__getitem__)(spec)
    assert ours.shape == ref.shape == (37 * 256,)
    torch.testing.assert_close(ours, ref, rtol=1e-4, atol=1e-5)


def test_speech_endpoint(tmp_path):
    """POST /v1/audio/speech: WAV (or raw PCM) bytes of SpeechSynth's waveform for the text; 400 on
    empty input or an unknown voice, 501 without a model."""
    import io
    import wave

    import numpy as np
    from fastapi import FastAPI
    from fastapi.testclient import TestClient
    from transformers import SpeechT5HifiGan, SpeechT5HifiGanConfig
    from gollek_b200.models.speecht5 import SpeechSynth
    from gollek_b200.server.audio import register_audio_routes
    cfg, m = _tiny()
    m.save_pretrained(str(tmp_path / "tts"))
    torch.manual_seed(3)
    SpeechT5HifiGan(SpeechT5HifiGanConfig(upsample_initial_channel=32, model_in_dim=80)).save_pretrained(
        str(tmp_path / "voc"))
    (tmp_path / "tts" / "speakers").mkdir()
    np.save(tmp_path / "tts" / "speakers" / "alice.npy", np.random.default_rng(0).standard_normal(16).astype("float32"))
    tok = lambda text: [3 + (ord(ch) % 37) for ch in text] + [2]  # noqa: E731
    synth = SpeechSynth(str(tmp_path / "tts"), str(tmp_path / "voc"), tokenizer=tok)
    want = synth.synthesize("hello there", "alice", seed=1)
    app = FastAPI()
    register_audio_routes(app, None, synth)
    with TestClient(app) as c:
        r = c.post("/v1/audio/speech", json={"input": "hello there", "voice": "alice", "seed": 1})
        assert r.status_code == 200 and r.headers["content-type"] == "audio/wav"
        with wave.open(io.BytesIO(r.content)) as w:
            assert w.getframerate() == 16000 and w.getnframes() == want.shape[0]
            got = np.frombuffer(w.readframes(w.getnframes()), dtype="<i2") / 32767.0
        assert np.abs(got - np.clip(want, -1, 1)).max() < 1e-4
        pcm = c.post("/v1/audio/speech", json={"input": "hello there", "voice": "alice", "seed": 1,
                                               "response_format": "pcm"})
        assert pcm.content == r.content[44:]
        assert c.post("/v1/audio/speech", json={"input": ""}).status_code == 400
        assert c.post("/v1/audio/speech", json={"input": "hi", "voice": "bob"}).status_code == 400
    bare = FastAPI()
    register_audio_routes(bare, None, None)
    with TestClient(bare) as c:
        assert c.post("/v1/audio/speech", json={"input": "hi"}).status_code == 501


@pytest.mark.gpu
def test_speecht5_gpu_bf16_close_to_fp32():
    """The same utterance on the GPU in bf16 (linears on the tcgen05 GEMM) against the fp32 CPU run:
    close spectrogram frames until the shorter of the two stops."""
    from gollek_b200.models.speecht5 import SpeechT5TTS
    cfg, m = _tiny()
    d = cfg.to_dict()
    d["speech_decoder_prenet_dropout"] = 0.0
    ids, spk = torch.arange(3, 30), torch.randn(16, generator=torch.Generator().manual_seed(9))
    a = SpeechT5TTS(d, m.state_dict().__getitem__).generate(ids, spk, minlenratio=0.5, maxlenratio=1.0)
    b = SpeechT5TTS(d, m.state_dict().__getitem__, device="cuda", dtype=torch.bfloat16).generate(
        ids, spk, minlenratio=0.5, maxlenratio=1.0).cpu()
    n = min(a.shape[0], b.shape[0])
    assert n >= 8
    assert float((a[:n] - b[:n]).norm() / a[:n].norm()) < 0.05


def test_speak_cli_with_sentencepiece_tokenizer(tmp_path):
    """``gollek speak``: the default tokenizer (the checkpoint's character SentencePiece model plus the
    end-of-sequence id) and a WAV file of the synthesized waveform."""
    import argparse
    import wave

    import sentencepiece as spm
    from transformers import SpeechT5HifiGan, SpeechT5HifiGanConfig
    from gollek_b200 import cli
    cfg, m = _tiny()
    m.save_pretrained(str(tmp_path / "tts"))
    torch.manual_seed(3)
    SpeechT5HifiGan(SpeechT5HifiGanConfig(upsample_initial_channel=32, model_in_dim=80)).save_pretrained(
        str(tmp_path / "voc"))
    corpus = tmp_path / "corpus.txt"
    corpus.write_text("\n".join(["the quick brown fox jumps over the lazy dog"] * 20))
    spm.SentencePieceTrainer.train(input=str(corpus), model_prefix=str(tmp_path / "tts" / "spm_char"),
                                   model_type="char", vocab_size=31, bos_id=0, pad_id=1, eos_id=2, unk_id=3)
    out = tmp_path / "a.wav"
    cli.cmd_speak(argparse.Namespace(model=str(tmp_path / "tts"), vocoder=str(tmp_path / "voc"), text="a lazy fox",
                                     out=str(out), voice=None, seed=0, device="cpu"))
    with wave.open(str(out)) as w:
        assert w.getframerate() == 16000 and w.getnframes() > 0 and w.getnframes() % 256 == 0
