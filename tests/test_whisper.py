"""Whisper ASR against transformers: log-mel features vs WhisperFeatureExtractor (80 and 128 bins),
greedy decoding vs a greedy loop over WhisperForConditionalGeneration's logits, timestamp rules,
language detection, WAV decoding / resampling, window splitting, and /v1/audio/transcriptions."""
import io
import json

import numpy as np
import pytest
import torch

from gollek_b200.models import whisper as W

# a tiny vocabulary: text 0..89, then the special tokens, then 63 timestamp tokens (0 .. 1.24 s)
EOT, SOT, TRANSLATE, TRANSCRIBE, EN, DE, NO_TS = 90, 91, 92, 93, 94, 95, 96
VOCAB = 160


def _tiny_whisper(tmp_path, seed=0):
    from transformers import WhisperConfig, WhisperForConditionalGeneration
    cfg = WhisperConfig(vocab_size=VOCAB, num_mel_bins=80, encoder_layers=2, decoder_layers=2,
                        encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=128,
                        d_model=64, max_source_positions=1500, max_target_positions=64, pad_token_id=EOT,
                        bos_token_id=EOT, eos_token_id=EOT, decoder_start_token_id=SOT)
    torch.manual_seed(seed)
    m = WhisperForConditionalGeneration(cfg).eval()
    with torch.no_grad():
        for p in m.parameters():
            p.mul_(4.0)  # decisive logits
    d = tmp_path / "whisper"
    m.save_pretrained(str(d), safe_serialization=True)
    gen = {"decoder_start_token_id": SOT, "eos_token_id": EOT, "no_timestamps_token_id": NO_TS,
           "lang_to_id": {"<|en|>": EN, "<|de|>": DE}, "task_to_id": {"transcribe": TRANSCRIBE, "translate": TRANSLATE},
           "is_multilingual": True, "suppress_tokens": [3], "begin_suppress_tokens": [EOT]}
    (d / "generation_config.json").write_text(json.dumps(gen))
    return m, str(d)


def _speechy(seconds, sr=16000, seed=0):
    rng = np.random.default_rng(seed)
    t = np.arange(int(seconds * sr)) / sr
    return (0.3 * np.sin(2 * np.pi * 220 * t) * (1 + np.sin(2 * np.pi * 3 * t)) + 0.05 * rng.standard_normal(t.size)
            ).astype(np.float32)


@pytest.mark.parametrize("n_mels", [80, 128])
def test_log_mel_matches_feature_extractor(n_mels):
    from transformers import WhisperFeatureExtractor
    x = _speechy(7.3)
    ours = W.log_mel_spectrogram(x, n_mels).numpy()
    theirs = WhisperFeatureExtractor(feature_size=n_mels)(x, sampling_rate=16000, return_tensors="np").input_features[0]
    assert ours.shape == theirs.shape == (n_mels, 3000)
    assert np.abs(ours - theirs).max() < 2e-4


def _hf_greedy(m, mel, prompt, n, no_ts, suppress, begin_suppress):
    ids = torch.tensor([prompt])
    out = []
    with torch.no_grad():
        for j in range(n):
            lg = m(input_features=mel[None], decoder_input_ids=ids).logits[0, -1].clone()
            lg[no_ts:] = float("-inf")
            lg[suppress] = float("-inf")
            if j == 0:
                lg[begin_suppress] = float("-inf")
            t = int(lg.argmax())
            if t == EOT:
                break
            out.append(t)
            ids = torch.cat([ids, torch.tensor([[t]])], 1)
    return out


def test_greedy_decoding_matches_transformers(tmp_path):
    m, d = _tiny_whisper(tmp_path)
    model = W.WhisperModel.from_pretrained(d, device="cpu", dtype=torch.float32)
    audios = [_speechy(4.0, seed=1), _speechy(9.5, seed=2), _speechy(1.0, seed=3)]
    mel = torch.stack([W.log_mel_spectrogram(a) for a in audios])
    enc = model.encode(mel)
    with torch.no_grad():
        ref_enc = m.model.encoder(mel).last_hidden_state
    torch.testing.assert_close(enc, ref_enc, rtol=2e-4, atol=2e-4)
    prompt = model.prompt("en", "transcribe", timestamps=False)
    assert prompt == [SOT, EN, TRANSCRIBE, NO_TS]
    ours = model.decode(enc, [prompt] * 3, max_new_tokens=20)
    for a, o in zip(mel, ours):
        assert o == _hf_greedy(m, a, prompt, 20, NO_TS, [3], [EOT])
    tr = model.decode(enc[:1], [model.prompt("de", "translate", False)], max_new_tokens=12)[0]
    assert tr == _hf_greedy(m, mel[0], [SOT, DE, TRANSLATE, NO_TS], 12, NO_TS, [3], [EOT])


def test_timestamp_rules_and_language_detection(tmp_path):
    m, d = _tiny_whisper(tmp_path, seed=3)
    model = W.WhisperModel.from_pretrained(d, device="cpu", dtype=torch.float32)
    mel = torch.stack([W.log_mel_spectrogram(_speechy(3.0, seed=s)) for s in range(4)])
    enc = model.encode(mel)
    tsb = model.tokens.ts_begin
    for toks in model.decode(enc, [model.prompt("en", "transcribe", True)] * 4, max_new_tokens=30, timestamps=True):
        assert toks and toks[0] >= tsb and toks[0] <= tsb + 50      # opens with a timestamp <= 1 s
        ts = [t for t in toks if t >= tsb]
        assert ts == sorted(ts)                                       # never decreasing
        run = 0
        for t in toks:                                                # never three timestamps in a row
            run = run + 1 if t >= tsb else 0
            assert run <= 2
        assert NO_TS not in toks
    with torch.no_grad():
        ref = m(input_features=mel, decoder_input_ids=torch.full((4, 1), SOT)).logits[:, -1]
    want = ["en" if a > b else "de" for a, b in zip(ref[:, EN].tolist(), ref[:, DE].tolist())]
    assert model.detect_language(enc) == want
    segs = W.segments_from_tokens([tsb + 0, 5, 6, tsb + 10, tsb + 10, 7, tsb + 20, 8], tsb, 30.0)
    assert segs == [{"start": 30.0, "end": 30.2, "tokens": [5, 6]}, {"start": 30.2, "end": 30.4, "tokens": [7]},
                    {"start": 30.0, "end": None, "tokens": [8]}]


def _wav(x, sr, ch=1, fmt="pcm16"):
    """A RIFF/WAVE file written by hand (16-bit PCM or 32-bit float)."""
    import struct
    data = np.repeat(x[:, None], ch, 1)
    if fmt == "pcm16":
        body, tag, bits = (np.clip(data, -1, 1) * 32767).astype("<i2").tobytes(), 1, 16
    else:
        body, tag, bits = data.astype("<f4").tobytes(), 3, 32
    align = ch * bits // 8
    fmt_chunk = struct.pack("<HHIIHH", tag, ch, sr, sr * align, align, bits)
    return (b"RIFF" + struct.pack("<I", 4 + 8 + len(fmt_chunk) + 8 + len(body)) + b"WAVE" + b"fmt "
            + struct.pack("<I", len(fmt_chunk)) + fmt_chunk + b"data" + struct.pack("<I", len(body)) + body)


def test_wav_decoding_resampling_and_windows(tmp_path):
    x = _speechy(2.0, sr=8000)
    y = W.load_audio(_wav(x, 8000, ch=2))
    assert y.dtype == np.float32 and abs(len(y) - 32000) <= 1
    from scipy.signal import resample_poly
    ref = resample_poly((np.clip(x, -1, 1) * 32767).astype(np.int16).astype(np.float32) / 32768.0, 2, 1)
    assert np.abs(y - ref).max() < 1e-6
    z = W.load_audio(_wav(_speechy(1.0), 16000, fmt="f32"))
    assert np.array_equal(z, _speechy(1.0))
    p = str(tmp_path / "a.wav")
    W.write_wav(p, _speechy(0.5))
    assert len(W.load_audio(open(p, "rb").read())) == 8000
    with pytest.raises(ValueError):
        W.load_audio(b"ID3\x03" + b"\0" * 64)
    long = _speechy(70.0)
    long[27 * 16000:27 * 16000 + 3200] = 0.0  # 200 ms of silence at 27 s
    wins = W.split_windows(long)
    assert wins[0][0] == 0 and 27 * 16000 <= wins[0][1] <= 27 * 16000 + 3200
    assert all(e - s <= 30 * 16000 for s, e in wins) and wins[-1][1] == len(long)
    assert all(a[1] == b[0] for a, b in zip(wins, wins[1:]))


def test_transcription_endpoint(tmp_path):
    """/v1/audio/transcriptions and /translations (multipart upload, json / text / verbose_json)
    return what WhisperASR.transcribe returns for the same file."""
    from fastapi.testclient import TestClient
    from gollek_b200.config import EngineConfig, preset
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.models.reference import init_random_weights
    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    from gollek_b200.utils.tokenizer import ByteTokenizer

    _, d = _tiny_whisper(tmp_path)
    asr = W.WhisperASR(d, device="cpu", dtype=torch.float32, tokenizer=ByteTokenizer(VOCAB))
    wav = _wav(_speechy(3.0, seed=5), 16000)
    want = asr.transcribe([wav], language="en")[0]
    cfg = preset("tiny-llama")
    eng = LLMEngine(EngineConfig(device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=64,
                                 max_model_len=128, use_cuda_graphs=False),
                    model_cfg=cfg, weights=init_random_weights(cfg, seed=0).__getitem__,
                    tokenizer=ByteTokenizer(cfg.vocab_size), num_blocks=16)
    ae = AsyncEngine(eng).start()
    try:
        with TestClient(create_app(ae, model_name="tiny", asr=asr)) as c:
            files = {"file": ("a.wav", wav, "audio/wav")}
            j = c.post("/v1/audio/transcriptions", files=files, data={"language": "en"}).json()
            assert j == {"text": want["text"]}
            v = c.post("/v1/audio/transcriptions", files=files,
                       data={"language": "en", "response_format": "verbose_json"}).json()
            assert v["text"] == want["text"] and v["language"] == "en" and v["duration"] == 3.0
            assert v["segments"][0]["start"] == 0.0
            t = c.post("/v1/audio/transcriptions", files=files, data={"language": "en", "response_format": "text"})
            assert t.text == want["text"]
            tr = c.post("/v1/audio/translations", files=files).json()
            assert tr["text"] == asr.transcribe([wav], language="en", task="translate")[0]["text"]
            bad = c.post("/v1/audio/transcriptions", files={"file": ("a.mp3", b"ID3" + b"\0" * 40, "audio/mpeg")})
            assert bad.status_code == 400
    finally:
        ae.shutdown()


@pytest.mark.gpu
def test_whisper_gpu_graph_decode(tmp_path):
    """bf16 on the GPU: the encoder is close to transformers' fp32 one; the CUDA-graph decode gives
    the same tokens as eager decoding, also when a second call reuses the captured graph."""
    m, d = _tiny_whisper(tmp_path)
    g = W.WhisperModel.from_pretrained(d, device="cuda", dtype=torch.bfloat16, use_cuda_graphs=True)
    e = W.WhisperModel.from_pretrained(d, device="cuda", dtype=torch.bfloat16, use_cuda_graphs=False)
    p = g.prompt("en", "transcribe", False)
    for seeds in ((1, 2, 3), (4, 5, 6)):
        mel = torch.stack([W.log_mel_spectrogram(_speechy(3.0 + s, seed=s)) for s in seeds])
        enc = g.encode(mel.cuda())
        with torch.no_grad():
            ref = m.model.encoder(mel).last_hidden_state
        assert float((enc.float().cpu() - ref).norm() / ref.norm()) < 3e-2
        assert g.decode(enc, [p] * 3, 20) == e.decode(enc, [p] * 3, 20)
    assert 3 in g._graphs
    assert W.log_mel_spectrogram(_speechy(2.0), device="cuda").shape == (80, 3000)
