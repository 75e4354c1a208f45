"""Whisper speech recognition: log-mel features, encoder, batched decoder with a dense KV cache.

* ``log_mel_spectrogram``: 16 kHz mono -> [n_mels, 3000] for a 30 s window: Hann-windowed STFT
  (n_fft 400, hop 160, reflect padding, last frame dropped), power spectrum, a Slaney-scale
  triangular mel filter bank with Slaney area normalisation (built here from the formulas of
  Slaney's Auditory Toolbox), log10 floored at 1e-10, clamped to (max - 8), then (x + 4) / 4.
* ``WhisperModel.encode``: the two convolutions (k = 3; the second with stride 2) as im2col GEMMs
  on ``ops.linear`` with GELU, learned positions, pre-LayerNorm blocks, final LayerNorm: one batched
  pass over every 30 s window of every request in the call.
* ``WhisperModel.decode``: all windows decode together; per layer a self-attention KV cache
  [B, H, max_target_positions, hd] written at the step's position and read under a length mask
  (static shapes, so one decode step is captured once per batch size as a CUDA graph on the GPU),
  and cross-attention K/V computed once from the encoder output. The projections and the logits run
  on ``ops.linear``.
* Decoding rules: the prompt is <|startoftranscript|> <|lang|> <|task|> [<|notimestamps|>];
  ``suppress_tokens`` always and ``begin_suppress_tokens`` at the first step (from the checkpoint's
  generation config); without timestamps every timestamp token is suppressed. With timestamps the
  published Whisper rules apply: the first token is a timestamp no later than 1 s, timestamps do
  not decrease, they come in pairs (a single timestamp after text is followed by a timestamp or the
  end token, a pair by text), and when the timestamp tokens together are more probable than the best
  text token, a timestamp is taken. Language detection (language None on a multilingual checkpoint)
  takes the most probable language token after <|startoftranscript|>, per window.
* ``load_audio``: RIFF/WAVE files (PCM 8/16/24/32-bit, IEEE float 32/64, WAVE_FORMAT_EXTENSIBLE),
  channels averaged, resampled to 16 kHz with a polyphase filter; ``split_windows`` cuts long audio
  into windows of at most 30 s at the quietest 100 ms frame of each window's last 5 s.

Reference: runner/safetensor/gollek-safetensor-audio/…/audio/WhisperEngine.java (constants :52-65,
transcribe / chunking :108-160, decoder prompt :299-302), processing/AudioFeatureExtractor.java
(log-mel), processing/VoiceActivityDetector.java (silence-based segmentation), and the HTTP surface
runner/safetensor/gollek-safetensor-api/…/api/AudioResource.java (/v1/audio/transcriptions :54,
/v1/audio/translations :98).
"""
from __future__ import annotations

import json
import math
import os
import struct
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from .. import ops
from .clip import _act, _layer_norm

SAMPLE_RATE = 16000
N_FFT = 400
HOP = 160
CHUNK_S = 30
N_SAMPLES = SAMPLE_RATE * CHUNK_S       # 480000
N_FRAMES = N_SAMPLES // HOP             # 3000
SECONDS_PER_TS = 0.02                   # one timestamp token step


# --------------------------------------------------------------------------------------- features
def _hz_to_mel(f: np.ndarray) -> np.ndarray:
    """Slaney mel scale: linear (3 mel per 200 Hz) below 1 kHz, logarithmic above (27 mel per
    factor 6.4)."""
    f = np.asarray(f, dtype=np.float64)
    lin = 3.0 * f / 200.0
    log = 15.0 + 27.0 * np.log(np.maximum(f, 1e-12) / 1000.0) / np.log(6.4)
    return np.where(f < 1000.0, lin, log)


def _mel_to_hz(m: np.ndarray) -> np.ndarray:
    m = np.asarray(m, dtype=np.float64)
    lin = 200.0 * m / 3.0
    log = 1000.0 * np.exp(np.log(6.4) * (m - 15.0) / 27.0)
    return np.where(m < 15.0, lin, log)


def mel_filters(n_mels: int, sr: int = SAMPLE_RATE, n_fft: int = N_FFT, fmin: float = 0.0,
                fmax: Optional[float] = None) -> np.ndarray:
    """[n_fft // 2 + 1, n_mels] triangular filters on the Slaney mel scale, each scaled to unit
    area (2 / bandwidth in Hz)."""
    fmax = sr / 2 if fmax is None else fmax
    bins = np.linspace(0.0, sr / 2, n_fft // 2 + 1)
    edges = _mel_to_hz(np.linspace(_hz_to_mel(fmin), _hz_to_mel(fmax), n_mels + 2))
    lo, mid, hi = edges[:-2], edges[1:-1], edges[2:]
    rise = (bins[:, None] - lo[None, :]) / (mid - lo)[None, :]
    fall = (hi[None, :] - bins[:, None]) / (hi - mid)[None, :]
    w = np.clip(np.minimum(rise, fall), 0.0, None)
    return (w * (2.0 / (hi - lo))[None, :]).astype(np.float32)


_MEL_CACHE: Dict[Tuple[int, str], torch.Tensor] = {}


def log_mel_spectrogram(audio, n_mels: int = 80, device: str = "cpu") -> torch.Tensor:
    """One window of 16 kHz mono audio (padded with zeros / cut to 30 s) -> [n_mels, 3000] fp32."""
    x = torch.as_tensor(np.asarray(audio, dtype=np.float32), device=device).flatten()
    x = F.pad(x[:N_SAMPLES], (0, max(0, N_SAMPLES - x.numel())))
    key = (n_mels, str(x.device))
    if key not in _MEL_CACHE:
        _MEL_CACHE[key] = torch.from_numpy(mel_filters(n_mels)).to(x.device)
    win = torch.hann_window(N_FFT, periodic=True, device=x.device)
    spec = torch.stft(x, N_FFT, HOP, window=win, center=True, pad_mode="reflect", return_complex=True)
    power = spec[:, :-1].abs() ** 2                                  # [201, 3000]
    mel = _MEL_CACHE[key].t() @ power                                # [n_mels, 3000]
    logm = torch.log10(torch.clamp(mel, min=1e-10))
    logm = torch.maximum(logm, logm.max() - 8.0)
    return (logm + 4.0) / 4.0


# ------------------------------------------------------------------------------------------ audio
def load_audio(data: bytes, sr: int = SAMPLE_RATE) -> np.ndarray:
    """RIFF/WAVE bytes -> mono float32 at ``sr``."""
    if len(data) < 12 or data[:4] != b"RIFF" or data[8:12] != b"WAVE":
        raise ValueError("unsupported audio container (RIFF/WAVE expected)")
    pos, fmt, payload = 12, None, None
    while pos + 8 <= len(data):
        cid, size = data[pos:pos + 4], struct.unpack_from("<I", data, pos + 4)[0]
        body = data[pos + 8:pos + 8 + size]
        if cid == b"fmt ":
            tag, ch, rate, _, align, bits = struct.unpack_from("<HHIIHH", body, 0)
            if tag == 0xFFFE and len(body) >= 26:  # WAVE_FORMAT_EXTENSIBLE: the sub-format's tag
                tag = struct.unpack_from("<H", body, 24)[0]
            fmt = (tag, ch, rate, align, bits)
        elif cid == b"data":
            payload = body
        pos += 8 + size + (size & 1)
    if fmt is None or payload is None:
        raise ValueError("WAVE file without fmt/data chunks")
    tag, ch, rate, align, bits = fmt
    if ch < 1 or align < 1:
        raise ValueError("bad WAVE format chunk")
    n = len(payload) // align
    raw = np.frombuffer(payload[:n * align], dtype=np.uint8).reshape(n, ch, align // ch)
    if tag == 1 and bits == 8:
        x = (raw[..., 0].astype(np.float32) - 128.0) / 128.0
    elif tag == 1 and bits == 16:
        x = raw.copy().view("<i2")[..., 0].astype(np.float32) / 32768.0
    elif tag == 1 and bits == 24:
        v = raw[..., 0].astype(np.int32) | (raw[..., 1].astype(np.int32) << 8) | (raw[..., 2].astype(np.int32) << 16)
        x = (np.where(v >= 1 << 23, v - (1 << 24), v)).astype(np.float32) / float(1 << 23)
    elif tag == 1 and bits == 32:
        x = raw.copy().view("<i4")[..., 0].astype(np.float32) / float(1 << 31)
    elif tag == 3 and bits in (32, 64):
        x = raw.copy().view("<f4" if bits == 32 else "<f8")[..., 0].astype(np.float32)
    else:
        raise ValueError(f"unsupported WAVE sample format (tag {tag}, {bits} bits)")
    x = x.mean(axis=1)
    if rate != sr:
        from scipy.signal import resample_poly
        g = math.gcd(int(rate), sr)
        x = resample_poly(x, sr // g, int(rate) // g).astype(np.float32)
    return np.ascontiguousarray(x, dtype=np.float32)


def write_wav(path: str, audio: np.ndarray, sr: int = SAMPLE_RATE) -> None:
    """Mono 16-bit PCM WAVE (for tests and tools)."""
    import wave
    pcm = (np.clip(np.asarray(audio, dtype=np.float32), -1.0, 1.0) * 32767.0).astype("<i2")
    with wave.open(path, "wb") as w:
        w.setnchannels(1)
        w.setsampwidth(2)
        w.setframerate(sr)
        w.writeframes(pcm.tobytes())


def split_windows(audio: np.ndarray, max_s: float = CHUNK_S, search_s: float = 5.0) -> List[Tuple[int, int]]:
    """[(start, end)] sample ranges of at most ``max_s``; each cut falls on the quietest 100 ms frame
    of the last ``search_s`` seconds of its window."""
    n, wmax = len(audio), int(max_s * SAMPLE_RATE)
    frame = SAMPLE_RATE // 10
    out, s = [], 0
    while n - s > wmax:
        lo = s + wmax - int(search_s * SAMPLE_RATE)
        seg = audio[lo:s + wmax]
        k = len(seg) // frame
        energy = (seg[:k * frame].reshape(k, frame) ** 2).mean(axis=1)
        cut = lo + int(np.argmin(energy)) * frame + frame // 2
        out.append((s, cut))
        s = cut
    if n > s or not out:
        out.append((s, n))
    return out


# ------------------------------------------------------------------------------------------ model
@dataclass
class WhisperConfig:
    d_model: int = 384
    encoder_layers: int = 4
    decoder_layers: int = 4
    encoder_heads: int = 6
    decoder_heads: int = 6
    encoder_ffn: int = 1536
    decoder_ffn: int = 1536
    num_mel_bins: int = 80
    max_source_positions: int = 1500
    max_target_positions: int = 448
    vocab_size: int = 51865
    activation: str = "gelu"
    eps: float = 1e-5

    @staticmethod
    def from_hf(d: dict) -> "WhisperConfig":
        return WhisperConfig(
            d_model=int(d["d_model"]), encoder_layers=int(d["encoder_layers"]),
            decoder_layers=int(d["decoder_layers"]), encoder_heads=int(d["encoder_attention_heads"]),
            decoder_heads=int(d["decoder_attention_heads"]), encoder_ffn=int(d["encoder_ffn_dim"]),
            decoder_ffn=int(d["decoder_ffn_dim"]), num_mel_bins=int(d.get("num_mel_bins", 80)),
            max_source_positions=int(d.get("max_source_positions", 1500)),
            max_target_positions=int(d.get("max_target_positions", 448)), vocab_size=int(d["vocab_size"]),
            activation=str(d.get("activation_function", "gelu")))


@dataclass
class WhisperTokens:
    """Special token ids of a Whisper vocabulary (multilingual defaults; a checkpoint's generation
    config overrides them)."""
    sot: int = 50258
    eot: int = 50257
    transcribe: int = 50359
    translate: int = 50358
    no_timestamps: int = 50363
    lang_to_id: Dict[str, int] = field(default_factory=lambda: {"en": 50259})
    suppress: List[int] = field(default_factory=list)
    begin_suppress: List[int] = field(default_factory=list)
    multilingual: bool = True

    @property
    def ts_begin(self) -> int:
        return self.no_timestamps + 1

    @staticmethod
    def from_generation_config(g: dict) -> "WhisperTokens":
        t = WhisperTokens()
        t.sot = int(g.get("decoder_start_token_id", t.sot))
        eos = g.get("eos_token_id", t.eot)
        t.eot = int(eos[0] if isinstance(eos, list) else eos)
        tasks = g.get("task_to_id") or {}
        t.transcribe = int(tasks.get("transcribe", t.transcribe))
        t.translate = int(tasks.get("translate", t.translate))
        t.no_timestamps = int(g.get("no_timestamps_token_id", t.no_timestamps))
        if g.get("lang_to_id"):
            t.lang_to_id = {k.strip("<|>"): int(v) for k, v in g["lang_to_id"].items()}
        t.suppress = [int(i) for i in g.get("suppress_tokens") or []]
        t.begin_suppress = [int(i) for i in g.get("begin_suppress_tokens") or []]
        t.multilingual = bool(g.get("is_multilingual", len(t.lang_to_id) > 1))
        return t


class WhisperModel:
    def __init__(self, cfg: WhisperConfig, get: Callable[[str], torch.Tensor], device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16, tokens: Optional[WhisperTokens] = None,
                 use_cuda_graphs: bool = True):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.tokens = tokens or WhisperTokens()
        self.use_cuda_graphs = use_cuda_graphs and self.device.type == "cuda"

        def t(n):
            return get(n).to(self.device, dtype).contiguous()

        def opt(n):
            try:
                return t(n)
            except KeyError:
                return None

        e, dcd = "model.encoder.", "model.decoder."
        d = cfg.d_model
        # conv weights [out, in, 3] -> GEMM [out, 3 * in] in (tap, channel) order, K padded to 8
        self.c1_w = self._conv_w(t(e + "conv1.weight"))
        self.c1_b = t(e + "conv1.bias")
        self.c2_w = self._conv_w(t(e + "conv2.weight"))
        self.c2_b = t(e + "conv2.bias")
        self.enc_pos = t(e + "embed_positions.weight")
        self.enc = [self._layer(get, f"{e}layers.{i}.", t, opt, cross=False) for i in range(cfg.encoder_layers)]
        self.enc_ln = (t(e + "layer_norm.weight"), t(e + "layer_norm.bias"))
        self.embed = t(dcd + "embed_tokens.weight")
        self.dec_pos = t(dcd + "embed_positions.weight")
        self.dec = [self._layer(get, f"{dcd}layers.{i}.", t, opt, cross=True) for i in range(cfg.decoder_layers)]
        self.dec_ln = (t(dcd + "layer_norm.weight"), t(dcd + "layer_norm.bias"))
        self.head = opt("proj_out.weight")
        if self.head is None:
            self.head = self.embed
        self._graphs: Dict[int, tuple] = {}
        self.max_graphs = 4

    @staticmethod
    def _conv_w(w: torch.Tensor) -> torch.Tensor:
        o, i, k = w.shape
        g = w.permute(0, 2, 1).reshape(o, k * i)
        pad = (-g.shape[1]) % 8
        return F.pad(g, (0, pad)).contiguous() if pad else g.contiguous()

    @staticmethod
    def _layer(get, p: str, t, opt, cross: bool) -> dict:
        def attn(a):
            q_w, k_w, v_w = t(p + a + ".q_proj.weight"), t(p + a + ".k_proj.weight"), t(p + a + ".v_proj.weight")
            q_b, v_b = t(p + a + ".q_proj.bias"), t(p + a + ".v_proj.bias")
            return {"q_w": q_w, "q_b": q_b, "kv_w": torch.cat([k_w, v_w]).contiguous(),
                    "kv_b": torch.cat([torch.zeros_like(v_b), v_b]),  # k_proj has no bias
                    "qkv_w": torch.cat([q_w, k_w, v_w]).contiguous(),
                    "qkv_b": torch.cat([q_b, torch.zeros_like(v_b), v_b]),
                    "o_w": t(p + a + ".out_proj.weight"), "o_b": t(p + a + ".out_proj.bias")}
        L = {"sa": attn("self_attn"), "ln1": (t(p + "self_attn_layer_norm.weight"), t(p + "self_attn_layer_norm.bias")),
             "ln3": (t(p + "final_layer_norm.weight"), t(p + "final_layer_norm.bias")),
             "fc1_w": t(p + "fc1.weight"), "fc1_b": t(p + "fc1.bias"),
             "fc2_w": t(p + "fc2.weight"), "fc2_b": t(p + "fc2.bias")}
        if cross:
            L["ca"] = attn("encoder_attn")
            L["ln2"] = (t(p + "encoder_attn_layer_norm.weight"), t(p + "encoder_attn_layer_norm.bias"))
        return L

    @staticmethod
    def from_pretrained(path: str, device: str = "cuda", dtype: torch.dtype = torch.bfloat16,
                        use_cuda_graphs: bool = True) -> "WhisperModel":
        from ..loaders.safetensors import SafetensorsCheckpoint
        with open(os.path.join(path, "config.json")) as fh:
            cfg = WhisperConfig.from_hf(json.load(fh))
        tok = WhisperTokens()
        gpath = os.path.join(path, "generation_config.json")
        if os.path.exists(gpath):
            with open(gpath) as fh:
                tok = WhisperTokens.from_generation_config(json.load(fh))
        ck = SafetensorsCheckpoint(path)
        return WhisperModel(cfg, ck.get, device, dtype, tok, use_cuda_graphs)

    # ---------------------------------------------------------------------------------- encoder
    def _mlp(self, L: dict, x: torch.Tensor) -> torch.Tensor:
        m = _act(ops.linear(x, L["fc1_w"]) + L["fc1_b"], self.cfg.activation)
        return ops.linear(m.contiguous(), L["fc2_w"]) + L["fc2_b"]

    def _conv(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, stride: int) -> torch.Tensor:
        """x [B, T, C] (channels last) -> [B, T', out]: k = 3, padding 1, as one GEMM."""
        B, T, C = x.shape
        xp = F.pad(x, (0, 0, 1, 1))
        cols = xp.unfold(1, 3, stride).permute(0, 1, 3, 2).reshape(B, -1, 3 * C)  # (tap, channel)
        Tn = cols.shape[1]
        pad = w.shape[1] - 3 * C
        cols = F.pad(cols, (0, pad)) if pad else cols
        y = ops.linear(cols.reshape(B * Tn, -1).contiguous(), w) + b
        return _act(y, "gelu").view(B, Tn, -1)

    @torch.inference_mode()
    def encode(self, mel: torch.Tensor) -> torch.Tensor:
        """mel [B, n_mels, 3000] -> encoder states [B, 1500, d]."""
        cfg = self.cfg
        x = mel.to(self.device, self.dtype).transpose(1, 2).contiguous()
        x = self._conv(x, self.c1_w, self.c1_b, 1)
        x = self._conv(x, self.c2_w, self.c2_b, 2)
        B, S, d = x.shape
        h = (x + self.enc_pos[:S]).reshape(B * S, d)
        H = cfg.encoder_heads
        for L in self.enc:
            a = _layer_norm(h, *L["ln1"], cfg.eps)
            qkv = (ops.linear(a, L["sa"]["qkv_w"]) + L["sa"]["qkv_b"]).view(B, S, 3, H, d // H)
            q, k, v = (z.transpose(1, 2) for z in qkv.unbind(2))
            o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B * S, d)
            h = h + ops.linear(o.contiguous(), L["sa"]["o_w"]) + L["sa"]["o_b"]
            h = h + self._mlp(L, _layer_norm(h, *L["ln3"], cfg.eps))
        return _layer_norm(h, *self.enc_ln, cfg.eps).view(B, S, d)

    # ---------------------------------------------------------------------------------- decoder
    def _cross_kv(self, enc: torch.Tensor) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        B, S, d = enc.shape
        H = self.cfg.decoder_heads
        out = []
        for L in self.dec:
            kv = (ops.linear(enc.reshape(B * S, d), L["ca"]["kv_w"]) + L["ca"]["kv_b"]).view(B, S, 2, H, d // H)
            out.append((kv[:, :, 0].transpose(1, 2).contiguous(), kv[:, :, 1].transpose(1, 2).contiguous()))
        return out

    def _new_state(self, B: int, enc: torch.Tensor) -> dict:
        H, d, T = self.cfg.decoder_heads, self.cfg.d_model, self.cfg.max_target_positions
        return {"k": torch.zeros(len(self.dec), B, H, T, d // H, device=self.device, dtype=self.dtype),
                "v": torch.zeros(len(self.dec), B, H, T, d // H, device=self.device, dtype=self.dtype),
                "cross": self._cross_kv(enc)}

    def _step(self, st: dict, tokens: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """One decoder position for every row: tokens [B], pos [B] (int64, device) -> logits [B, V]
        fp32. Static shapes (the cache is read under a mask), so the step can be graph-captured."""
        cfg = self.cfg
        B, d, H = tokens.shape[0], cfg.d_model, cfg.decoder_heads
        hd, T = d // H, cfg.max_target_positions
        h = self.embed[tokens] + self.dec_pos[pos]
        visible = (torch.arange(T, device=self.device)[None, :] <= pos[:, None])           # [B, T]
        mask = torch.zeros(B, 1, 1, T, device=self.device, dtype=self.dtype).masked_fill(
            ~visible[:, None, None, :], float("-inf"))
        at = pos.view(B, 1, 1, 1).expand(B, H, 1, hd)
        for i, L in enumerate(self.dec):
            a = _layer_norm(h, *L["ln1"], cfg.eps)
            qkv = (ops.linear(a, L["sa"]["qkv_w"]) + L["sa"]["qkv_b"]).view(B, 3, H, hd)
            st["k"][i].scatter_(2, at, qkv[:, 1, :, None, :])  # each row's k, v at its position
            st["v"][i].scatter_(2, at, qkv[:, 2, :, None, :])
            o = F.scaled_dot_product_attention(qkv[:, 0, :, None, :], st["k"][i], st["v"][i], attn_mask=mask)
            h = h + ops.linear(o.reshape(B, d).contiguous(), L["sa"]["o_w"]) + L["sa"]["o_b"]
            a = _layer_norm(h, *L["ln2"], cfg.eps)
            q = (ops.linear(a, L["ca"]["q_w"]) + L["ca"]["q_b"]).view(B, H, 1, hd)
            ck, cv = st["cross"][i]
            o = F.scaled_dot_product_attention(q, ck, cv)
            h = h + ops.linear(o.reshape(B, d).contiguous(), L["ca"]["o_w"]) + L["ca"]["o_b"]
            h = h + self._mlp(L, _layer_norm(h, *L["ln3"], cfg.eps))
        h = _layer_norm(h, *self.dec_ln, cfg.eps)
        return ops.linear(h.contiguous(), self.head).float()

    def _step_fn(self, st: dict, B: int):
        """The decode step for a batch of B, replayed from a CUDA graph on the GPU."""
        if not self.use_cuda_graphs:
            return lambda tok, pos: self._step(st, tok, pos)
        tok = torch.zeros(B, dtype=torch.long, device=self.device)
        pos = torch.zeros(B, dtype=torch.long, device=self.device)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside the capture (lazy init, allocator)
                self._step(st, tok, pos)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        # thread-local capture: a serving engine may launch work from its own thread meanwhile
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            out = self._step(st, tok, pos)

        def run(t_in, p_in):
            tok.copy_(t_in)
            pos.copy_(p_in)
            g.replay()
            return out
        return run

    def _runner(self, B: int, enc: torch.Tensor):
        """The step function of batch size B over ``enc``. With CUDA graphs, the graph and its state
        (self-attention cache, cross K/V) are kept per batch size (at most ``max_graphs``) and the
        cross K/V of a new call are copied into place; cache positions above the step's position
        are masked, so the cache needs no clearing."""
        ent = self._graphs.get(B)
        if ent is None:
            st = self._new_state(B, enc)
            ent = (st, self._step_fn(st, B))
            if self.use_cuda_graphs:
                if len(self._graphs) >= self.max_graphs:
                    self._graphs.pop(next(iter(self._graphs)))
                self._graphs[B] = ent
        else:
            for (k, v), (ck, cv) in zip(ent[0]["cross"], self._cross_kv(enc)):
                k.copy_(ck)
                v.copy_(cv)
        return ent[1]

    # --------------------------------------------------------------------------------- decoding
    def _rules(self, logits: torch.Tensor, seqs: List[List[int]], n_prompt: int, timestamps: bool) -> torch.Tensor:
        """Token suppression and the timestamp rules, row by row, on fp32 logits [B, V]."""
        tk = self.tokens
        V = logits.shape[1]
        neg = float("-inf")
        if tk.suppress:
            logits[:, [i for i in tk.suppress if i < V]] = neg
        tsb = tk.ts_begin
        for r, s in enumerate(seqs):
            gen = s[n_prompt:]
            if not gen and tk.begin_suppress:
                logits[r, [i for i in tk.begin_suppress if i < V]] = neg
            if not timestamps:
                logits[r, tk.no_timestamps:] = neg
                continue
            logits[r, tk.no_timestamps] = neg
            last_ts = len(gen) >= 1 and gen[-1] >= tsb
            prev_ts = len(gen) < 2 or gen[-2] >= tsb
            if last_ts:
                if prev_ts:
                    logits[r, tsb:] = neg       # a closed pair: text (or the end) follows
                else:
                    logits[r, :tk.eot] = neg    # an open segment: a timestamp or the end follows
            if not gen:
                logits[r, :tsb] = neg           # the first token is a timestamp ...
                logits[r, tsb + int(1.0 / SECONDS_PER_TS) + 1:] = neg   # ... no later than 1 s
            seen = [t for t in gen if t >= tsb]
            if seen:                            # timestamps never decrease
                floor = seen[-1] + (0 if last_ts and not prev_ts else 1)
                logits[r, tsb:min(floor, V)] = neg
            lp = torch.log_softmax(logits[r], -1)
            if torch.logsumexp(lp[tsb:], 0) > lp[:tsb].max():
                logits[r, :tsb] = neg
        return logits

    @torch.inference_mode()
    def detect_language(self, enc: torch.Tensor) -> List[str]:
        tk = self.tokens
        if not tk.multilingual or len(tk.lang_to_id) < 2:
            return [next(iter(tk.lang_to_id), "en")] * enc.shape[0]
        B = enc.shape[0]
        st = self._new_state(B, enc)
        logits = self._step(st, torch.full((B,), tk.sot, device=self.device, dtype=torch.long),
                            torch.zeros(B, dtype=torch.long, device=self.device))
        names = list(tk.lang_to_id)
        ids = torch.tensor([tk.lang_to_id[n] for n in names], device=self.device)
        best = logits[:, ids].argmax(-1).tolist()
        return [names[i] for i in best]

    def prompt(self, language: Optional[str], task: str, timestamps: bool) -> List[int]:
        tk = self.tokens
        p = [tk.sot]
        if tk.multilingual:
            if language not in tk.lang_to_id:
                raise ValueError(f"unknown language {language!r}")
            p += [tk.lang_to_id[language], tk.translate if task == "translate" else tk.transcribe]
        if not timestamps:
            p.append(tk.no_timestamps)
        return p

    @torch.inference_mode()
    def decode(self, enc: torch.Tensor, prompts: List[List[int]], max_new_tokens: int = 224,
               timestamps: bool = False, temperature: float = 0.0,
               generator: Optional[torch.Generator] = None) -> List[List[int]]:
        """Batched decoding of every row to <|endoftext|> or ``max_new_tokens``; returns the new tokens."""
        B = enc.shape[0]
        n0 = len(prompts[0])
        if any(len(p) != n0 for p in prompts):
            raise ValueError("decode prompts must have equal length")
        T = self.cfg.max_target_positions
        max_new = min(max_new_tokens, T - n0)
        step = self._runner(B, enc)
        seqs = [list(p) for p in prompts]
        done = [False] * B
        logits = None
        for j in range(n0):  # the prompt, one position at a time (at most four)
            tok = torch.tensor([p[j] for p in prompts], device=self.device)
            logits = step(tok, torch.full((B,), j, device=self.device, dtype=torch.long))
        for j in range(max_new):
            lg = self._rules(logits.clone(), seqs, n0, timestamps)
            if temperature > 0:
                probs = torch.softmax(lg / temperature, -1)
                nxt = torch.multinomial(probs, 1, generator=generator).squeeze(1)
            else:
                nxt = lg.argmax(-1)
            nl = nxt.tolist()
            for r in range(B):
                if done[r]:
                    continue
                seqs[r].append(nl[r])
                if nl[r] == self.tokens.eot:
                    done[r] = True
            if all(done) or j == max_new - 1:
                break
            nxt = torch.tensor([s[-1] for s in seqs], device=self.device)  # finished rows repeat eot
            logits = step(nxt, torch.full((B,), n0 + j, device=self.device, dtype=torch.long))
        return [[t for t in s[n0:] if t != self.tokens.eot] for s in seqs]


# -------------------------------------------------------------------------------------- pipeline
def segments_from_tokens(tokens: List[int], ts_begin: int, offset_s: float) -> List[dict]:
    """Timestamped output -> [{"start", "end", "tokens"}]; text between a pair of timestamps is a
    segment (a trailing open segment ends at the window's end, given as None)."""
    segs, cur, start = [], [], None
    for t in tokens:
        if t >= ts_begin:
            ts = offset_s + (t - ts_begin) * SECONDS_PER_TS
            if start is None:
                start = ts
            else:
                segs.append({"start": round(start, 2), "end": round(ts, 2), "tokens": cur})
                cur, start = [], None
        else:
            cur.append(t)
    if cur:
        segs.append({"start": round(start if start is not None else offset_s, 2), "end": None, "tokens": cur})
    return segs


class WhisperASR:
    """Speech to text over a Whisper checkpoint directory (HF names; tokenizer.json beside it)."""

    def __init__(self, path: str, device: str = "cuda", dtype: torch.dtype = torch.bfloat16,
                 model: Optional[WhisperModel] = None, tokenizer=None, use_cuda_graphs: bool = True):
        self.model = model or WhisperModel.from_pretrained(path, device, dtype, use_cuda_graphs)
        if tokenizer is None and path and os.path.exists(os.path.join(path, "tokenizer.json")):
            from ..utils.tokenizer import HFTokenizer
            tokenizer = HFTokenizer(os.path.join(path, "tokenizer.json"))
        self.tokenizer = tokenizer
        self.name = os.path.basename(os.path.normpath(path)) if path else "whisper"

    def _text(self, ids: List[int]) -> str:
        ids = [t for t in ids if t < self.model.tokens.eot]
        return self.tokenizer.decode(ids).strip() if self.tokenizer is not None else " ".join(map(str, ids))

    def transcribe(self, audios: Sequence, language: Optional[str] = None, task: str = "transcribe",
                   timestamps: bool = False, max_new_tokens: int = 224, temperature: float = 0.0,
                   seed: int = 0) -> List[dict]:
        """Each audio (WAV bytes or a 16 kHz float array) -> {"text", "language", "segments",
        "duration"}. Every window of every audio is encoded and decoded in one batch."""
        m = self.model
        pcm = [load_audio(a) if isinstance(a, (bytes, bytearray)) else np.asarray(a, dtype=np.float32)
               for a in audios]
        wins = [(i, s, e) for i, x in enumerate(pcm) for s, e in split_windows(x)]
        mel = torch.stack([log_mel_spectrogram(pcm[i][s:e], m.cfg.num_mel_bins, str(m.device))
                           for i, s, e in wins])
        enc = m.encode(mel)
        langs = [language] * len(wins) if language or not m.tokens.multilingual else m.detect_language(enc)
        if not m.tokens.multilingual:
            langs = [language or "en"] * len(wins)
        gen = torch.Generator(device=m.device).manual_seed(seed) if temperature > 0 else None
        out_tok: List[Optional[List[int]]] = [None] * len(wins)
        # windows with the same prompt (language) decode together
        for lang in sorted(set(langs), key=str):
            idx = [k for k, l in enumerate(langs) if l == lang]
            toks = m.decode(enc[idx], [m.prompt(lang, task, timestamps)] * len(idx), max_new_tokens, timestamps,
                            temperature, gen)
            for k, t in zip(idx, toks):
                out_tok[k] = t
        results = []
        for i, x in enumerate(pcm):
            texts, segs, ls = [], [], []
            for k, (j, s, e) in enumerate(wins):
                if j != i:
                    continue
                ls.append(langs[k])
                toks = out_tok[k]
                if timestamps:
                    for sg in segments_from_tokens(toks, m.tokens.ts_begin, s / SAMPLE_RATE):
                        sg["end"] = sg["end"] if sg["end"] is not None else round(e / SAMPLE_RATE, 2)
                        sg["text"] = self._text(sg.pop("tokens"))
                        segs.append(sg)
                        texts.append(sg["text"])
                else:
                    t = self._text(toks)
                    texts.append(t)
                    segs.append({"start": round(s / SAMPLE_RATE, 2), "end": round(e / SAMPLE_RATE, 2), "text": t})
            results.append({"text": " ".join(t for t in texts if t), "language": max(set(ls), key=ls.count),
                            "segments": segs, "duration": round(len(x) / SAMPLE_RATE, 3)})
        return results
