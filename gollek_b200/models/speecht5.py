"""SpeechT5 text-to-speech (text -> 80-bin log-mel spectrogram -> 16 kHz waveform).

Model (Ao et al., "SpeechT5: Unified-Modal Encoder-Decoder Pre-Training for Spoken Language
Processing", 2022), loaded from HF-layout ``SpeechT5ForTextToSpeech`` and ``SpeechT5HifiGan``
checkpoints; the reference serves it from Java (runner/safetensor/gollek-safetensor-audio/…/audio/
SpeechT5Engine.java) behind its audio REST resource:

* text encoder: token embeddings + alpha-scaled sinusoidal positions, LayerNorm, post-norm layers
  whose self-attention adds a relative-position term q . pe[clip(i - j)] (a learned table over
  +-``encoder_max_relative_position``);
* speech decoder: prenet (two ReLU layers with dropout kept on at inference, a fresh seeded mask
  per step; then a projection and alpha-scaled positions, then the unit-normalised speaker
  embedding concatenated and projected), post-norm layers with causal self-attention (cache
  of past frames) and cross-attention (encoder keys / values computed once);
* each decoder step emits ``reduction_factor`` mel frames (feat_out) and a stop logit (prob_out);
  decoding ends when sigmoid(stop) summed over the step's frames reaches ``threshold`` (after
  ``minlenratio``, before ``maxlenratio`` times the text length / reduction factor); a convolutional
  postnet (5 conv + batch-norm layers, tanh between) refines the whole spectrogram;
* HiFi-GAN vocoder: input normalised by the checkpoint's mean / scale, transposed-convolution
  upsampling, multi-kernel dilated residual blocks averaged per stage, tanh output.

The linear layers run through ``ops.linear`` (tcgen05 GEMM on the GPU); attention, norms and the
convolutions are short sequences and use PyTorch operators.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Optional

import torch
import torch.nn.functional as F

from .. import ops


def _sinusoid(n: int, dim: int) -> torch.Tensor:
    pos = torch.arange(n, dtype=torch.float32)[:, None]
    div = torch.exp(torch.arange(0, dim, 2, dtype=torch.float32) * -(math.log(10000.0) / dim))
    pe = torch.zeros(n, dim)
    pe[:, 0::2] = torch.sin(pos * div)
    pe[:, 1::2] = torch.cos(pos * div)
    return pe


class SpeechT5TTS:
    """Greedy SpeechT5 text-to-speech for one utterance at a time."""

    def __init__(self, cfg: dict, get: Callable[[str], torch.Tensor], device: str = "cpu",
                 dtype: torch.dtype = torch.float32):
        self.cfg, self.device, self.dtype = cfg, device, dtype
        self.d = int(cfg["hidden_size"])
        self.heads_enc = int(cfg["encoder_attention_heads"])
        self.heads_dec = int(cfg["decoder_attention_heads"])
        self.mel = int(cfg.get("num_mel_bins", 80))
        self.rf = int(cfg.get("reduction_factor", 2))
        self.eps = float(cfg.get("layer_norm_eps", 1e-5))
        self.max_rel = int(cfg.get("encoder_max_relative_position", 160))
        self.prenet_dropout = float(cfg.get("speech_decoder_prenet_dropout", 0.5))
        self.act = cfg.get("hidden_act", "gelu")
        self.w: Dict[str, torch.Tensor] = {}
        self._get = get
        self.pe_text = _sinusoid(int(cfg.get("max_text_positions", 450)), self.d).to(device)
        self.pe_speech = _sinusoid(int(cfg.get("max_speech_positions", 4000)), self.d).to(device)
        self.n_enc, self.n_dec = int(cfg["encoder_layers"]), int(cfg["decoder_layers"])
        self.n_post = int(cfg.get("speech_decoder_postnet_layers", 5))
        self.n_prenet = int(cfg.get("speech_decoder_prenet_layers", 2))

    def t(self, name: str, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        key = (name, dtype)
        if key not in self.w:
            self.w[key] = self._get(name).to(self.device, dtype or torch.float32)
        return self.w[key]

    # ----------------------------------------------------------------------------------- blocks
    def _lin(self, x: torch.Tensor, p: str) -> torch.Tensor:
        w = self.t(p + ".weight", self.dtype)
        if w.shape[0] % 8 or w.shape[1] % 8:  # e.g. the 2-way stop head: below the GEMM's 16-byte rows
            y = x.to(self.dtype) @ w.t()
        else:
            y = ops.linear(x.to(self.dtype).contiguous(), w)
        return y.float() + self.t(p + ".bias")

    def _ln(self, x: torch.Tensor, p: str) -> torch.Tensor:
        return F.layer_norm(x, (self.d,), self.t(p + ".weight"), self.t(p + ".bias"), self.eps)

    def _ffn(self, x: torch.Tensor, p: str) -> torch.Tensor:
        h = self._lin(x, p + ".intermediate_dense")
        h = F.gelu(h) if self.act == "gelu" else F.relu(h)
        return self._lin(h, p + ".output_dense")

    def _attn(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int,
              bias: Optional[torch.Tensor] = None, causal: bool = False) -> torch.Tensor:
        """q [Tq, d] (already scaled), k / v [Tk, d]; bias [Tq, Tk, hd] relative-position keys."""
        hd = self.d // heads
        qh, kh, vh = q.view(-1, heads, hd), k.view(-1, heads, hd), v.view(-1, heads, hd)
        s = torch.einsum("qhd,khd->hqk", qh, kh)
        if bias is not None:
            s = s + torch.einsum("qhd,qkd->hqk", qh, bias)
        if causal:
            Tq, Tk = s.shape[1], s.shape[2]
            s = s.masked_fill(torch.ones(Tq, Tk, dtype=torch.bool, device=s.device).triu(Tk - Tq + 1), float("-inf"))
        return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vh).reshape(-1, self.d)

    # ----------------------------------------------------------------------------------- encoder
    def encode(self, ids: torch.Tensor) -> torch.Tensor:
        p = "speecht5.encoder."
        S = ids.shape[0]
        x = self.t(p + "prenet.embed_tokens.weight")[ids.long().to(self.device)]
        x = x + self.t(p + "prenet.encode_positions.alpha") * self.pe_text[:S]
        x = self._ln(x, p + "wrapped_encoder.layer_norm")
        rel = torch.arange(S, device=self.device)
        rel = (rel[:, None] - rel[None, :]).clamp(-self.max_rel, self.max_rel - 1) + self.max_rel
        bias = self.t(p + "wrapped_encoder.embed_positions.pe_k.weight")[rel]          # [S, S, hd]
        hd = self.d // self.heads_enc
        for i in range(self.n_enc):
            lp = f"{p}wrapped_encoder.layers.{i}."
            q = self._lin(x, lp + "attention.q_proj") * hd ** -0.5
            a = self._attn(q, self._lin(x, lp + "attention.k_proj"), self._lin(x, lp + "attention.v_proj"),
                           self.heads_enc, bias)
            x = self._ln(x + self._lin(a, lp + "attention.out_proj"), lp + "layer_norm")
            x = self._ln(x + self._ffn(x, lp + "feed_forward"), lp + "final_layer_norm")
        return x

    # ----------------------------------------------------------------------------------- decoder
    def _prenet(self, frames: torch.Tensor, spk: torch.Tensor, masks) -> torch.Tensor:
        """Prenet output of the last frame of ``frames`` [T, mel] (positions 0..T-1)."""
        p = "speecht5.decoder.prenet."
        h = frames[-1:]
        for i in range(self.n_prenet):
            h = F.relu(self._lin(h, f"{p}layers.{i}"))
            if masks is not None:
                h = h * masks[i]
        h = self._lin(h, p + "final_layer")
        h = h + self.t(p + "encode_positions.alpha") * self.pe_speech[frames.shape[0] - 1]
        h = torch.cat([h, F.normalize(spk.float().to(self.device), dim=-1)[None]], -1)
        return F.relu(self._lin(h, p + "speaker_embeds_layer"))

    def _post(self, spec: torch.Tensor) -> torch.Tensor:
        """Convolutional postnet over a [T, mel] spectrogram (residual)."""
        p = "speech_decoder_postnet.layers."
        h = spec.t()[None]
        for i in range(self.n_post):
            w = self.t(f"{p}{i}.conv.weight")
            h = F.conv1d(h, w, padding=(w.shape[-1] - 1) // 2)
            h = F.batch_norm(h, self.t(f"{p}{i}.batch_norm.running_mean"), self.t(f"{p}{i}.batch_norm.running_var"),
                             self.t(f"{p}{i}.batch_norm.weight"), self.t(f"{p}{i}.batch_norm.bias"), False, 0.0,
                             float(self.cfg.get("batch_norm_eps", 1e-5)))
            if i < self.n_post - 1:
                h = torch.tanh(h)
        return spec + h[0].t()

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, speaker: torch.Tensor, threshold: float = 0.5, minlenratio: float = 0.0,
                 maxlenratio: float = 20.0, seed: int = 0) -> torch.Tensor:
        """Token ids [S] and a speaker embedding -> refined log-mel spectrogram [T, mel]."""
        enc = self.encode(ids)
        S = enc.shape[0]
        maxlen = int(S * maxlenratio / self.rf)
        minlen = int(S * minlenratio / self.rf)
        hd = self.d // self.heads_dec
        p = "speecht5.decoder.wrapped_decoder.layers."
        cross = [(self._lin(enc, f"{p}{i}.encoder_attn.k_proj"), self._lin(enc, f"{p}{i}.encoder_attn.v_proj"))
                 for i in range(self.n_dec)]
        kv = [[None, None] for _ in range(self.n_dec)]
        # the prenet's dropout stays on at inference (the model was trained to decode through it): a fresh
        # mask per step from a seeded generator, so an utterance is reproducible from (text, speaker, seed)
        g = torch.Generator(device="cpu").manual_seed(seed)
        units = int(self.cfg.get("speech_decoder_prenet_units", 256))
        frames = torch.zeros(1, self.mel, device=self.device)
        spec = []
        step = 0
        while True:
            step += 1
            masks = None
            if self.prenet_dropout > 0:
                masks = [(torch.rand(units, generator=g) >= self.prenet_dropout).float().to(self.device)
                         / (1 - self.prenet_dropout) for _ in range(self.n_prenet)]
            x = self._prenet(frames, speaker, masks)
            for i in range(self.n_dec):
                lp = f"{p}{i}."
                q = self._lin(x, lp + "self_attn.q_proj") * hd ** -0.5
                k, v = self._lin(x, lp + "self_attn.k_proj"), self._lin(x, lp + "self_attn.v_proj")
                kv[i][0] = k if kv[i][0] is None else torch.cat([kv[i][0], k])
                kv[i][1] = v if kv[i][1] is None else torch.cat([kv[i][1], v])
                a = self._attn(q, kv[i][0], kv[i][1], self.heads_dec)
                x = self._ln(x + self._lin(a, lp + "self_attn.out_proj"), lp + "self_attn_layer_norm")
                q = self._lin(x, lp + "encoder_attn.q_proj") * hd ** -0.5
                a = self._attn(q, cross[i][0], cross[i][1], self.heads_dec)
                x = self._ln(x + self._lin(a, lp + "encoder_attn.out_proj"), lp + "encoder_attn_layer_norm")
                x = self._ln(x + self._ffn(x, lp + "feed_forward"), lp + "final_layer_norm")
            out = self._lin(x, "speech_decoder_postnet.feat_out").view(self.rf, self.mel)
            spec.append(out)
            frames = torch.cat([frames, out[-1:]])
            prob = torch.sigmoid(self._lin(x, "speech_decoder_postnet.prob_out"))
            if step < minlen:
                continue
            if step >= maxlen or float(prob.sum()) >= threshold:
                break
        return self._post(torch.cat(spec))


class HiFiGan:
    """HiFi-GAN vocoder: log-mel [T, mel] -> waveform [T * prod(upsample_rates)]."""

    def __init__(self, cfg: dict, get: Callable[[str], torch.Tensor], device: str = "cpu"):
        self.cfg, self.device = cfg, device
        self.rates = list(cfg.get("upsample_rates", [4, 4, 4, 4]))
        self.kernels = list(cfg.get("resblock_kernel_sizes", [3, 7, 11]))
        self.dilations = [list(d) for d in cfg.get("resblock_dilation_sizes", [[1, 3, 5]] * 3)]
        self.slope = float(cfg.get("leaky_relu_slope", 0.1))
        self.normalize = bool(cfg.get("normalize_before", True))
        self.sampling_rate = int(cfg.get("sampling_rate", 16000))
        self._get, self.w = get, {}

    def t(self, name: str) -> torch.Tensor:
        if name not in self.w:
            self.w[name] = self._get(name).to(self.device, torch.float32)
        return self.w[name]

    def _conv(self, x, p, dilation=1):
        w = self.t(p + ".weight")
        return F.conv1d(x, w, self.t(p + ".bias"), padding=(w.shape[-1] * dilation - dilation) // 2, dilation=dilation)

    @torch.no_grad()
    def __call__(self, spec: torch.Tensor) -> torch.Tensor:
        x = spec.float().to(self.device)
        if self.normalize:
            x = (x - self.t("mean")) / self.t("scale")
        h = self._conv(x.t()[None], "conv_pre")
        nk = len(self.kernels)
        for i, (r, ks) in enumerate(zip(self.rates, self.cfg.get("upsample_kernel_sizes", [8, 8, 8, 8]))):
            h = F.leaky_relu(h, self.slope)
            h = F.conv_transpose1d(h, self.t(f"upsampler.{i}.weight"), self.t(f"upsampler.{i}.bias"), stride=r,
                                   padding=(ks - r) // 2)
            acc = None
            for j, dil in enumerate(self.dilations[:nk]):
                y = h
                b = f"resblocks.{i * nk + j}"
                for m, d in enumerate(dil):
                    z = self._conv(F.leaky_relu(y, self.slope), f"{b}.convs1.{m}", d)
                    y = y + self._conv(F.leaky_relu(z, self.slope), f"{b}.convs2.{m}")
                acc = y if acc is None else acc + y
            h = acc / nk
        h = self._conv(F.leaky_relu(h), "conv_post")  # default negative slope 0.01 before the output conv
        return torch.tanh(h)[0, 0]


class SpeechSynth:
    """Text -> waveform with a SpeechT5 text-to-speech checkpoint directory and a HiFi-GAN vocoder
    directory (HF layouts: config.json + safetensors). Text becomes ids through ``tokenizer``
    (callable) or, by default, the checkpoint's character-level SentencePiece model
    (``spm_char.model``) with the end-of-sequence id appended. Voices are speaker embeddings stored as
    ``speakers/<voice>.npy`` (or ``.pt``) in the checkpoint directory; ``voice=None`` uses a fixed
    seeded unit vector."""

    def __init__(self, model_dir: str, vocoder_dir: str, device: str = "cpu", dtype: torch.dtype = torch.float32,
                 tokenizer: Optional[Callable[[str], list]] = None):
        import json
        import os
        from ..loaders.safetensors import SafetensorsCheckpoint
        with open(os.path.join(model_dir, "config.json")) as f:
            self.cfg = json.load(f)
        with open(os.path.join(vocoder_dir, "config.json")) as f:
            vcfg = json.load(f)
        self.model_dir = model_dir
        self.tts = SpeechT5TTS(self.cfg, SafetensorsCheckpoint(model_dir).get, device, dtype)
        self.vocoder = HiFiGan(vcfg, SafetensorsCheckpoint(vocoder_dir).get, device)
        self.sampling_rate = self.vocoder.sampling_rate
        if tokenizer is None:
            import sentencepiece as spm
            sp = spm.SentencePieceProcessor(model_file=os.path.join(model_dir, "spm_char.model"))
            eos = int(self.cfg.get("eos_token_id", 2))
            tokenizer = lambda text: sp.encode(text) + [eos]  # noqa: E731
        self.tokenizer = tokenizer

    def speaker(self, voice: Optional[str]) -> torch.Tensor:
        import os
        dim = int(self.cfg.get("speaker_embedding_dim", 512))
        if voice:
            if not voice.replace("-", "").replace("_", "").isalnum():
                raise ValueError(f"bad voice name {voice!r}")
            for ext in (".npy", ".pt"):
                path = os.path.join(self.model_dir, "speakers", voice + ext)
                if os.path.exists(path):
                    if ext == ".npy":
                        import numpy as np
                        return torch.from_numpy(np.load(path)).float().flatten()[:dim]
                    return torch.load(path).float().flatten()[:dim]
            raise ValueError(f"unknown voice {voice!r}")
        return torch.randn(dim, generator=torch.Generator().manual_seed(0))

    def synthesize(self, text: str, voice: Optional[str] = None, seed: int = 0):
        """-> float32 numpy waveform in [-1, 1] at ``sampling_rate``."""
        ids = torch.tensor(self.tokenizer(text), dtype=torch.long)
        if ids.numel() == 0:
            raise ValueError("empty input")
        spec = self.tts.generate(ids, self.speaker(voice), seed=seed)
        return self.vocoder(spec).cpu().numpy()

    def wav_bytes(self, text: str, voice: Optional[str] = None, seed: int = 0) -> bytes:
        import io
        import wave
        import numpy as np
        pcm = (np.clip(self.synthesize(text, voice, seed), -1.0, 1.0) * 32767.0).astype("<i2")
        buf = io.BytesIO()
        with wave.open(buf, "wb") as w:
            w.setnchannels(1)
            w.setsampwidth(2)
            w.setframerate(self.sampling_rate)
            w.writeframes(pcm.tobytes())
        return buf.getvalue()
