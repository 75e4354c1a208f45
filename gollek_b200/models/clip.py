"""CLIP text and image encoders (the conditioning encoder of Stable Diffusion; CLIP text / image embeddings).

Reference behaviour: runner/safetensor/gollek-runner-safetensor/…/runner/sd/CLIPModel.java:17-118
(token + position embeddings, pre-LayerNorm blocks with causal self-attention and a GELU MLP,
final LayerNorm; Hugging Face ``text_model.*`` tensor names). Here the projections run on the
tcgen05 GEMM (``ops.linear``) and the LayerNorm on the K1 norm kernel in its centred mode (bias
added after); attention over at most ``max_position_embeddings`` (77) tokens is a plain causal
softmax. ``encode`` also returns the pooled state at the end-of-text token and, when the
checkpoint has ``text_projection``, the projected text embedding (as transformers'
CLIPTextModelWithProjection).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Callable, Dict, Optional

import torch

from .. import ops


@dataclass
class CLIPTextConfig:
    vocab_size: int = 49408
    hidden_size: int = 768
    intermediate_size: int = 3072
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    max_position_embeddings: int = 77
    layer_norm_eps: float = 1e-5
    hidden_act: str = "quick_gelu"
    eos_token_id: int = 49407
    projection_dim: int = 0  # 0: no text projection

    @staticmethod
    def from_hf(d: dict) -> "CLIPTextConfig":
        t = d.get("text_config", d)
        return CLIPTextConfig(
            vocab_size=int(t.get("vocab_size", 49408)), hidden_size=int(t.get("hidden_size", 768)),
            intermediate_size=int(t.get("intermediate_size", 3072)),
            num_hidden_layers=int(t.get("num_hidden_layers", 12)),
            num_attention_heads=int(t.get("num_attention_heads", 12)),
            max_position_embeddings=int(t.get("max_position_embeddings", 77)),
            layer_norm_eps=float(t.get("layer_norm_eps", 1e-5)), hidden_act=str(t.get("hidden_act", "quick_gelu")),
            eos_token_id=int(t.get("eos_token_id", 49407)),
            projection_dim=int(t.get("projection_dim", d.get("projection_dim", 0)) or 0))


def _act(x: torch.Tensor, kind: str) -> torch.Tensor:
    xf = x.float()
    if kind == "quick_gelu":
        y = xf * torch.sigmoid(1.702 * xf)
    elif kind in ("gelu", "gelu_new", "gelu_pytorch_tanh"):
        y = torch.nn.functional.gelu(xf, approximate="none" if kind == "gelu" else "tanh")
    else:
        raise ValueError(f"unsupported CLIP activation {kind!r}")
    return y.to(x.dtype)


def _has(get, name: str) -> bool:
    try:
        get(name)
        return True
    except KeyError:
        return False


def _layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    return ops.rms_norm(x.contiguous(), w, eps, center=True) + b


def _load_blocks(get, prefix: str, n: int, device, dtype) -> list:
    layers = []
    for i in range(n):
        p = f"{prefix}.{i}."

        def t(name):
            return get(p + name).to(device, dtype).contiguous()
        layers.append({"ln1_w": t("layer_norm1.weight"), "ln1_b": t("layer_norm1.bias"),
                       "qkv_w": torch.cat([t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"),
                                           t("self_attn.v_proj.weight")]),
                       "qkv_b": torch.cat([t("self_attn.q_proj.bias"), t("self_attn.k_proj.bias"),
                                           t("self_attn.v_proj.bias")]),
                       "o_w": t("self_attn.out_proj.weight"), "o_b": t("self_attn.out_proj.bias"),
                       "ln2_w": t("layer_norm2.weight"), "ln2_b": t("layer_norm2.bias"),
                       "fc1_w": t("mlp.fc1.weight"), "fc1_b": t("mlp.fc1.bias"),
                       "fc2_w": t("mlp.fc2.weight"), "fc2_b": t("mlp.fc2.bias")})
    return layers


def _encoder(h: torch.Tensor, layers: list, B: int, S: int, nh: int, eps: float, act: str, causal: bool) -> torch.Tensor:
    """Pre-LayerNorm transformer blocks over h [B * S, d] (causal for text, full for image patches)."""
    d = h.shape[1]
    hd = d // nh
    mask = torch.full((S, S), float("-inf"), device=h.device).triu(1) if causal else None
    for L in layers:
        x = _layer_norm(h, L["ln1_w"], L["ln1_b"], eps)
        qkv = (ops.linear(x, L["qkv_w"]) + L["qkv_b"]).view(B, S, 3, nh, hd).float()
        q, k, v = qkv.unbind(2)
        s = torch.einsum("bqhd,bkhd->bhqk", q, k) * hd ** -0.5
        if mask is not None:
            s = s + mask
        a = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), v).reshape(B * S, d).to(h.dtype)
        h = h + ops.linear(a.contiguous(), L["o_w"]) + L["o_b"]
        x = _layer_norm(h, L["ln2_w"], L["ln2_b"], eps)
        m = _act(ops.linear(x, L["fc1_w"]) + L["fc1_b"], act)
        h = h + ops.linear(m.contiguous(), L["fc2_w"]) + L["fc2_b"]
    return h


class CLIPTextEncoder:
    def __init__(self, cfg: CLIPTextConfig, get: Callable[[str], torch.Tensor], device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        names = [("text_model.embeddings.token_embedding.weight", "tok"),
                 ("text_model.embeddings.position_embedding.weight", "pos"),
                 ("text_model.final_layer_norm.weight", "lnf_w"), ("text_model.final_layer_norm.bias", "lnf_b")]
        self.w: Dict[str, torch.Tensor] = {k: get(n).to(self.device, dtype).contiguous() for n, k in names}
        self.layers = _load_blocks(get, "text_model.encoder.layers", cfg.num_hidden_layers, self.device, dtype)
        self.proj = None
        try:
            self.proj = get("text_projection.weight").to(self.device, dtype).contiguous()
        except KeyError:
            pass

    @staticmethod
    def from_pretrained(path: str, device: str = "cuda", dtype: torch.dtype = torch.bfloat16) -> "CLIPTextEncoder":
        from ..loaders.safetensors import SafetensorsCheckpoint
        with open(os.path.join(path, "config.json")) as f:
            cfg = CLIPTextConfig.from_hf(json.load(f))
        return CLIPTextEncoder(cfg, SafetensorsCheckpoint(path).get, device, dtype)

    @torch.inference_mode()
    def encode(self, input_ids: torch.Tensor) -> Dict[str, Optional[torch.Tensor]]:
        """input_ids [B, S] (S <= max_position_embeddings) -> {"last_hidden_state" [B, S, d],
        "pooler_output" [B, d] (state at the end-of-text token), "text_embeds" [B, proj] or None}."""
        cfg = self.cfg
        ids = input_ids.to(self.device).long()
        B, S = ids.shape
        if S > cfg.max_position_embeddings:
            raise ValueError(f"at most {cfg.max_position_embeddings} tokens")
        d, nh = cfg.hidden_size, cfg.num_attention_heads
        h = (self.w["tok"][ids] + self.w["pos"][:S][None]).reshape(B * S, d).contiguous()
        h = _encoder(h, self.layers, B, S, nh, cfg.layer_norm_eps, cfg.hidden_act, causal=True)
        last = _layer_norm(h, self.w["lnf_w"], self.w["lnf_b"], cfg.layer_norm_eps).view(B, S, d)
        if cfg.eos_token_id == 2:  # legacy checkpoints: the end-of-text id is the largest id
            pos = ids.argmax(-1)
        else:
            pos = (ids == cfg.eos_token_id).int().argmax(-1)
        pooled = last[torch.arange(B, device=self.device), pos]
        emb = ops.linear(pooled.contiguous(), self.proj) if self.proj is not None else None
        return {"last_hidden_state": last, "pooler_output": pooled, "text_embeds": emb}


@dataclass
class CLIPVisionConfig:
    hidden_size: int = 1024
    intermediate_size: int = 4096
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    image_size: int = 224
    patch_size: int = 14
    num_channels: int = 3
    layer_norm_eps: float = 1e-5
    hidden_act: str = "quick_gelu"
    projection_dim: int = 0

    @staticmethod
    def from_hf(d: dict) -> "CLIPVisionConfig":
        v = d.get("vision_config", d)
        return CLIPVisionConfig(
            hidden_size=int(v.get("hidden_size", 1024)), intermediate_size=int(v.get("intermediate_size", 4096)),
            num_hidden_layers=int(v.get("num_hidden_layers", 24)),
            num_attention_heads=int(v.get("num_attention_heads", 16)), image_size=int(v.get("image_size", 224)),
            patch_size=int(v.get("patch_size", 14)), num_channels=int(v.get("num_channels", 3)),
            layer_norm_eps=float(v.get("layer_norm_eps", 1e-5)), hidden_act=str(v.get("hidden_act", "quick_gelu")),
            projection_dim=int(v.get("projection_dim", d.get("projection_dim", 0)) or 0))


class CLIPVisionEncoder:
    """CLIP image tower (ViT): non-overlapping patches projected by the patch embedding (a GEMM over
    the unfolded patches), a class token, position embeddings, pre-LayerNorm, full self-attention
    blocks, post-LayerNorm of the class token and the visual projection (HF ``vision_model.*``)."""

    def __init__(self, cfg: CLIPVisionConfig, get: Callable[[str], torch.Tensor], device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        pre = "vision_tower.vision_model." if _has(get, "vision_tower.vision_model.pre_layrnorm.weight") \
            else "vision_model."

        def t(n):
            return get(pre + n).to(self.device, dtype).contiguous()
        pw = t("embeddings.patch_embedding.weight").reshape(cfg.hidden_size, -1)
        self.kpad = (-pw.shape[1]) % 8  # the GEMM wants K % 8 == 0 (ViT-L/14: 3*14*14 = 588 -> 592)
        self.patch_w = torch.nn.functional.pad(pw, (0, self.kpad)).contiguous()
        self.cls = t("embeddings.class_embedding")
        self.pos = t("embeddings.position_embedding.weight")
        self.pre_w, self.pre_b = t("pre_layrnorm.weight"), t("pre_layrnorm.bias")
        self.post_w, self.post_b = t("post_layernorm.weight"), t("post_layernorm.bias")
        self.layers = _load_blocks(get, pre + "encoder.layers", cfg.num_hidden_layers, self.device, dtype)
        self.proj = None
        try:
            self.proj = get("visual_projection.weight").to(self.device, dtype).contiguous()
        except KeyError:
            pass

    def _embed(self, pixel_values: torch.Tensor):
        cfg = self.cfg
        x = pixel_values.to(self.device, self.dtype)
        B = x.shape[0]
        p, d = cfg.patch_size, cfg.hidden_size
        patches = torch.nn.functional.unfold(x, kernel_size=p, stride=p).transpose(1, 2)  # [B, n, C*p*p]
        n = patches.shape[1]
        pm = torch.nn.functional.pad(patches.reshape(B * n, -1), (0, self.kpad)).contiguous()
        pe = ops.linear(pm, self.patch_w).view(B, n, d)
        h = torch.cat([self.cls.view(1, 1, d).expand(B, 1, d), pe], 1) + self.pos[: n + 1][None]
        S = n + 1
        return _layer_norm(h.reshape(B * S, d), self.pre_w, self.pre_b, cfg.layer_norm_eps), B, S

    @torch.inference_mode()
    def hidden_state(self, pixel_values: torch.Tensor, layer: int = -1) -> torch.Tensor:
        """Hidden state [B, 1 + patches, d] after ``layer`` blocks (HF ``hidden_states[layer]``: 0 is
        the pre-LayerNorm embeddings, negative counts from the end)."""
        cfg = self.cfg
        n = len(self.layers)
        k = layer if layer >= 0 else n + 1 + layer
        h, B, S = self._embed(pixel_values)
        h = _encoder(h, self.layers[:k], B, S, cfg.num_attention_heads, cfg.layer_norm_eps, cfg.hidden_act,
                     causal=False)
        return h.view(B, S, cfg.hidden_size)

    @torch.inference_mode()
    def encode(self, pixel_values: torch.Tensor) -> Dict[str, Optional[torch.Tensor]]:
        """pixel_values [B, C, image_size, image_size] (already normalised) -> {"last_hidden_state"
        [B, 1 + patches, d], "pooler_output" [B, d], "image_embeds" [B, proj] or None}."""
        cfg = self.cfg
        h, B, S = self._embed(pixel_values)
        d = cfg.hidden_size
        h = _encoder(h, self.layers, B, S, cfg.num_attention_heads, cfg.layer_norm_eps, cfg.hidden_act, causal=False)
        last = h.view(B, S, d)
        pooled = _layer_norm(last[:, 0].contiguous(), self.post_w, self.post_b, cfg.layer_norm_eps)
        emb = ops.linear(pooled.contiguous(), self.proj) if self.proj is not None else None
        return {"last_hidden_state": last, "pooler_output": pooled, "image_embeds": emb}
