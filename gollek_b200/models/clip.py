"""CLIP text encoder (the conditioning encoder of Stable Diffusion and CLIP text embeddings).

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


class CLIPTextEncoder:
    def __init__(self, cfg: CLIPTextConfig, get: Callable[[str], torch.Tensor], device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        names = [("text_model.embeddings.token_embedding.weight", "tok"),
                 ("text_model.embeddings.position_embedding.weight", "pos"),
                 ("text_model.final_layer_norm.weight", "lnf_w"), ("text_model.final_layer_norm.bias", "lnf_b")]
        self.w: Dict[str, torch.Tensor] = {k: get(n).to(self.device, dtype).contiguous() for n, k in names}
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"text_model.encoder.layers.{i}."

            def t(n):
                return get(p + n).to(self.device, dtype).contiguous()
            qkv_w = torch.cat([t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"), t("self_attn.v_proj.weight")])
            qkv_b = torch.cat([t("self_attn.q_proj.bias"), t("self_attn.k_proj.bias"), t("self_attn.v_proj.bias")])
            self.layers.append({"ln1_w": t("layer_norm1.weight"), "ln1_b": t("layer_norm1.bias"),
                                "qkv_w": qkv_w, "qkv_b": qkv_b, "o_w": t("self_attn.out_proj.weight"),
                                "o_b": t("self_attn.out_proj.bias"), "ln2_w": t("layer_norm2.weight"),
                                "ln2_b": t("layer_norm2.bias"), "fc1_w": t("mlp.fc1.weight"), "fc1_b": t("mlp.fc1.bias"),
                                "fc2_w": t("mlp.fc2.weight"), "fc2_b": t("mlp.fc2.bias")})
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

    def _ln(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, w, self.cfg.layer_norm_eps, center=True) + b

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
        hd = d // nh
        h = (self.w["tok"][ids] + self.w["pos"][:S][None]).reshape(B * S, d).contiguous()
        causal = torch.full((S, S), float("-inf"), device=self.device).triu(1)
        for L in self.layers:
            x = self._ln(h, L["ln1_w"], L["ln1_b"])
            qkv = (ops.linear(x, L["qkv_w"]) + L["qkv_b"]).view(B, S, 3, nh, hd).float()
            q, k, v = qkv.unbind(2)
            s = torch.einsum("bqhd,bkhd->bhqk", q, k) * hd ** -0.5 + causal
            a = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), v).reshape(B * S, d).to(self.dtype)
            h = h + ops.linear(a.contiguous(), L["o_w"]) + L["o_b"]
            x = self._ln(h, L["ln2_w"], L["ln2_b"])
            m = _act(ops.linear(x, L["fc1_w"]) + L["fc1_b"], cfg.hidden_act)
            h = h + ops.linear(m.contiguous(), L["fc2_w"]) + L["fc2_b"]
        last = self._ln(h, self.w["lnf_w"], self.w["lnf_b"]).view(B, S, d)
        if cfg.eos_token_id == 2:  # legacy checkpoints: the end-of-text id is the largest id
            pos = ids.argmax(-1)
        else:
            pos = (ids == cfg.eos_token_id).int().argmax(-1)
        pooled = last[torch.arange(B, device=self.device), pos]
        emb = ops.linear(pooled.contiguous(), self.proj) if self.proj is not None else None
        return {"last_hidden_state": last, "pooler_output": pooled, "text_embeds": emb}
