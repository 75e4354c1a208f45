"""Vision-language serving, LLaVA layout: a CLIP image tower + an MLP projector whose output rows
replace the image placeholder tokens in the language model's input embeddings.

* ``preprocess_image``: resize the shorter side to the tower's image size (bicubic; the longer side
  scaled and truncated to an integer), centre crop,
  scale to [0, 1], normalise with the CLIP mean / std (as CLIPImageProcessor).
* ``LlavaVision.encode``: hidden states of layer ``vision_feature_layer`` of the CLIP tower (the
  patch rows; the class row is dropped for the "default" selection), then linear → GELU → linear
  (``multi_modal_projector``) into the language model's hidden size: one row per patch.
* ``load_llava``: splits a LLaVA checkpoint (HF ``LlavaForConditionalGeneration`` names, new
  ``model.language_model.*`` or old ``language_model.model.*`` layout) into the text model's
  ModelConfig + weight getter (served by the ordinary engine) and the vision side.
The engine expands every image placeholder token of a prompt to the image's patch count, keeps the
projected rows with the sequence and writes them over the embedding output of those prompt rows
in the prefill (``AttnMetadata.mm_rows`` / ``mm_embeds``); the image content salts the
prefix-cache block hashes, so equal token ids with different images never share KV.

Reference: runner/safetensor/gollek-safetensor-vision/…/vision/VisionEncoder.java and
MultimodalModelFamilies.java (image encoder + projector feeding a text decoder).
"""
from __future__ import annotations

import json
import os
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from .clip import CLIPVisionConfig, CLIPVisionEncoder, _act

CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


def preprocess_image(img, size: int, mean=CLIP_MEAN, std=CLIP_STD) -> torch.Tensor:
    """PIL image (or HxWx3 uint8 array) -> normalised pixel values [3, size, size] fp32."""
    from PIL import Image
    if not isinstance(img, Image.Image):
        img = Image.fromarray(np.asarray(img, dtype=np.uint8))
    img = img.convert("RGB")
    w, h = img.size
    # shorter side -> size, longer side scaled and truncated (as CLIPImageProcessor)
    nw, nh = (size, max(size, int(size * h / w))) if w <= h else (max(size, int(size * w / h)), size)
    img = img.resize((nw, nh), Image.BICUBIC)
    left, top = (nw - size) // 2, (nh - size) // 2
    img = img.crop((left, top, left + size, top + size))
    x = torch.from_numpy(np.asarray(img, dtype=np.float32) / 255.0).permute(2, 0, 1)
    return (x - torch.tensor(mean)[:, None, None]) / torch.tensor(std)[:, None, None]


def decode_image(data: bytes):
    """Image file bytes (PNG, JPEG, ...) -> PIL image."""
    import io
    from PIL import Image
    return Image.open(io.BytesIO(data))


def load_image_url(url: str, timeout_s: float = 10.0):
    """An OpenAI ``image_url``: a ``data:image/...;base64,`` URL, or an http(s) URL fetched with a
    timeout. Other schemes (``file:`` ...) are refused: a request must not read server files."""
    import base64
    if url.startswith("data:"):
        head, _, payload = url.partition(",")
        if ";base64" not in head:
            raise ValueError("image data URL must be base64-encoded")
        return decode_image(base64.b64decode(payload, validate=False))
    if url.startswith(("http://", "https://")):
        import requests
        r = requests.get(url, timeout=timeout_s)
        r.raise_for_status()
        return decode_image(r.content)
    raise ValueError("image_url must be a data: or http(s) URL")


def flatten_content_parts(messages: List[dict], placeholder: str, max_images: int = 16):
    """OpenAI content-part lists -> plain string contents. Text parts are concatenated; every image
    part (``image_url`` / ``input_image``) becomes ``placeholder`` at its place and its image is
    loaded. Returns (messages, images in prompt order)."""
    out, images = [], []
    for m in messages:
        c = m.get("content")
        if not isinstance(c, list):
            out.append(m)
            continue
        text = []
        for part in c:
            kind = part.get("type")
            if kind in ("text", "input_text"):
                text.append(str(part.get("text", "")))
            elif kind in ("image_url", "input_image"):
                ref = part.get("image_url")
                url = ref.get("url") if isinstance(ref, dict) else ref
                if not isinstance(url, str):
                    raise ValueError("image part without a url")
                if len(images) >= max_images:
                    raise ValueError(f"more than {max_images} images in one request")
                images.append(load_image_url(url))
                text.append(placeholder)
            else:
                raise ValueError(f"unsupported content part type {kind!r}")
        out.append({**m, "content": "".join(text)})
    return out, images


class LlavaVision:
    def __init__(self, cfg: dict, get: Callable[[str], torch.Tensor], device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16):
        self.cfg = cfg
        self.device, self.dtype = torch.device(device), dtype
        self.vcfg = CLIPVisionConfig.from_hf(cfg["vision_config"])
        self.feature_layer = int(cfg.get("vision_feature_layer", -2))
        self.select = cfg.get("vision_feature_select_strategy", "default")
        self.image_token_index = int(cfg.get("image_token_index", cfg.get("image_token_id", 32000)))
        self.act = cfg.get("projector_hidden_act", "gelu")
        self.tower = CLIPVisionEncoder(self.vcfg, get, device, dtype)

        def t(n):
            return get(n).to(self.device, dtype).contiguous()
        self.w1, self.w2 = t("multi_modal_projector.linear_1.weight"), t("multi_modal_projector.linear_2.weight")
        try:
            self.b1, self.b2 = t("multi_modal_projector.linear_1.bias"), t("multi_modal_projector.linear_2.bias")
        except KeyError:
            self.b1 = self.b2 = None
        n = (self.vcfg.image_size // self.vcfg.patch_size) ** 2
        self.tokens_per_image = n if self.select == "default" else n + 1

    @torch.inference_mode()
    def encode(self, pixel_values: torch.Tensor) -> torch.Tensor:
        """pixel_values [B, 3, S, S] -> projected rows [B, tokens_per_image, text hidden]."""
        hs = self.tower.hidden_state(pixel_values, self.feature_layer)  # [B, 1 + n, d_vision]
        if self.select == "default":
            hs = hs[:, 1:]
        B, n, d = hs.shape
        x = hs.reshape(B * n, d).contiguous()
        y = ops.linear(x, self.w1)
        if self.b1 is not None:
            y = y + self.b1
        y = _act(y, self.act)
        y = ops.linear(y.contiguous(), self.w2)
        if self.b2 is not None:
            y = y + self.b2
        return y.view(B, n, -1)


def _llava_names(names) -> Tuple[str, str, Optional[str]]:
    """(text prefix, vision/projector prefix, lm_head name or None if tied) of a LLaVA checkpoint.

    Checkpoints name the same tensors under several prefixes (``language_model.model.*``,
    ``model.language_model.*``, ``model.language_model.model.*`` ...), so the prefixes are read off
    the anchor tensors ``embed_tokens.weight`` and ``multi_modal_projector.linear_1.weight``."""
    names = sorted(names)
    emb = [n for n in names if n.endswith("embed_tokens.weight") and "vision" not in n]
    proj = [n for n in names if n.endswith("multi_modal_projector.linear_1.weight")]
    if not emb or not proj:
        raise KeyError("not a LLaVA checkpoint: no embed_tokens / multi_modal_projector tensors")
    head = [n for n in names if n.endswith("lm_head.weight")]
    return (emb[0][:-len("embed_tokens.weight")], proj[0][:-len("multi_modal_projector.linear_1.weight")],
            head[0] if head else None)


def load_llava(directory: str, device: str = "cuda", dtype: torch.dtype = torch.bfloat16):
    """(text ModelConfig, text weight getter in Llama names, LlavaVision) of a LLaVA checkpoint."""
    from ..config import ModelConfig
    from ..loaders.safetensors import SafetensorsCheckpoint
    with open(os.path.join(directory, "config.json")) as fh:
        cfg = json.load(fh)
    ck = SafetensorsCheckpoint(directory)
    tp, vp, head = _llava_names(ck.keys())
    text = ModelConfig.from_hf(cfg["text_config"])

    def text_get(name: str) -> torch.Tensor:
        if name == "lm_head.weight":
            return ck.get(head) if head else ck.get(tp + "embed_tokens.weight")
        if name.startswith("model."):
            return ck.get(tp + name[len("model."):])
        return ck.get(name)

    vision = LlavaVision(cfg, lambda n: ck.get(vp + n), device, dtype)
    return text, text_get, vision


def expand_image_tokens(ids: List[int], image_token: int, per_image: int) -> Tuple[List[int], List[int]]:
    """Each image placeholder in ``ids`` becomes ``per_image`` copies; returns (ids, positions of the
    image rows in order)."""
    out, pos = [], []
    for t in ids:
        if t == image_token:
            pos.extend(range(len(out), len(out) + per_image))
            out.extend([image_token] * per_image)
        else:
            out.append(t)
    return out, pos
