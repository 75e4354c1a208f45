"""Offline quantization of a safetensors checkpoint with AWQ, AutoRound or QuIP.

``quantize_checkpoint(src, dst, method)`` reads a Llama-family checkpoint (standard decoder layers:
q/k/v/o projections, gated MLP, RMSNorm), quantizes every layer's seven linears and writes a
checkpoint that ``engine.load_model_source`` serves:

* ``awq``: calibration inputs of each linear from the dense fp32 model (``ReferenceDecoder`` with its
  capture hook); scales from ``awq_search`` folded upstream so the model computes the same function
  before rounding: q/k/v -> input_layernorm, gate/up -> post_attention_layernorm, down -> the rows of
  up_proj, o -> the rows of v_proj (scales tied across the query heads of a KV group). Written as
  AutoAWQ GEMM tensors (quant_method "awq").
* ``autoround``: each linear optimized on its own calibration inputs (``quantize_autoround``),
  written in AutoRound's native layout (quant_method "auto-round").
* ``quip``: data-free incoherence + E8 lattice codes (``quantize_quip``), dequantized to bf16 at load
  (quant_method "quip").

Calibration sequences are token ids: the caller's (``calib_ids``), else ids drawn uniformly over the
vocabulary with a fixed seed (no dataset is bundled).
"""
from __future__ import annotations

import json
import os
import shutil
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..config import ModelConfig
from ..models.reference import ReferenceDecoder

SITES = {"qkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), "o": ("self_attn.o_proj",),
         "gate_up": ("mlp.gate_proj", "mlp.up_proj"), "down": ("mlp.down_proj",)}


def _check_family(cfg: ModelConfig, method: str) -> None:
    unsupported = (cfg.is_moe or cfg.is_mla or bool(cfg.hybrid_schedule) or cfg.parallel_block
                   or cfg.sandwich_norm)
    if method != "quip" and unsupported:
        raise ValueError(f"{method}: calibrated quantization supports the standard Llama-family layer")
    if method == "awq" and (cfg.norm_unit_offset or cfg.norm_center or cfg.attention_bias):
        raise ValueError("awq: the scales are folded into plain RMSNorm weights and unbiased projections")


def calibration_activations(cfg: ModelConfig, weights: Dict[str, torch.Tensor], seqs: Sequence[Sequence[int]],
                            max_rows: int = 2048, seed: int = 0) -> Dict[Tuple[int, str], torch.Tensor]:
    """Inputs [n, K] of the linears of every layer (site names as in ``SITES``) over ``seqs``."""
    ref = ReferenceDecoder(cfg, weights)
    acts: Dict[Tuple[int, str], List[torch.Tensor]] = {}
    ref.capture = lambda i, site, x: acts.setdefault((i, site), []).append(x.detach().float())
    with torch.no_grad():
        for ids in seqs:
            ref.forward(torch.tensor(list(ids)))
    g = torch.Generator().manual_seed(seed)
    out = {}
    for key, xs in acts.items():
        X = torch.cat(xs)
        if X.shape[0] > max_rows:
            X = X[torch.randperm(X.shape[0], generator=g)[:max_rows]]
        out[key] = X
    return out


def quantize_checkpoint(src: str, dst: str, method: str, group: int = 128, calib_ids: Optional[Sequence] = None,
                        calib_seqs: int = 4, calib_len: int = 256, iters: int = 200, stages: int = 1,
                        seed: int = 0) -> dict:
    """Quantize ``src`` (checkpoint directory with config.json) into ``dst``; returns a summary."""
    from ..loaders.safetensors import SafetensorsCheckpoint, save_file
    from .autoround import quantize_autoround, to_autoround
    from .awq import awq_search, to_awq
    from .int4 import quantize_rtn
    from .quip import quantize_quip
    if method not in ("awq", "autoround", "quip", "nvfp4", "mxfp4"):
        raise ValueError(f"unknown method {method!r}")
    with open(os.path.join(src, "config.json")) as f:
        hf = json.load(f)
    if hf.get("quantization_config"):
        raise ValueError(f"{src} is already quantized")
    cfg = ModelConfig.from_hf(hf)
    _check_family(cfg, method)
    ck = SafetensorsCheckpoint(src)
    w = {k: ck.get(k) for k in ck.keys()}
    acts = {}
    if method in ("awq", "autoround"):
        if calib_ids is None:
            g = torch.Generator().manual_seed(seed)
            calib_ids = [torch.randint(0, cfg.vocab_size, (calib_len,), generator=g).tolist() for _ in range(calib_seqs)]
        acts = calibration_activations(cfg, {k: v.float() for k, v in w.items()}, calib_ids, seed=seed)
    out: Dict[str, torch.Tensor] = {}
    n_q = 0
    H, Hk, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        lin = {n: w[p + n + ".weight"].float() for site in SITES.values() for n in site}
        if method == "awq":
            norms = {"in": w[p + "input_layernorm.weight"].float(), "post": w[p + "post_attention_layernorm.weight"].float()}
            # down first: its input scales are folded into up_proj's rows before gate/up is quantized
            s, (qd,) = awq_search([lin["mlp.down_proj"]], acts[(i, "down")], group)
            lin["mlp.up_proj"] = lin["mlp.up_proj"] / s[:, None]
            qs = {"mlp.down_proj": qd}
            # o: its input channels come from v_proj's rows (tied over the query heads of a KV group)
            s, (qo,) = awq_search([lin["self_attn.o_proj"]], acts[(i, "o")], group, tie=(H // Hk, D))
            sv = s.view(Hk, H // Hk, D)[:, 0, :].reshape(-1)
            lin["self_attn.v_proj"] = lin["self_attn.v_proj"] / sv[:, None]
            qs["self_attn.o_proj"] = qo
            for site, norm in (("qkv", "in"), ("gate_up", "post")):
                names = SITES[site]
                s, qq = awq_search([lin[n] for n in names], acts[(i, site)], group)
                norms[norm] = norms[norm] / s
                qs.update(dict(zip(names, qq)))
            out[p + "input_layernorm.weight"] = norms["in"].to(torch.bfloat16)
            out[p + "post_attention_layernorm.weight"] = norms["post"].to(torch.bfloat16)
            for n, q in qs.items():
                for k, t in to_awq(q).items():
                    out[p + n + "." + k] = t
                n_q += 1
        elif method == "autoround":
            for site, names in SITES.items():
                for n in names:
                    q = quantize_autoround(lin[n], acts[(i, site)], group, iters=iters, seed=seed)
                    t = to_autoround(q)
                    out[p + n + ".weight"] = t["weight"]
                    out[p + n + ".scale"] = t["scale"]
                    out[p + n + ".zp"] = t["zp"]
                    n_q += 1
        elif method in ("nvfp4", "mxfp4"):
            from .fp4 import quantize_mxfp4, quantize_nvfp4, to_tensors as fp4_tensors
            for n, W in lin.items():
                q = quantize_nvfp4(W) if method == "nvfp4" else quantize_mxfp4(W)
                for suf, t in fp4_tensors(q).items():
                    out[p + n + ".weight" + suf] = t
                n_q += 1
        else:
            for n, W in lin.items():
                q = quantize_quip(W, stages=stages, seed=seed)
                for st, c in enumerate(q.codes):
                    out[f"{p}{n}.quip_codes{st}"] = c.contiguous()
                out[p + n + ".quip_scales"] = q.scales.contiguous()
                n_q += 1
    for k, v in w.items():  # everything else unchanged
        if k not in out and not any(k == f"model.layers.{i}.{n}.weight" for i in range(cfg.num_hidden_layers)
                                    for site in SITES.values() for n in site):
            out[k] = v
    os.makedirs(dst, exist_ok=True)
    save_file(out, os.path.join(dst, "model.safetensors"), {"quantization": method})
    if method == "awq":
        qc = {"quant_method": "awq", "bits": 4, "group_size": group, "zero_point": True, "version": "gemm"}
    elif method == "autoround":
        qc = {"quant_method": "auto-round", "bits": 4, "group_size": group, "sym": False, "iters": iters,
              "packing_format": "auto_round"}
    elif method == "nvfp4":
        qc = {"quant_method": "modelopt", "quant_algo": "NVFP4", "group_size": 16}
    elif method == "mxfp4":
        qc = {"quant_method": "mxfp4", "group_size": 32}
    else:
        qc = {"quant_method": "quip", "stages": stages, "seed": seed, "codebook": "e8-ball10", "group_size": 64}
    hf["quantization_config"] = qc
    with open(os.path.join(dst, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)
    for extra in ("tokenizer.json", "tokenizer_config.json", "generation_config.json", "special_tokens_map.json"):
        if os.path.exists(os.path.join(src, extra)):
            shutil.copy(os.path.join(src, extra), dst)
    return {"method": method, "linears": n_q, "tensors": len(out), "dst": dst}
