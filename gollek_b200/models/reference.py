"""Plain-PyTorch fp32 reference decoder (the correctness oracle).

Dense (non-paged) forward of the Llama / Mixtral family in Hugging Face
semantics: pre-norm RMSNorm, GQA attention with NeoX ("rotate-half") RoPE whose
theta comes from the config, SwiGLU FFN or top-k softmax MoE, final RMSNorm and
an untied lm_head. It restates what the reference's Direct engine computes
(runner/safetensor/gollek-safetensor-engine/…/engine/forward/DirectForwardPass.java:40-321,
MoE routing …/generation/moe/MoeForwardPass.java:107-128) without its
hard-coded RoPE theta, and is cross-checked against ``transformers`` in tests.

Weights use Hugging Face tensor names (``model.layers.{i}.self_attn.q_proj.weight``…).
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from ..config import ModelConfig

Weights = Dict[str, torch.Tensor]


def init_random_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02,
                        dtype: torch.dtype = torch.float32, device: str = "cpu") -> Weights:
    """Random-init weights of the architecture: every matrix ~ N(0, std), norm weights = 1.

    Tensors are generated in a fixed order from one generator seeded with ``seed`` so a
    checkpoint written from them is reproducible.
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h, q, kv, f = cfg.hidden_size, cfg.q_size, cfg.kv_size, cfg.intermediate_size

    def rnd(*shape):
        t = torch.empty(*shape, dtype=torch.float32 if dtype == torch.float32 else dtype, device=device)
        t.normal_(0.0, std, generator=g)
        return t

    w: Weights = {"model.embed_tokens.weight": rnd(cfg.vocab_size, h)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = torch.ones(h, dtype=dtype, device=device)
        w[p + "self_attn.q_proj.weight"] = rnd(q, h)
        w[p + "self_attn.k_proj.weight"] = rnd(kv, h)
        w[p + "self_attn.v_proj.weight"] = rnd(kv, h)
        w[p + "self_attn.o_proj.weight"] = rnd(h, q)
        w[p + "post_attention_layernorm.weight"] = torch.ones(h, dtype=dtype, device=device)
        if cfg.is_moe:
            w[p + "block_sparse_moe.gate.weight"] = rnd(cfg.num_local_experts, h)
            for e in range(cfg.num_local_experts):
                pe = p + f"block_sparse_moe.experts.{e}."
                w[pe + "w1.weight"] = rnd(f, h)
                w[pe + "w3.weight"] = rnd(f, h)
                w[pe + "w2.weight"] = rnd(h, f)
        else:
            w[p + "mlp.gate_proj.weight"] = rnd(f, h)
            w[p + "mlp.up_proj.weight"] = rnd(f, h)
            w[p + "mlp.down_proj.weight"] = rnd(h, f)
    w["model.norm.weight"] = torch.ones(h, dtype=dtype, device=device)
    if not cfg.tie_word_embeddings:
        w["lm_head.weight"] = rnd(cfg.vocab_size, h)
    return w


def rope_inv_freq(cfg: ModelConfig) -> torch.Tensor:
    """Per-pair inverse frequencies, including ``linear`` and ``llama3`` scaling."""
    d = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    rs = cfg.rope_scaling
    if rs.kind == "linear":
        inv = inv / rs.factor
    elif rs.kind == "llama3":
        low_wl = rs.original_max_position_embeddings / rs.low_freq_factor
        high_wl = rs.original_max_position_embeddings / rs.high_freq_factor
        wl = 2 * math.pi / inv
        smooth = (rs.original_max_position_embeddings / wl - rs.low_freq_factor) / (
            rs.high_freq_factor - rs.low_freq_factor)
        scaled = torch.where(wl > low_wl, inv / rs.factor, inv)
        mid = (wl <= low_wl) & (wl >= high_wl)
        scaled = torch.where(mid, (1 - smooth) * inv / rs.factor + smooth * inv, scaled)
        inv = scaled
    return inv.to(torch.float32)


def rope_cos_sin(cfg: ModelConfig, max_pos: int, device="cpu") -> torch.Tensor:
    """``[max_pos, head_dim]`` table: first half cos, second half sin (fp32)."""
    inv = rope_inv_freq(cfg).to(device)
    t = torch.arange(max_pos, dtype=torch.float32, device=device)
    freqs = torch.outer(t, inv)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1)


def apply_rope_neox(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """x: [T, H, D]; rotate-half RoPE at ``positions`` (fp32 math)."""
    d = x.shape[-1]
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, : d // 2].float(), cs[:, None, d // 2:].float()
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def moe_ref(x: torch.Tensor, gate_w: torch.Tensor, experts: list, top_k: int) -> torch.Tensor:
    """Mixtral MoE: softmax over all experts → top-k → renormalise → weighted SwiGLU experts."""
    logits = x.float() @ gate_w.float().t()
    probs = torch.softmax(logits, dim=-1)
    topw, topi = probs.topk(top_k, dim=-1)
    topw = topw / topw.sum(-1, keepdim=True)
    out = torch.zeros_like(x, dtype=torch.float32)
    for e, (w1, w3, w2) in enumerate(experts):
        mask = (topi == e)
        rows = mask.any(-1).nonzero().flatten()
        if rows.numel() == 0:
            continue
        wt = (topw * mask).sum(-1)[rows]
        xe = x[rows].float()
        ye = (torch.nn.functional.silu(xe @ w1.float().t()) * (xe @ w3.float().t())) @ w2.float().t()
        out[rows] += wt[:, None] * ye
    return out.to(x.dtype)


class ReferenceDecoder:
    """Dense fp32 forward over a whole token sequence (no KV cache): the oracle."""

    def __init__(self, cfg: ModelConfig, weights: Weights):
        self.cfg = cfg
        self.w = {k: v.float() for k, v in weights.items()}
        self.cos_sin = rope_cos_sin(cfg, max(cfg.max_position_embeddings, 4096))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """ids: [S] → logits [S, vocab] (fp32)."""
        cfg, w = self.cfg, self.w
        S = ids.shape[0]
        pos = torch.arange(S)
        h = w["model.embed_tokens.weight"][ids.long()]
        H, Hk, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        mask = torch.full((S, S), float("-inf")).triu(1)
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}."
            x = rms_norm_ref(h, w[p + "input_layernorm.weight"], cfg.rms_norm_eps)
            q = (x @ w[p + "self_attn.q_proj.weight"].t()).view(S, H, D)
            k = (x @ w[p + "self_attn.k_proj.weight"].t()).view(S, Hk, D)
            v = (x @ w[p + "self_attn.v_proj.weight"].t()).view(S, Hk, D)
            q = apply_rope_neox(q, self.cos_sin, pos)
            k = apply_rope_neox(k, self.cos_sin, pos)
            rep = H // Hk
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
            s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(D) + mask
            a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(S, H * D)
            h = h + a @ w[p + "self_attn.o_proj.weight"].t()
            x = rms_norm_ref(h, w[p + "post_attention_layernorm.weight"], cfg.rms_norm_eps)
            if cfg.is_moe:
                pe = p + "block_sparse_moe."
                experts = [(w[pe + f"experts.{e}.w1.weight"], w[pe + f"experts.{e}.w3.weight"],
                            w[pe + f"experts.{e}.w2.weight"]) for e in range(cfg.num_local_experts)]
                h = h + moe_ref(x, w[pe + "gate.weight"], experts, cfg.num_experts_per_tok)
            else:
                g = x @ w[p + "mlp.gate_proj.weight"].t()
                u = x @ w[p + "mlp.up_proj.weight"].t()
                h = h + (torch.nn.functional.silu(g) * u) @ w[p + "mlp.down_proj.weight"].t()
        h = rms_norm_ref(h, w["model.norm.weight"], cfg.rms_norm_eps)
        head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
        return h @ head.t()

    def greedy(self, prompt: list, n_new: int) -> tuple:
        """Greedy decode by re-running the dense forward; returns (tokens, per-step logits)."""
        ids = list(prompt)
        all_logits = []
        for _ in range(n_new):
            logits = self.forward(torch.tensor(ids))[-1]
            all_logits.append(logits)
            ids.append(int(logits.argmax()))
        return ids[len(prompt):], torch.stack(all_logits)
