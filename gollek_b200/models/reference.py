"""Plain-PyTorch fp32 reference decoder (the correctness oracle).

Dense (non-paged) forward of the supported families (Llama, Mistral, Mixtral, Qwen2/3, Gemma 1/2/3,
Phi-3) in Hugging Face semantics: pre-norm RMSNorm ((1 + w) for Gemma), GQA attention with NeoX
("rotate-half") RoPE whose theta comes from the config (per layer type for Gemma-3), optional
projection biases, QK-norm, sliding windows and logit softcapping, SwiGLU/GeGLU FFN or top-k softmax
MoE, sandwich norms (Gemma-2/3), final RMSNorm and a tied or untied lm_head. It restates what the reference's Direct engine computes
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
    """Random-init weights of the architecture under its Hugging Face names: every matrix and
    bias ~ N(0, std); norm weights 1 (or ~N(0, 0.05) for the (1 + w) norms of Gemma).

    Tensors are generated in a fixed order from one generator seeded with ``seed`` so a
    checkpoint written from them is reproducible.
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h, q, kv, f, D = cfg.hidden_size, cfg.q_size, cfg.kv_size, cfg.intermediate_size, cfg.head_dim
    fam = cfg.architecture

    def rnd(*shape, s=std):
        t = torch.empty(*shape, dtype=torch.float32 if dtype == torch.float32 else dtype, device=device)
        t.normal_(0.0, s, generator=g)
        return t

    def norm(n):
        if cfg.norm_unit_offset:
            return rnd(n, s=0.05).to(dtype)
        return torch.ones(n, dtype=dtype, device=device)

    w: Weights = {"model.embed_tokens.weight": rnd(cfg.vocab_size, h)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = norm(h)
        if cfg.is_gdn_layer(i):  # gated delta rule layer of a hybrid stack
            hd = cfg.gdn_heads * cfg.gdn_head_dim
            pl = p + "linear_attn."
            for n in ("q", "k", "v", "g"):
                w[pl + f"{n}_proj.weight"] = rnd(hd, h)
            w[pl + "a_proj.weight"] = rnd(cfg.gdn_heads, h)
            w[pl + "b_proj.weight"] = rnd(cfg.gdn_heads, h)
            w[pl + "A_log"] = torch.log(1.0 + 15.0 * torch.rand(cfg.gdn_heads, generator=g, device=device)).to(
                torch.float32)
            w[pl + "dt_bias"] = rnd(cfg.gdn_heads, s=0.5).to(torch.float32)
            w[pl + "norm.weight"] = torch.ones(cfg.gdn_head_dim, dtype=dtype, device=device)
            w[pl + "o_proj.weight"] = rnd(h, hd)
        elif cfg.is_mla:
            nh, qk = cfg.num_attention_heads, cfg.head_dim
            pa = p + "self_attn."
            if cfg.q_lora_rank:
                w[pa + "q_a_proj.weight"] = rnd(cfg.q_lora_rank, h)
                w[pa + "q_a_layernorm.weight"] = torch.ones(cfg.q_lora_rank, dtype=dtype, device=device)
                w[pa + "q_b_proj.weight"] = rnd(nh * qk, cfg.q_lora_rank, s=0.1)
            else:
                w[pa + "q_proj.weight"] = rnd(nh * qk, h)
            w[pa + "kv_a_proj_with_mqa.weight"] = rnd(cfg.kv_lora_rank + cfg.qk_rope_head_dim, h)
            w[pa + "kv_a_layernorm.weight"] = torch.ones(cfg.kv_lora_rank, dtype=dtype, device=device)
            w[pa + "kv_b_proj.weight"] = rnd(nh * (cfg.qk_nope_head_dim + cfg.v_head_dim), cfg.kv_lora_rank, s=0.1)
            w[pa + "o_proj.weight"] = rnd(h, nh * cfg.v_head_dim)
        elif fam == "phi3":
            w[p + "self_attn.qkv_proj.weight"] = rnd(q + 2 * kv, h)
        else:
            w[p + "self_attn.q_proj.weight"] = rnd(q, h)
            w[p + "self_attn.k_proj.weight"] = rnd(kv, h)
            w[p + "self_attn.v_proj.weight"] = rnd(kv, h)
        if cfg.attention_bias and not cfg.is_gdn_layer(i):
            w[p + "self_attn.q_proj.bias"] = rnd(q)
            w[p + "self_attn.k_proj.bias"] = rnd(kv)
            w[p + "self_attn.v_proj.bias"] = rnd(kv)
        if cfg.qk_norm and not cfg.is_gdn_layer(i):
            w[p + "self_attn.q_norm.weight"] = norm(D)
            w[p + "self_attn.k_norm.weight"] = norm(D)
        if not cfg.is_gdn_layer(i) and not cfg.is_mla:
            w[p + "self_attn.o_proj.weight"] = rnd(h, q)
        if not cfg.parallel_block:
            w[p + "post_attention_layernorm.weight"] = norm(h)
        if cfg.sandwich_norm:
            w[p + "pre_feedforward_layernorm.weight"] = norm(h)
            w[p + "post_feedforward_layernorm.weight"] = norm(h)
        if cfg.is_moe_layer(i) and cfg.moe_scoring == "sigmoid":  # DeepSeek-V3 MoE
            pm, fe = p + "mlp.", cfg.moe_ffn
            w[pm + "gate.weight"] = rnd(cfg.num_local_experts, h, s=0.1)
            w[pm + "gate.e_score_correction_bias"] = rnd(cfg.num_local_experts, s=0.05).float()
            for e in range(cfg.num_local_experts):
                pe = pm + f"experts.{e}."
                w[pe + "gate_proj.weight"] = rnd(fe, h)
                w[pe + "up_proj.weight"] = rnd(fe, h)
                w[pe + "down_proj.weight"] = rnd(h, fe)
            if cfg.n_shared_experts:
                fs = fe * cfg.n_shared_experts
                w[pm + "shared_experts.gate_proj.weight"] = rnd(fs, h)
                w[pm + "shared_experts.up_proj.weight"] = rnd(fs, h)
                w[pm + "shared_experts.down_proj.weight"] = rnd(h, fs)
        elif cfg.is_moe_layer(i):
            w[p + "block_sparse_moe.gate.weight"] = rnd(cfg.num_local_experts, h)
            for e in range(cfg.num_local_experts):
                pe = p + f"block_sparse_moe.experts.{e}."
                w[pe + "w1.weight"] = rnd(f, h)
                w[pe + "w3.weight"] = rnd(f, h)
                w[pe + "w2.weight"] = rnd(h, f)
        elif fam == "phi3":
            w[p + "mlp.gate_up_proj.weight"] = rnd(2 * f, h)
            w[p + "mlp.down_proj.weight"] = rnd(h, f)
        else:
            w[p + "mlp.gate_proj.weight"] = rnd(f, h)
            w[p + "mlp.up_proj.weight"] = rnd(f, h)
            w[p + "mlp.down_proj.weight"] = rnd(h, f)
    w["model.norm.weight"] = norm(h)
    if not cfg.tie_word_embeddings:
        w["lm_head.weight"] = rnd(cfg.vocab_size, h)
    return w


def layer_tensors(get, cfg: ModelConfig, i: int, moe: bool = False) -> dict:
    """Layer ``i``'s tensors under canonical keys, whatever the family's checkpoint layout:
    q, k, v, o, (q_bias, k_bias, v_bias), (q_norm, k_norm), in_norm, post_norm, (pre_ff_norm,
    post_ff_norm), gate, up, down; MLA: q_a, q_a_norm, q_b (or q), kv_a, kv_a_norm, kv_b; MoE layers:
    with ``moe``, router, (router_bias), experts [(gate, up, down)], (shared (gate, up, down)) (the
    serving model reads only its own experts by name instead). ``get(name)`` returns a tensor (or a quantized weight that
    supports row slicing). Phi-3's fused ``qkv_proj`` / ``gate_up_proj`` are split by rows."""
    p = f"model.layers.{i}."
    q_sz, kv_sz, f = cfg.q_size, cfg.kv_size, cfg.intermediate_size
    if cfg.is_gdn_layer(i):
        pl = p + "linear_attn."
        t = {"in_norm": get(p + "input_layernorm.weight"), "post_norm": get(p + "post_attention_layernorm.weight"),
             "gdn": True, "o": get(pl + "o_proj.weight"), "A_log": get(pl + "A_log"), "dt_bias": get(pl + "dt_bias"),
             "gnorm": get(pl + "norm.weight")}
        for n in ("q", "k", "v", "g", "a", "b"):
            t["g" + n] = get(pl + f"{n}_proj.weight")
    else:
        t = {"in_norm": get(p + "input_layernorm.weight"), "o": get(p + "self_attn.o_proj.weight"),
             "post_norm": None if cfg.parallel_block else get(p + "post_attention_layernorm.weight")}
    if cfg.is_gdn_layer(i):
        pass
    elif cfg.is_mla:
        pa = p + "self_attn."
        if cfg.q_lora_rank:
            t["q_a"], t["q_a_norm"] = get(pa + "q_a_proj.weight"), get(pa + "q_a_layernorm.weight")
            t["q_b"] = get(pa + "q_b_proj.weight")
        else:
            t["q"] = get(pa + "q_proj.weight")
        t["kv_a"], t["kv_a_norm"] = get(pa + "kv_a_proj_with_mqa.weight"), get(pa + "kv_a_layernorm.weight")
        t["kv_b"] = get(pa + "kv_b_proj.weight")
    elif cfg.architecture == "phi3":
        qkv = get(p + "self_attn.qkv_proj.weight")
        t["q"], t["k"], t["v"] = qkv[:q_sz], qkv[q_sz:q_sz + kv_sz], qkv[q_sz + kv_sz:q_sz + 2 * kv_sz]
    else:
        t["q"] = get(p + "self_attn.q_proj.weight")
        t["k"] = get(p + "self_attn.k_proj.weight")
        t["v"] = get(p + "self_attn.v_proj.weight")
    if cfg.attention_bias and not cfg.is_gdn_layer(i):
        for n in ("q", "k", "v"):
            t[n + "_bias"] = get(p + f"self_attn.{n}_proj.bias")
    if cfg.qk_norm and not cfg.is_gdn_layer(i):
        t["q_norm"] = get(p + "self_attn.q_norm.weight")
        t["k_norm"] = get(p + "self_attn.k_norm.weight")
    if cfg.sandwich_norm:
        t["pre_ff_norm"] = get(p + "pre_feedforward_layernorm.weight")
        t["post_ff_norm"] = get(p + "post_feedforward_layernorm.weight")
    if cfg.is_moe_layer(i) and not moe:
        pass
    elif cfg.is_moe_layer(i) and cfg.moe_scoring == "sigmoid":
        pm = p + "mlp."
        t["router"], t["router_bias"] = get(pm + "gate.weight"), get(pm + "gate.e_score_correction_bias")
        t["experts"] = [tuple(get(pm + f"experts.{e}.{n}_proj.weight") for n in ("gate", "up", "down"))
                        for e in range(cfg.num_local_experts)]
        if cfg.n_shared_experts:
            t["shared"] = tuple(get(pm + f"shared_experts.{n}_proj.weight") for n in ("gate", "up", "down"))
    elif cfg.is_moe_layer(i):
        pm = p + "block_sparse_moe."
        t["router"] = get(pm + "gate.weight")
        t["experts"] = [tuple(get(pm + f"experts.{e}.{n}.weight") for n in ("w1", "w3", "w2"))
                        for e in range(cfg.num_local_experts)]
    else:
        if cfg.architecture == "phi3":
            gu = get(p + "mlp.gate_up_proj.weight")
            t["gate"], t["up"] = gu[:f], gu[f:2 * f]
        else:
            t["gate"] = get(p + "mlp.gate_proj.weight")
            t["up"] = get(p + "mlp.up_proj.weight")
        t["down"] = get(p + "mlp.down_proj.weight")
    return t


def rope_inv_freq(cfg: ModelConfig, theta: Optional[float] = None, long: bool = False) -> torch.Tensor:
    """Per-pair inverse frequencies, including ``linear``, ``llama3``, ``longrope`` and ``yarn``
    scaling (YaRN, arXiv 2309.00071: pairs that turn more than ``beta_fast`` times over the original
    context keep their frequency, pairs that turn fewer than ``beta_slow`` times are divided by
    ``factor``, with a linear ramp between)."""
    d = cfg.rope_dim
    theta = theta or cfg.rope_theta
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    rs = cfg.rope_scaling
    if rs.kind == "yarn":
        inv = inv.float().double()  # the published tables are computed in fp32
        orig = rs.original_max_position_embeddings

        def dim_of(rotations):  # pair index whose wavelength fits ``rotations`` times in ``orig``
            return d * math.log(orig / (rotations * 2 * math.pi)) / (2 * math.log(theta))

        lo = max(math.floor(dim_of(rs.beta_fast)), 0)
        hi = min(math.ceil(dim_of(rs.beta_slow)), d - 1)
        if lo == hi:
            hi += 0.001
        ramp = ((torch.arange(d // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
        keep = 1 - ramp  # 1: extrapolate (original frequency), 0: interpolate (divided by factor)
        inv = inv / rs.factor * (1 - keep) + inv * keep
    elif rs.kind == "linear":
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
    elif rs.kind == "longrope":
        fac = rs.long_factor if long else rs.short_factor
        if fac is not None:
            inv = inv / torch.tensor(fac, dtype=torch.float64)
    return inv.to(torch.float32)


def rope_cos_sin(cfg: ModelConfig, max_pos: int, device="cpu", theta: Optional[float] = None) -> torch.Tensor:
    """``[max_pos, head_dim]`` table: first half cos, second half sin (fp32). ``longrope`` uses the
    short factors below the original context length and the long ones from there on, with the
    attention scaling sqrt(1 + ln(s) / ln(original)) for s = max_position / original."""
    t = torch.arange(max_pos, dtype=torch.float32, device=device)
    rs = cfg.rope_scaling
    if rs.kind == "longrope":
        orig = rs.original_max_position_embeddings
        fs = torch.outer(t, rope_inv_freq(cfg, theta, long=False).to(device))
        fl = torch.outer(t, rope_inv_freq(cfg, theta, long=True).to(device))
        freqs = torch.where((t >= orig)[:, None], fl, fs)
        s = cfg.max_position_embeddings / orig
        mscale = math.sqrt(1 + math.log(s) / math.log(orig)) if s > 1 else 1.0
        return torch.cat([freqs.cos() * mscale, freqs.sin() * mscale], dim=-1)
    freqs = torch.outer(t, rope_inv_freq(cfg, theta).to(device))
    if rs.kind == "yarn":
        from ..config import yarn_mscale
        att = yarn_mscale(rs.factor, rs.mscale) / yarn_mscale(rs.factor, rs.mscale_all_dim) \
            if (rs.mscale and rs.mscale_all_dim) else yarn_mscale(rs.factor)
        return torch.cat([freqs.cos() * att, freqs.sin() * att], dim=-1)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1)


def apply_rope_neox(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """x: [T, H, D]; rotate-half RoPE at ``positions`` (fp32 math)."""
    d = x.shape[-1]
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, : d // 2].float(), cs[:, None, d // 2:].float()
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def apply_rope_interleaved(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """x: [T, H, D]; RoPE on interleaved pairs (2i, 2i+1) with frequency i (Cohere), fp32 math."""
    d = x.shape[-1]
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, : d // 2].float(), cs[:, None, d // 2:].float()
    xf = x.float()
    x1, x2 = xf[..., 0::2], xf[..., 1::2]
    return torch.stack([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).flatten(-2).to(x.dtype)


def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float, unit_offset: bool = False,
                 center: bool = False) -> torch.Tensor:
    xf = x.float()
    if center:  # bias-free LayerNorm (Cohere)
        xf = xf - xf.mean(-1, keepdim=True)
    wf = w.float() + 1.0 if unit_offset else w.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * wf).to(x.dtype)


def moe_ref(x: torch.Tensor, gate_w: torch.Tensor, experts: list, top_k: int, **route) -> torch.Tensor:
    """MoE FFN: router top-k (Mixtral softmax by default; ``route`` selects DeepSeek-V3's sigmoid
    group-limited routing, see ``ops.reference.moe_route``) → weighted SwiGLU experts."""
    from ..ops.reference import moe_route
    topi, topw = moe_route(x.float() @ gate_w.float().t(), top_k, **route)
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


def route_options(cfg: ModelConfig, bias: Optional[torch.Tensor] = None) -> dict:
    """Keyword options of ``ops.reference.moe_route`` for the family's router."""
    if cfg.moe_scoring == "softmax":
        return {}
    return dict(renorm=cfg.norm_topk_prob, scoring=cfg.moe_scoring, bias=bias, n_group=cfg.n_group,
                topk_group=cfg.topk_group, scale=cfg.routed_scaling_factor)


class ReferenceDecoder:
    """Dense fp32 forward over a whole token sequence (no KV cache): the oracle."""

    def __init__(self, cfg: ModelConfig, weights: Weights):
        self.cfg = cfg
        self.w = {k: v.float() for k, v in weights.items()}
        # capture(layer, site, x): called with the input rows of the dense linears of the standard
        # decoder layer, site in {"qkv", "o", "gate_up", "down"} (offline quantizer calibration)
        self.capture = None
        n = max(cfg.max_position_embeddings, 4096)
        self.cos_sin = rope_cos_sin(cfg, n)
        self.cos_sin_local = rope_cos_sin(cfg, n, theta=cfg.rope_local_theta) if cfg.rope_local_theta else None

    def forward(self, ids: torch.Tensor, key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """ids: [S] → logits [S, vocab] (fp32). ``key_mask`` [S, S] bool (optional): False hides key
        k from query q on top of the causal mask (evicted KV)."""
        cfg, w = self.cfg, self.w
        S = ids.shape[0]
        pos = torch.arange(S)
        h = w["model.embed_tokens.weight"][ids.long()] * cfg.embed_scale
        H, Hk, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        uo, eps, ctr = cfg.norm_unit_offset, cfg.rms_norm_eps, cfg.norm_center
        causal = torch.full((S, S), float("-inf")).triu(1)
        for i in range(cfg.num_hidden_layers):
            L = layer_tensors(w.__getitem__, cfg, i)
            x = rms_norm_ref(h, L["in_norm"], eps, uo, ctr)
            if L.get("gdn"):
                a = self._gdn(x, L)
                h = h + a
                x = rms_norm_ref(h, L["post_norm"], eps, uo)
                h = h + self._ffn(x, L, i)
                continue
            win = cfg.layer_window(i)
            mask = causal
            if key_mask is not None:
                mask = mask.masked_fill(~key_mask, float("-inf"))
            if win > 0:
                mask = mask + torch.full((S, S), float("-inf")).tril(-win)
            if cfg.is_mla:
                a = self._mla(x, L, pos, mask)
                h = h + a
                x = rms_norm_ref(h, L["post_norm"], eps, uo)
                h = h + self._ffn(x, L, i)
                continue
            if self.capture is not None:
                self.capture(i, "qkv", x)
            q = x @ L["q"].t()
            k = x @ L["k"].t()
            v = x @ L["v"].t()
            if cfg.attention_bias:
                q, k, v = q + L["q_bias"], k + L["k_bias"], v + L["v_bias"]
            q, k, v = q.view(S, H, D), k.view(S, Hk, D), v.view(S, Hk, D)
            if cfg.qk_norm:
                q = rms_norm_ref(q, L["q_norm"], eps, uo)
                k = rms_norm_ref(k, L["k_norm"], eps, uo)
            cs = self.cos_sin_local if (self.cos_sin_local is not None and win > 0) else self.cos_sin
            if not (cfg.rope_sliding_only and win == 0):
                rope = apply_rope_interleaved if cfg.rope_interleaved else apply_rope_neox
                q = rope(q, cs, pos)
                k = rope(k, cs, pos)
            rep = H // Hk
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
            s = torch.einsum("qhd,khd->hqk", q, k) * cfg.attn_scale
            if cfg.attn_logit_softcapping:
                c = cfg.attn_logit_softcapping
                s = c * torch.tanh(s / c)
            a = torch.einsum("hqk,khd->qhd", torch.softmax(s + mask, -1), v).reshape(S, H * D)
            if self.capture is not None:
                self.capture(i, "o", a)
            a = a @ L["o"].t()
            if cfg.parallel_block:  # attention and MLP both read x (one norm per layer)
                h = h + a + self._ffn(x, L, i)
                continue
            if cfg.sandwich_norm:
                h = h + rms_norm_ref(a, L["post_norm"], eps, uo)
                x = rms_norm_ref(h, L["pre_ff_norm"], eps, uo)
            else:
                h = h + a
                x = rms_norm_ref(h, L["post_norm"], eps, uo)
            m = self._ffn(x, L, i)
            if cfg.sandwich_norm:
                m = rms_norm_ref(m, L["post_ff_norm"], eps, uo)
            h = h + m
        h = rms_norm_ref(h, w["model.norm.weight"], eps, uo, ctr)
        head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
        logits = h @ head.t()
        if cfg.logit_scale != 1.0:
            logits = logits * cfg.logit_scale
        if cfg.final_logit_softcapping:
            c = cfg.final_logit_softcapping
            logits = c * torch.tanh(logits / c)
        return logits

    def _mla(self, x: torch.Tensor, L: dict, pos: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        """Multi-head latent attention (DeepSeek-V3), decompressed: per-head keys [k_nope | k_rope]
        with one k_rope shared by all heads, values from the normalised latent. With
        ``rope_interleaved`` the rope dims are pairs (2i, 2i+1), rotated and returned as
        [evens | odds] (the layout the checkpoint's attention uses)."""
        cfg = self.cfg
        S, H, eps = x.shape[0], cfg.num_attention_heads, cfg.rms_norm_eps
        nope, rd, vd = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
        if cfg.q_lora_rank:
            q = rms_norm_ref(x @ L["q_a"].t(), L["q_a_norm"], eps) @ L["q_b"].t()
        else:
            q = x @ L["q"].t()
        q = q.view(S, H, nope + rd)
        ckv = x @ L["kv_a"].t()
        kv = (rms_norm_ref(ckv[:, :cfg.kv_lora_rank], L["kv_a_norm"], eps) @ L["kv_b"].t()).view(S, H, nope + vd)
        q_rot, k_rot = q[..., nope:], ckv[:, None, cfg.kv_lora_rank:]
        if cfg.rope_interleaved:
            q_rot = torch.cat([q_rot[..., 0::2], q_rot[..., 1::2]], -1)
            k_rot = torch.cat([k_rot[..., 0::2], k_rot[..., 1::2]], -1)
        q_rot = apply_rope_neox(q_rot, self.cos_sin, pos)
        k_rot = apply_rope_neox(k_rot, self.cos_sin, pos)
        q = torch.cat([q[..., :nope], q_rot], -1)
        k = torch.cat([kv[..., :nope], k_rot.expand(S, H, rd)], -1)
        s = torch.einsum("qhd,khd->hqk", q, k) * cfg.attn_scale
        a = torch.einsum("hqk,khd->qhd", torch.softmax(s + mask, -1), kv[..., nope:]).reshape(S, H * vd)
        return a @ L["o"].t()

    def _ffn(self, x: torch.Tensor, L: dict, i: int) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        if cfg.is_moe_layer(i):
            M = layer_tensors(w.__getitem__, cfg, i, moe=True)
            out = moe_ref(x, M["router"], M["experts"], cfg.num_experts_per_tok,
                          **route_options(cfg, M.get("router_bias")))
            if "shared" in M:
                g, u, d = M["shared"]
                out = out + (torch.nn.functional.silu(x @ g.t()) * (x @ u.t())) @ d.t()
            return out
        if self.capture is not None:
            self.capture(i, "gate_up", x)
        g = x @ L["gate"].t()
        act = torch.nn.functional.silu(g) if cfg.hidden_act == "silu" else \
            torch.nn.functional.gelu(g, approximate="tanh")
        hmid = act * (x @ L["up"].t())
        if self.capture is not None:
            self.capture(i, "down", hmid)
        return hmid @ L["down"].t()

    def _gdn(self, x: torch.Tensor, L: dict) -> torch.Tensor:
        """Gated delta rule layer over the whole sequence (fresh state)."""
        from ..ops import reference as ref_ops
        cfg = self.cfg
        Hg, D = cfg.gdn_heads, cfg.gdn_head_dim
        S = x.shape[0]
        proj = torch.cat([x @ L["g" + n].t() for n in ("q", "k", "v", "g", "a", "b")], dim=-1)
        state = torch.zeros(1, Hg, D, D)
        o = ref_ops.gdn_scan(proj, state, torch.zeros(1, dtype=torch.int32), torch.ones(1, dtype=torch.int32),
                             torch.tensor([0, S], dtype=torch.int32), L["A_log"], L["dt_bias"], Hg)
        y = ref_ops.gdn_gated_norm(o, proj[:, 3 * Hg * D:4 * Hg * D], L["gnorm"], cfg.rms_norm_eps)
        return y @ L["o"].t()

    def greedy(self, prompt: list, n_new: int) -> tuple:
        """Greedy decode by re-running the dense forward; returns (tokens, per-step logits)."""
        ids = list(prompt)
        all_logits = []
        for _ in range(n_new):
            logits = self.forward(torch.tensor(ids))[-1]
            all_logits.append(logits)
            ids.append(int(logits.argmax()))
        return ids[len(prompt):], torch.stack(all_logits)
