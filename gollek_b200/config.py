"""Typed configuration for models and the serving engine.

``ModelConfig`` parses a Hugging Face ``config.json`` (or GGUF metadata, see
``gollek_b200.loaders.gguf``) into the fields the model graph needs. It mirrors
the reference's ``ModelConfig`` parser (core/spi/gollek-spi-model/…/spi/model/
ModelConfig.java:116-117, 257-295, 595-603) with one deliberate difference:
``rope_theta`` is always read from the config (the reference's Direct engine
hard-codes 10000, runner/safetensor/gollek-safetensor-engine/…/attention/
FlashAttentionKernel.java:103-105), so Llama-3's 500000 is honoured.

``EngineConfig`` replaces the reference's SmallRye config mappings
(runner/llamacpp/gollek-runner-llamacpp/…/LlamaCppProviderConfig.java:29-175)
and perf-mode profiles (core/optimization/gollek-plugin-perfmode/…/
PerformanceModeService.java) with one dataclass loadable from YAML/JSON, the
environment (``GOLLEK_*``) and CLI flags.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any, Optional


@dataclass
class RopeScaling:
    """RoPE frequency scaling (HF ``rope_scaling``): ``none``, ``linear``, ``llama3``,
    ``longrope`` (Phi-3 long-context: per-pair short/long factors) or ``yarn`` (DeepSeek-V3:
    NTK-by-parts interpolation between ``beta_fast`` and ``beta_slow`` rotations, cos/sin scaled
    by mscale(factor, mscale) / mscale(factor, mscale_all_dim))."""
    kind: str = "none"
    factor: float = 1.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192
    short_factor: Optional[list] = None
    long_factor: Optional[list] = None
    beta_fast: float = 32.0
    beta_slow: float = 1.0
    mscale: float = 0.0
    mscale_all_dim: float = 0.0

    @staticmethod
    def from_hf(d: Optional[dict]) -> "RopeScaling":
        if not d:
            return RopeScaling()
        kind = d.get("rope_type", d.get("type", "none")) or "none"
        if kind == "default":
            kind = "none"
        if kind == "su":
            kind = "longrope"
        return RopeScaling(
            kind=kind,
            factor=float(d.get("factor", 1.0) or 1.0),
            low_freq_factor=float(d.get("low_freq_factor", 1.0)),
            high_freq_factor=float(d.get("high_freq_factor", 4.0)),
            original_max_position_embeddings=int(d.get("original_max_position_embeddings", 8192) or 8192),
            short_factor=d.get("short_factor"),
            long_factor=d.get("long_factor"),
            beta_fast=float(d.get("beta_fast") or 32.0),
            beta_slow=float(d.get("beta_slow") or 1.0),
            mscale=float(d.get("mscale") or 0.0),
            mscale_all_dim=float(d.get("mscale_all_dim") or 0.0),
        )


def yarn_mscale(scale: float, m: float = 1.0) -> float:
    """YaRN attention-temperature factor 0.1 * m * ln(scale) + 1 (1 for scale <= 1)."""
    import math
    return 1.0 if scale <= 1 else 0.1 * m * math.log(scale) + 1.0


# Model families handled by the decoder graph (models/llama.py). Llama-like families differ in
# projection biases, QK-norm, sliding windows, norm placement and activation; Gemma adds a
# sqrt(hidden) embedding scale, (1 + w) RMSNorm weights, GeGLU, sandwich norms and softcapping.
# DeepSeek-V3 (also DeepSeek-R1 and Kimi-K2) adds multi-head latent attention and group-limited
# sigmoid-routed MoE with shared experts.
FAMILIES = ("llama", "mistral", "mixtral", "qwen2", "qwen3", "gemma", "gemma2", "gemma3", "phi3", "cohere2",
            "deepseek_v3")


@dataclass
class ModelConfig:
    """Architecture hyper-parameters of a decoder-only transformer (the families in ``FAMILIES``)."""
    architecture: str = "llama"          # one of FAMILIES
    vocab_size: int = 32000
    hidden_size: int = 4096
    intermediate_size: int = 14336
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: RopeScaling = field(default_factory=RopeScaling)
    max_position_embeddings: int = 8192
    tie_word_embeddings: bool = False
    # MoE (Mixtral)
    num_local_experts: int = 0
    num_experts_per_tok: int = 0
    # extras some families use
    attention_bias: bool = False         # q/k/v projection biases (Qwen2)
    qk_norm: bool = False                # per-head RMSNorm of q and k before RoPE (Qwen3, Gemma-3)
    sliding_window: int = 0              # 0 = full attention
    layer_types: Optional[list] = None   # per layer "full_attention" | "sliding_attention" (None: all
                                         # layers sliding when sliding_window > 0)
    rope_local_theta: float = 0.0        # RoPE base of sliding layers when it differs (Gemma-3)
    attn_logit_softcapping: float = 0.0  # Gemma-2
    final_logit_softcapping: float = 0.0
    query_pre_attn_scalar: float = 0.0   # attention scale = this ** -0.5 (Gemma); 0 = head_dim
    hidden_act: str = "silu"             # "silu" (SwiGLU) | "gelu_tanh" (GeGLU)
    norm_unit_offset: bool = False       # RMSNorm scales by (1 + w) (Gemma)
    embed_scale: float = 1.0             # embeddings multiplied by this (Gemma: sqrt(hidden))
    sandwich_norm: bool = False          # norms after attention / MLP outputs too (Gemma-2/3)
    # Cohere-2: bias-free LayerNorm, attention and MLP in parallel off one norm, interleaved-pair RoPE
    # on sliding-window layers only (full layers use no positions), logits times logit_scale
    norm_center: bool = False
    parallel_block: bool = False
    rope_interleaved: bool = False
    rope_sliding_only: bool = False
    logit_scale: float = 1.0
    # hybrid gated-delta-rule / attention stacks: "H1" = {G,G,G,G,A,G}, "H2" = {G,G,A,G,G,A} per 6
    # layers (G = Gated DeltaNet layer, A = softmax attention); None = attention only
    hybrid_schedule: Optional[str] = None
    gdn_num_heads: int = 0               # GDN heads (0: num_attention_heads); head dim 128
    # multi-head latent attention (DeepSeek-V3): q = W_qb norm(W_qa x) (or W_q x without q_lora_rank),
    # [c | k_rope] = W_kva x, [k_nope | v] = W_kvb norm(c) per head; RoPE on the qk_rope_head_dim dims
    # (k_rope shared by all heads); head_dim = qk_nope_head_dim + qk_rope_head_dim
    q_lora_rank: int = 0
    kv_lora_rank: int = 0                # > 0 selects MLA
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0
    # MoE variants: expert width, shared experts, router scoring and group limit, dense first layers
    moe_intermediate_size: int = 0       # 0: intermediate_size
    n_shared_experts: int = 0
    moe_scoring: str = "softmax"         # "softmax" (Mixtral) | "sigmoid" (DeepSeek-V3, bias-corrected choice)
    n_group: int = 1                     # experts are chosen inside the topk_group best of n_group groups
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    norm_topk_prob: bool = True
    first_k_dense_replace: int = 0       # layers [0, k) use a dense MLP of intermediate_size
    bos_token_id: int = 1
    eos_token_id: int = 2

    @property
    def is_moe(self) -> bool:
        return self.num_local_experts > 0

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @property
    def rope_dim(self) -> int:
        """Rotary dims per head (the qk_rope_head_dim part under MLA)."""
        return self.qk_rope_head_dim if self.is_mla else self.head_dim

    @property
    def moe_ffn(self) -> int:
        return self.moe_intermediate_size or self.intermediate_size

    def is_moe_layer(self, i: int) -> bool:
        return self.is_moe and i >= self.first_k_dense_replace

    @property
    def attn_scale(self) -> float:
        s = (self.query_pre_attn_scalar or self.head_dim) ** -0.5
        rs = self.rope_scaling
        if self.is_mla and rs.kind == "yarn" and rs.mscale_all_dim:
            s *= yarn_mscale(rs.factor, rs.mscale_all_dim) ** 2
        return s

    def layer_window(self, i: int) -> int:
        """Sliding window of layer ``i`` (0 = full attention)."""
        if self.sliding_window <= 0:
            return 0
        if self.layer_types is None:
            return self.sliding_window
        return self.sliding_window if self.layer_types[i] == "sliding_attention" else 0

    def is_gdn_layer(self, i: int) -> bool:
        """Layer ``i`` is a gated-delta-rule layer under the hybrid schedule."""
        if not self.hybrid_schedule:
            return False
        pat = {"H1": (1, 1, 1, 1, 0, 1), "H2": (1, 1, 0, 1, 1, 0)}.get(self.hybrid_schedule.upper())
        if pat is None:
            raise ValueError(f"unknown hybrid_schedule {self.hybrid_schedule!r} (H1 | H2)")
        return bool(pat[i % 6])

    @property
    def gdn_heads(self) -> int:
        return self.gdn_num_heads or self.num_attention_heads

    @property
    def gdn_head_dim(self) -> int:
        return 128

    def layer_rope_theta(self, i: int) -> float:
        if self.rope_local_theta and self.layer_window(i) > 0:
            return self.rope_local_theta
        return self.rope_theta

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def _attn_params(self) -> int:
        h = self.hidden_size
        if not self.is_mla:
            return h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        nh, qk = self.num_attention_heads, self.head_dim
        q = (h * self.q_lora_rank + self.q_lora_rank * nh * qk) if self.q_lora_rank else h * nh * qk
        kv = h * (self.kv_lora_rank + self.qk_rope_head_dim) + self.kv_lora_rank * nh * (
            self.qk_nope_head_dim + self.v_head_dim)
        return q + kv + nh * self.v_head_dim * h

    def _ffn_params(self, i: int, active: bool) -> int:
        h = self.hidden_size
        if not self.is_moe_layer(i):
            return 3 * h * self.intermediate_size
        n = self.num_experts_per_tok if active else self.num_local_experts
        return 3 * h * self.moe_ffn * (n + self.n_shared_experts) + h * self.num_local_experts

    def num_params(self) -> int:
        h, v = self.hidden_size, self.vocab_size
        body = sum(self._attn_params() + self._ffn_params(i, False) + 2 * h for i in range(self.num_hidden_layers))
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return body + emb + h

    def flops_per_token(self) -> float:
        """Dense matmul FLOPs per token (2 per MAC), ignoring attention scores."""
        h = self.hidden_size
        body = sum(self._attn_params() + self._ffn_params(i, True) for i in range(self.num_hidden_layers))
        return 2.0 * (body + h * self.vocab_size)

    @staticmethod
    def from_hf(d: dict) -> "ModelConfig":
        """Parse a Hugging Face ``config.json`` dictionary (transformers 4.x or 5.x layout)."""
        if "text_config" in d and isinstance(d["text_config"], dict):  # multimodal wrappers (Gemma-3)
            d = {**d["text_config"], "architectures": d.get("architectures")}
            d.setdefault("model_type", "gemma3_text")
        archs = d.get("architectures") or []
        mt = str(d.get("model_type", "llama"))
        fam = {"llama": "llama", "mistral": "mistral", "mixtral": "mixtral", "qwen2": "qwen2", "qwen3": "qwen3",
               "gemma": "gemma", "gemma2": "gemma2", "gemma3_text": "gemma3", "gemma3": "gemma3",
               "phi3": "phi3", "cohere2": "cohere2", "yi": "llama", "deepseek_v3": "deepseek_v3",
               "kimi_k2": "deepseek_v3"}.get(mt)
        if fam is None and any("DeepseekV3" in a for a in archs):
            fam = "deepseek_v3"
        if fam is None:
            fam = "mixtral" if any("Mixtral" in a for a in archs) else "llama"
        gemma = fam.startswith("gemma")
        nh = int(d.get("num_attention_heads", 32))
        hs = int(d.get("hidden_size", 4096))
        nl = int(d.get("num_hidden_layers", 32))
        eos = d.get("eos_token_id", 2)
        if isinstance(eos, list):
            eos = eos[0]
        # RoPE: transformers 5 nests it in rope_parameters (per layer type for Gemma-3)
        rp = d.get("rope_parameters") or {}
        full_rp = rp.get("full_attention", rp) if isinstance(rp, dict) else {}
        local_rp = rp.get("sliding_attention", {}) if isinstance(rp, dict) else {}
        theta = d.get("rope_theta") or full_rp.get("rope_theta") or (1_000_000.0 if fam == "gemma3" else 10000.0)
        scaling = d.get("rope_scaling")
        if scaling is None and full_rp.get("rope_type") not in (None, "default"):
            scaling = full_rp
        if scaling and "original_max_position_embeddings" not in scaling and d.get("original_max_position_embeddings"):
            scaling = {**scaling, "original_max_position_embeddings": d["original_max_position_embeddings"]}
        local_theta = d.get("rope_local_base_freq") or local_rp.get("rope_theta") or (10000.0 if fam == "gemma3" else 0.0)
        # sliding windows
        sw = int(d.get("sliding_window") or 0)
        layer_types = d.get("layer_types")
        if fam in ("qwen2", "qwen3"):
            if not d.get("use_sliding_window", False):
                sw, layer_types = 0, None
            elif layer_types is None:
                mwl = int(d.get("max_window_layers", 0) or 0)
                layer_types = ["sliding_attention" if i >= mwl else "full_attention" for i in range(nl)]
        elif fam == "gemma2" and layer_types is None and sw:
            layer_types = ["sliding_attention" if (i + 1) % 2 else "full_attention" for i in range(nl)]
        elif fam == "gemma3" and layer_types is None and sw:
            pat = int(d.get("sliding_window_pattern", 6) or 6)
            layer_types = ["sliding_attention" if (i + 1) % pat else "full_attention" for i in range(nl)]
        elif fam == "gemma":
            sw, layer_types = 0, None
        elif fam == "cohere2" and layer_types is None and sw:
            pat = int(d.get("sliding_window_pattern", 4) or 4)
            layer_types = ["sliding_attention" if (i + 1) % pat else "full_attention" for i in range(nl)]
        cohere = fam == "cohere2"
        ds = fam == "deepseek_v3"
        mla = {}
        if ds:
            mla = dict(q_lora_rank=int(d.get("q_lora_rank") or 0), kv_lora_rank=int(d.get("kv_lora_rank") or 512),
                       qk_nope_head_dim=int(d.get("qk_nope_head_dim", 128)),
                       qk_rope_head_dim=int(d.get("qk_rope_head_dim", 64)), v_head_dim=int(d.get("v_head_dim", 128)),
                       moe_intermediate_size=int(d.get("moe_intermediate_size", 0) or 0),
                       n_shared_experts=int(d.get("n_shared_experts", 0) or 0), moe_scoring="sigmoid",
                       n_group=int(d.get("n_group", 1) or 1), topk_group=int(d.get("topk_group", 1) or 1),
                       routed_scaling_factor=float(d.get("routed_scaling_factor", 1.0) or 1.0),
                       norm_topk_prob=bool(d.get("norm_topk_prob", True)),
                       first_k_dense_replace=int(d.get("first_k_dense_replace", 0) or 0))
        act = str(d.get("hidden_activation") or d.get("hidden_act") or "silu")
        act = "gelu_tanh" if (gemma or act.startswith("gelu")) else "silu"
        return ModelConfig(
            architecture=fam,
            vocab_size=int(d.get("vocab_size", 32000)),
            hidden_size=hs,
            intermediate_size=int(d.get("intermediate_size", 4 * hs)),
            num_hidden_layers=nl,
            num_attention_heads=nh,
            num_key_value_heads=int(d.get("num_key_value_heads", nh) or nh),
            head_dim=(mla["qk_nope_head_dim"] + mla["qk_rope_head_dim"]) if ds else int(d.get("head_dim") or hs // nh),
            rms_norm_eps=float(d.get("layer_norm_eps", 1e-5) if cohere else d.get("rms_norm_eps", 1e-6 if gemma else 1e-5)),
            rope_theta=float(theta),
            rope_scaling=RopeScaling.from_hf(scaling),
            max_position_embeddings=int(d.get("max_position_embeddings", 8192)),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", gemma or cohere)),
            num_local_experts=int(d.get("n_routed_experts" if ds else "num_local_experts", 0) or 0),
            num_experts_per_tok=int(d.get("num_experts_per_tok", 0) or 0),
            attention_bias=True if fam == "qwen2" else bool(d.get("attention_bias", False)),
            qk_norm=fam in ("qwen3", "gemma3"),
            sliding_window=sw,
            layer_types=list(layer_types) if layer_types else None,
            rope_local_theta=float(local_theta) if fam == "gemma3" else 0.0,
            attn_logit_softcapping=float(d.get("attn_logit_softcapping") or 0.0),
            final_logit_softcapping=float(d.get("final_logit_softcapping") or 0.0),
            query_pre_attn_scalar=float(d.get("query_pre_attn_scalar") or 0.0) if gemma else 0.0,
            hidden_act=act,
            norm_unit_offset=gemma,
            embed_scale=float(hs) ** 0.5 if gemma else 1.0,
            sandwich_norm=fam in ("gemma2", "gemma3"),
            norm_center=cohere,
            parallel_block=cohere,
            rope_interleaved=cohere or (ds and bool(d.get("rope_interleave", True))),
            rope_sliding_only=cohere,
            logit_scale=float(d.get("logit_scale", 1.0) or 1.0) if cohere else 1.0,
            bos_token_id=int(d.get("bos_token_id", 1) or 1),
            eos_token_id=int(eos if eos is not None else 2),
            **mla,
        )

    def to_hf(self) -> dict:
        fam = self.architecture
        names = {"llama": ("LlamaForCausalLM", "llama"), "mistral": ("MistralForCausalLM", "mistral"),
                 "mixtral": ("MixtralForCausalLM", "mixtral"), "qwen2": ("Qwen2ForCausalLM", "qwen2"),
                 "qwen3": ("Qwen3ForCausalLM", "qwen3"), "gemma": ("GemmaForCausalLM", "gemma"),
                 "gemma2": ("Gemma2ForCausalLM", "gemma2"), "gemma3": ("Gemma3ForCausalLM", "gemma3_text"),
                 "phi3": ("Phi3ForCausalLM", "phi3"), "cohere2": ("Cohere2ForCausalLM", "cohere2"),
                 "deepseek_v3": ("DeepseekV3ForCausalLM", "deepseek_v3")}
        arch, mt = names.get(fam, names["mixtral" if self.is_moe else "llama"])
        d = {
            "architectures": [arch],
            "model_type": mt,
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "rms_norm_eps": self.rms_norm_eps,
            "rope_theta": self.rope_theta,
            "max_position_embeddings": self.max_position_embeddings,
            "tie_word_embeddings": self.tie_word_embeddings,
            "attention_bias": self.attention_bias,
            "bos_token_id": self.bos_token_id,
            "eos_token_id": self.eos_token_id,
            "hidden_act": "gelu_pytorch_tanh" if self.hidden_act == "gelu_tanh" else "silu",
            "torch_dtype": "bfloat16",
        }
        if fam.startswith("gemma"):
            d["hidden_activation"] = d["hidden_act"]
        if fam == "phi3":  # its default pad id (32000) lies outside small vocabularies
            d["pad_token_id"] = min(32000, self.vocab_size - 1)
        if self.sliding_window:
            d["sliding_window"] = self.sliding_window
            if fam in ("qwen2", "qwen3"):
                d["use_sliding_window"] = True
                d["max_window_layers"] = 0
        elif fam in ("mistral", "phi3", "gemma2", "gemma3"):
            d["sliding_window"] = None
        if self.layer_types:
            d["layer_types"] = list(self.layer_types)
        if self.query_pre_attn_scalar:
            q = self.query_pre_attn_scalar
            d["query_pre_attn_scalar"] = int(q) if float(q).is_integer() else q
        if fam in ("gemma2", "gemma3"):
            d["attn_logit_softcapping"] = self.attn_logit_softcapping or None
            d["final_logit_softcapping"] = self.final_logit_softcapping or None
        if fam == "gemma3":
            d["rope_local_base_freq"] = self.rope_local_theta or 10000.0
        if fam == "cohere2":
            d["layer_norm_eps"] = d.pop("rms_norm_eps")
            d["logit_scale"] = self.logit_scale
            d["pad_token_id"] = 0
        if self.rope_scaling.kind != "none":
            rs = self.rope_scaling
            d["rope_scaling"] = {"rope_type": rs.kind, "factor": rs.factor,
                                 "low_freq_factor": rs.low_freq_factor,
                                 "high_freq_factor": rs.high_freq_factor,
                                 "original_max_position_embeddings": rs.original_max_position_embeddings}
            if rs.kind == "yarn":
                d["rope_scaling"] = {"rope_type": "yarn", "factor": rs.factor, "beta_fast": rs.beta_fast,
                                     "beta_slow": rs.beta_slow, "mscale": rs.mscale,
                                     "mscale_all_dim": rs.mscale_all_dim,
                                     "original_max_position_embeddings": rs.original_max_position_embeddings}
            if rs.kind == "longrope":
                d["rope_scaling"] = {"type": "longrope", "short_factor": rs.short_factor,
                                     "long_factor": rs.long_factor}
                d["original_max_position_embeddings"] = rs.original_max_position_embeddings
        if self.is_moe:
            d["num_local_experts"] = self.num_local_experts
            d["num_experts_per_tok"] = self.num_experts_per_tok
        if fam == "deepseek_v3":
            d.pop("head_dim")
            d.pop("num_local_experts", None)
            d.update(q_lora_rank=self.q_lora_rank or None, kv_lora_rank=self.kv_lora_rank,
                     qk_nope_head_dim=self.qk_nope_head_dim, qk_rope_head_dim=self.qk_rope_head_dim,
                     v_head_dim=self.v_head_dim, n_routed_experts=self.num_local_experts,
                     moe_intermediate_size=self.moe_ffn, n_shared_experts=self.n_shared_experts,
                     n_group=self.n_group, topk_group=self.topk_group,
                     routed_scaling_factor=self.routed_scaling_factor, norm_topk_prob=self.norm_topk_prob,
                     first_k_dense_replace=self.first_k_dense_replace, rope_interleave=self.rope_interleaved)
        return d


# Named architectures used by tests and benchmarks (random-init weights; shapes only).
PRESETS: dict[str, ModelConfig] = {
    "tiny-llama": ModelConfig(
        architecture="llama", vocab_size=32000, hidden_size=256, intermediate_size=688,
        num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
        rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=2048),
    "tiny-hybrid": ModelConfig(
        architecture="llama", vocab_size=1024, hidden_size=256, intermediate_size=512,
        num_hidden_layers=6, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
        rope_theta=10000.0, max_position_embeddings=2048, hybrid_schedule="H2", gdn_num_heads=2),
    "tiny-cohere2": ModelConfig(
        architecture="cohere2", vocab_size=1024, hidden_size=256, intermediate_size=512,
        num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
        rope_theta=10000.0, max_position_embeddings=2048, tie_word_embeddings=True, sliding_window=24,
        layer_types=["sliding_attention", "sliding_attention", "sliding_attention", "full_attention"],
        norm_center=True, parallel_block=True, rope_interleaved=True, rope_sliding_only=True, logit_scale=0.25),
    "tiny-mixtral": ModelConfig(
        architecture="mixtral", vocab_size=1024, hidden_size=256, intermediate_size=512,
        num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
        rope_theta=10000.0, num_local_experts=8, num_experts_per_tok=2, max_position_embeddings=2048),
    "tiny-deepseek-v3": ModelConfig(
        architecture="deepseek_v3", vocab_size=1024, hidden_size=256, intermediate_size=512,
        num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=4, head_dim=96, rms_norm_eps=1e-6,
        rope_theta=10000.0, max_position_embeddings=2048, q_lora_rank=128, kv_lora_rank=64,
        qk_nope_head_dim=64, qk_rope_head_dim=32, v_head_dim=64, rope_interleaved=True,
        num_local_experts=16, num_experts_per_tok=4, moe_intermediate_size=128, n_shared_experts=1,
        moe_scoring="sigmoid", n_group=4, topk_group=2, routed_scaling_factor=2.5, first_k_dense_replace=1),
    "llama-3-8b": ModelConfig(
        architecture="llama", vocab_size=128256, hidden_size=4096, intermediate_size=14336,
        num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
        rms_norm_eps=1e-5, rope_theta=500000.0, max_position_embeddings=8192,
        bos_token_id=128000, eos_token_id=128001),
    "llama-3-70b": ModelConfig(
        architecture="llama", vocab_size=128256, hidden_size=8192, intermediate_size=28672,
        num_hidden_layers=80, num_attention_heads=64, num_key_value_heads=8, head_dim=128,
        rms_norm_eps=1e-5, rope_theta=500000.0, max_position_embeddings=8192,
        bos_token_id=128000, eos_token_id=128001),
    # tiny random-init members of the other families (tests: each exercises its family's features)
    "tiny-qwen2": ModelConfig(
        architecture="qwen2", vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=8, num_key_value_heads=2, head_dim=32, rms_norm_eps=1e-6, rope_theta=1e6,
        attention_bias=True, tie_word_embeddings=True, max_position_embeddings=2048),
    "tiny-qwen3": ModelConfig(
        architecture="qwen3", vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
        qk_norm=True, max_position_embeddings=2048),
    "tiny-mistral": ModelConfig(
        architecture="mistral", vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=8, num_key_value_heads=2, head_dim=32, rope_theta=10000.0, sliding_window=24,
        max_position_embeddings=2048),
    "tiny-gemma": ModelConfig(
        architecture="gemma", vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=2, num_key_value_heads=1, head_dim=256, rms_norm_eps=1e-6, hidden_act="gelu_tanh",
        norm_unit_offset=True, embed_scale=16.0, tie_word_embeddings=True, max_position_embeddings=2048),
    "tiny-gemma2": ModelConfig(
        architecture="gemma2", vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, rms_norm_eps=1e-6, hidden_act="gelu_tanh",
        norm_unit_offset=True, embed_scale=16.0, tie_word_embeddings=True, sandwich_norm=True,
        sliding_window=16, layer_types=["sliding_attention", "full_attention"] * 2, attn_logit_softcapping=50.0,
        final_logit_softcapping=30.0, query_pre_attn_scalar=64.0, max_position_embeddings=2048),
    "tiny-gemma3": ModelConfig(
        architecture="gemma3", vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=6,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-6, hidden_act="gelu_tanh",
        norm_unit_offset=True, embed_scale=16.0, tie_word_embeddings=True, sandwich_norm=True, qk_norm=True,
        sliding_window=16, layer_types=["sliding_attention"] * 5 + ["full_attention"], rope_theta=1e6,
        rope_local_theta=10000.0, query_pre_attn_scalar=128.0, max_position_embeddings=2048),
    "tiny-phi3": ModelConfig(
        architecture="phi3", vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=8, num_key_value_heads=8, head_dim=32, rope_theta=10000.0, sliding_window=40,
        max_position_embeddings=2048),
    # full-size members (random init for benchmarks; real checkpoints carry their own config.json)
    "qwen2.5-7b": ModelConfig(
        architecture="qwen2", vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
        num_attention_heads=28, num_key_value_heads=4, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
        attention_bias=True, max_position_embeddings=32768, eos_token_id=151645),
    "qwen3-8b": ModelConfig(
        architecture="qwen3", vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
        qk_norm=True, max_position_embeddings=40960, eos_token_id=151645),
    "mistral-7b": ModelConfig(
        architecture="mistral", vocab_size=32768, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1e6, max_position_embeddings=32768),
    "gemma-2-9b": ModelConfig(
        architecture="gemma2", vocab_size=256000, hidden_size=3584, intermediate_size=14336, num_hidden_layers=42,
        num_attention_heads=16, num_key_value_heads=8, head_dim=256, rms_norm_eps=1e-6, hidden_act="gelu_tanh",
        norm_unit_offset=True, embed_scale=3584 ** 0.5, tie_word_embeddings=True, sandwich_norm=True,
        sliding_window=4096, layer_types=["sliding_attention", "full_attention"] * 21, attn_logit_softcapping=50.0,
        final_logit_softcapping=30.0, query_pre_attn_scalar=256.0, max_position_embeddings=8192,
        bos_token_id=2, eos_token_id=1),
    "phi-3-mini-4k": ModelConfig(
        architecture="phi3", vocab_size=32064, hidden_size=3072, intermediate_size=8192, num_hidden_layers=32,
        num_attention_heads=32, num_key_value_heads=32, head_dim=96, rope_theta=10000.0, sliding_window=2047,
        max_position_embeddings=4096, eos_token_id=32000),
    "mixtral-8x7b": ModelConfig(
        architecture="mixtral", vocab_size=32000, hidden_size=4096, intermediate_size=14336,
        num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
        rms_norm_eps=1e-5, rope_theta=1000000.0, num_local_experts=8, num_experts_per_tok=2,
        max_position_embeddings=32768),
    "deepseek-v3": ModelConfig(
        architecture="deepseek_v3", vocab_size=129280, hidden_size=7168, intermediate_size=18432,
        num_hidden_layers=61, num_attention_heads=128, num_key_value_heads=128, head_dim=192, rms_norm_eps=1e-6,
        rope_theta=10000.0, max_position_embeddings=163840,
        rope_scaling=RopeScaling(kind="yarn", factor=40.0, original_max_position_embeddings=4096, beta_fast=32.0,
                                 beta_slow=1.0, mscale=1.0, mscale_all_dim=1.0),
        q_lora_rank=1536, kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
        rope_interleaved=True, num_local_experts=256, num_experts_per_tok=8, moe_intermediate_size=2048,
        n_shared_experts=1, moe_scoring="sigmoid", n_group=8, topk_group=4, routed_scaling_factor=2.5,
        first_k_dense_replace=3, bos_token_id=0, eos_token_id=1),
}


def preset(name: str, **overrides: Any) -> ModelConfig:
    cfg = dataclasses.replace(PRESETS[name])
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


@dataclass
class SamplingDefaults:
    """Server-side sampling defaults (reference: plugins/gollek-plugin-sampling/…/
    SamplingPolicyPlugin.java:44-54 — temperature 0.7, top_k 40, top_p 0.95, repetition 1.1)."""
    temperature: float = 0.7
    top_k: int = 40
    top_p: float = 0.95
    min_p: float = 0.0
    repetition_penalty: float = 1.1
    max_tokens: int = 512


@dataclass
class EngineConfig:
    """Serving-engine configuration (one dataclass for everything the engine tunes)."""
    model: str = "tiny-llama"                 # preset name or checkpoint path
    dtype: str = "bfloat16"
    quantization: str = "none"                # none | fp8 | int8 | gguf | int4 | nf4 (GPTQ/AWQ checkpoints: automatic)
    device: str = "cuda"
    tensor_parallel_size: int = 1
    enable_expert_parallel: bool = False  # MoE: experts partitioned over the TP ranks (EP = TP size)
    ep_rebalance_interval: int = 0        # EP: re-place experts by routed load every N engine steps (0 = off)
    # EP: token-sharded MoE layers with the NVLink all-to-all (dispatch -> grouped expert GEMMs ->
    # combine) when the TP comm has an NVLink multicast object; otherwise replicated activations
    ep_all_to_all: bool = True
    # tensor parallelism: steps of at least this many tokens run as two halves whose collectives
    # (on a second stream) overlap the other half's compute; the GEMMs leave `tp_overlap_sms` SMs
    # free for them (0 = never split). Only from `tp_overlap_min_world` ranks up: at 2 ranks the
    # collective share is small and the halved GEMMs cost more than the overlap saves (measured:
    # Llama-3-8B TP2 bench 18.3K tok/s without, 17.9K with)
    tp_overlap_min_tokens: int = 1024
    tp_overlap_sms: int = 16
    tp_overlap_min_world: int = 4
    # measure instead of assuming: the first 12 eligible steps alternate split / whole, their device
    # time per token is compared (medians, agreed across the ranks) and the faster mode is kept
    tp_overlap_autotune: bool = True
    # speculative decoding: "none" | "ngram" (prompt lookup) | "draft" (draft model ``draft_model``)
    speculative_method: str = "none"
    num_speculative_tokens: int = 4
    ngram_min: int = 1
    ngram_max: int = 4
    draft_model: Optional[str] = None
    # overlap the host side of step N+1 (schedule, batch build, launches) with step N on the GPU;
    # steps that need host-visible history (penalties, speculative decoding, P/D hand-off) run
    # synchronously
    async_scheduling: bool = True
    # host garbage collection: with thousands of running sequences every full collection walks all
    # their token lists (~0.1 s each, every ~10 steps); raise the collection thresholds and freeze
    # the objects built at start-up so a step's host work stays flat (cycles are still collected)
    gc_tuning: bool = True
    # weight offload: the last `offload_layers` layers stream from pinned host memory, prefetched
    # `offload_prefetch` layers ahead (for models larger than device memory; disables CUDA graphs)
    offload_layers: int = 0
    offload_prefetch: int = 2
    # multi-tenant admission: tenant -> {"max_running": n, "max_kv_blocks": n}; requests of a tenant
    # at its quota wait while other tenants' requests are admitted
    tenant_quotas: dict = field(default_factory=dict)
    # checkpoint / resume: prefix-cache snapshot and unfinished-request snapshot paths (written at
    # shutdown, read at startup when present)
    prefix_cache_snapshot: Optional[str] = None
    request_snapshot: Optional[str] = None
    expert_parallel_size: int = 1
    # paged KV cache
    block_size: int = 16
    num_gpu_blocks: Optional[int] = None      # None => size from memory fraction
    gpu_memory_utilization: float = 0.85
    kv_cache_dtype: str = "auto"              # auto (= model dtype) | fp8 (e4m3, a scale per token and head)
    enable_prefix_caching: bool = True
    # KV eviction under memory pressure (opt-in; changes outputs): when the block pool is more than
    # `kv_eviction_threshold` full, the longest running sequences drop their least important KV
    # blocks (key-norm + recency score) down to `kv_retention_target` of their blocks; the first
    # `kv_protect_sink_blocks` blocks and the most recent `kv_protect_recent` fraction are kept
    kv_eviction: bool = False
    kv_eviction_threshold: float = 0.85
    kv_retention_target: float = 0.6
    kv_protect_sink_blocks: int = 1
    kv_protect_recent: float = 0.2
    kv_eviction_min_blocks: int = 8
    # scheduler
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    max_model_len: int = 8192
    scheduling_policy: str = "fcfs"           # fcfs | wait (KV-capacity admission with length prediction)
    wait_admission_fraction: float = 0.95
    preemption_mode: str = "recompute"
    # LoRA
    enable_lora: bool = False
    max_loras: int = 64
    max_lora_rank: int = 16
    # execution
    use_cuda_graphs: bool = True
    cuda_graph_batch_sizes: tuple = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512)
    comm_backend: str = "fused"               # fused (own P2P kernels) | nccl (baseline)
    seed: int = 0
    perf_mode: str = "balanced"               # balanced | interactivity | throughput
    sampling: SamplingDefaults = field(default_factory=SamplingDefaults)

    def apply_perf_mode(self) -> None:
        """Profiles mirroring core/optimization/gollek-plugin-perfmode/…/PerformanceModeService.java."""
        if self.perf_mode == "interactivity":
            self.max_num_seqs = min(self.max_num_seqs, 64)
            self.max_num_batched_tokens = min(self.max_num_batched_tokens, 2048)
        elif self.perf_mode == "throughput":
            self.max_num_seqs = max(self.max_num_seqs, 512)
            self.max_num_batched_tokens = max(self.max_num_batched_tokens, 16384)

    @staticmethod
    def load(path: Optional[str] = None, env: Optional[dict] = None, **overrides: Any) -> "EngineConfig":
        """Build from (in increasing precedence) a YAML/JSON file, ``GOLLEK_*`` env vars, keyword overrides."""
        cfg = EngineConfig()
        data: dict = {}
        if path:
            with open(path) as f:
                text = f.read()
            if path.endswith((".yaml", ".yml")):
                import yaml
                data = yaml.safe_load(text) or {}
            else:
                data = json.loads(text)
        env = os.environ if env is None else env
        fields = {f.name: f for f in dataclasses.fields(EngineConfig)}
        for name in fields:
            key = "GOLLEK_" + name.upper()
            if key in env:
                data[name] = env[key]
        data.update(overrides)
        for k, v in data.items():
            if k not in fields:
                raise ValueError(f"unknown engine config key {k!r}")
            if k == "sampling" and isinstance(v, dict):
                v = SamplingDefaults(**v)
            else:
                cur = getattr(cfg, k)
                v = _coerce(v, cur)
            setattr(cfg, k, v)
        cfg.apply_perf_mode()
        return cfg


def _coerce(v: Any, cur: Any) -> Any:
    if isinstance(v, str) and not isinstance(cur, str):
        if isinstance(cur, bool):
            return v.lower() in ("1", "true", "yes", "on")
        if isinstance(cur, int) or cur is None:
            try:
                return int(v)
            except ValueError:
                return float(v)
        if isinstance(cur, float):
            return float(v)
        if isinstance(cur, tuple):
            return tuple(int(x) for x in v.split(","))
    if isinstance(cur, tuple) and isinstance(v, list):
        return tuple(v)
    return v
