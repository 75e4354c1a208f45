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
    """RoPE frequency scaling (HF ``rope_scaling``): ``none``, ``linear`` or ``llama3``."""
    kind: str = "none"
    factor: float = 1.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192

    @staticmethod
    def from_hf(d: Optional[dict]) -> "RopeScaling":
        if not d:
            return RopeScaling()
        kind = d.get("rope_type", d.get("type", "none")) or "none"
        if kind == "default":
            kind = "none"
        return RopeScaling(
            kind=kind,
            factor=float(d.get("factor", 1.0)),
            low_freq_factor=float(d.get("low_freq_factor", 1.0)),
            high_freq_factor=float(d.get("high_freq_factor", 4.0)),
            original_max_position_embeddings=int(d.get("original_max_position_embeddings", 8192)),
        )


@dataclass
class ModelConfig:
    """Architecture hyper-parameters of a decoder-only transformer (Llama / Mixtral family)."""
    architecture: str = "llama"          # "llama" | "mixtral"
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
    attention_bias: bool = False
    bos_token_id: int = 1
    eos_token_id: int = 2

    @property
    def is_moe(self) -> bool:
        return self.num_local_experts > 0

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def num_params(self) -> int:
        h, f, v = self.hidden_size, self.intermediate_size, self.vocab_size
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        ffn = 3 * h * f * max(1, self.num_local_experts)
        if self.is_moe:
            ffn += h * self.num_local_experts
        per_layer = attn + ffn + 2 * h
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_hidden_layers * per_layer + emb + h

    def flops_per_token(self) -> float:
        """Dense matmul FLOPs per token (2 per MAC), ignoring attention scores."""
        h, f = self.hidden_size, self.intermediate_size
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        ffn = 3 * h * f * (self.num_experts_per_tok if self.is_moe else 1)
        return 2.0 * (self.num_hidden_layers * (attn + ffn) + h * self.vocab_size)

    @staticmethod
    def from_hf(d: dict) -> "ModelConfig":
        """Parse a Hugging Face ``config.json`` dictionary."""
        archs = d.get("architectures") or []
        model_type = d.get("model_type", "llama")
        arch = "mixtral" if (model_type == "mixtral" or any("Mixtral" in a for a in archs)) else "llama"
        nh = int(d.get("num_attention_heads", 32))
        hs = int(d.get("hidden_size", 4096))
        eos = d.get("eos_token_id", 2)
        if isinstance(eos, list):
            eos = eos[0]
        return ModelConfig(
            architecture=arch,
            vocab_size=int(d.get("vocab_size", 32000)),
            hidden_size=hs,
            intermediate_size=int(d.get("intermediate_size", 4 * hs)),
            num_hidden_layers=int(d.get("num_hidden_layers", 32)),
            num_attention_heads=nh,
            num_key_value_heads=int(d.get("num_key_value_heads", nh)),
            head_dim=int(d.get("head_dim") or hs // nh),
            rms_norm_eps=float(d.get("rms_norm_eps", 1e-5)),
            rope_theta=float(d.get("rope_theta", (d.get("rope_parameters") or {}).get("rope_theta", 10000.0))),
            rope_scaling=RopeScaling.from_hf(d.get("rope_scaling")),
            max_position_embeddings=int(d.get("max_position_embeddings", 8192)),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            num_local_experts=int(d.get("num_local_experts", 0) or 0),
            num_experts_per_tok=int(d.get("num_experts_per_tok", 0) or 0),
            attention_bias=bool(d.get("attention_bias", False)),
            bos_token_id=int(d.get("bos_token_id", 1) or 1),
            eos_token_id=int(eos if eos is not None else 2),
        )

    def to_hf(self) -> dict:
        d = {
            "architectures": ["MixtralForCausalLM" if self.is_moe else "LlamaForCausalLM"],
            "model_type": "mixtral" if self.is_moe else "llama",
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
            "hidden_act": "silu",
            "torch_dtype": "bfloat16",
        }
        if self.rope_scaling.kind != "none":
            rs = self.rope_scaling
            d["rope_scaling"] = {"rope_type": rs.kind, "factor": rs.factor,
                                 "low_freq_factor": rs.low_freq_factor,
                                 "high_freq_factor": rs.high_freq_factor,
                                 "original_max_position_embeddings": rs.original_max_position_embeddings}
        if self.is_moe:
            d["num_local_experts"] = self.num_local_experts
            d["num_experts_per_tok"] = self.num_experts_per_tok
        return d


# Named architectures used by tests and benchmarks (random-init weights; shapes only).
PRESETS: dict[str, ModelConfig] = {
    "tiny-llama": ModelConfig(
        architecture="llama", vocab_size=32000, hidden_size=256, intermediate_size=688,
        num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
        rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=2048),
    "tiny-mixtral": ModelConfig(
        architecture="mixtral", vocab_size=1024, hidden_size=256, intermediate_size=512,
        num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
        rope_theta=10000.0, num_local_experts=8, num_experts_per_tok=2, max_position_embeddings=2048),
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
    "mixtral-8x7b": ModelConfig(
        architecture="mixtral", vocab_size=32000, hidden_size=4096, intermediate_size=14336,
        num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
        rms_norm_eps=1e-5, rope_theta=1000000.0, num_local_experts=8, num_experts_per_tok=2,
        max_position_embeddings=32768),
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
    quantization: str = "none"                # none | fp8 | gguf
    device: str = "cuda"
    tensor_parallel_size: int = 1
    enable_expert_parallel: bool = False  # MoE: experts partitioned over the TP ranks (EP = TP size)
    expert_parallel_size: int = 1
    # paged KV cache
    block_size: int = 16
    num_gpu_blocks: Optional[int] = None      # None => size from memory fraction
    gpu_memory_utilization: float = 0.85
    kv_cache_dtype: str = "auto"              # auto (= model dtype) | fp8
    enable_prefix_caching: bool = True
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
