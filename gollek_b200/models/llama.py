"""Serving graph of the decoder families: Llama-2/3, Mistral, Mixtral (top-k MoE), Qwen2/3,
Gemma 1/2/3 and Phi-3 (their differences are ModelConfig switches; see ``config.FAMILIES``).

One instance runs on one GPU (one process per GPU); under tensor parallelism it holds the
rank's Megatron-style shard: QKV and gate/up column-parallel (whole heads / FFN slices),
o_proj and down_proj row-parallel followed by an all-reduce, lm_head vocab-parallel
followed by an all-gather; embedding and norms replicated. Weights are fused at load time:
``w_qkv = [q; k; v]`` rows and ``w_gate_up`` = gate/up rows interleaved in groups of 64 so
the GEMM's SwiGLU epilogue emits ``silu(gate) * up`` directly.

Per layer (decode or mixed chunked-prefill step):
  fused_add_rms_norm → GEMM(qkv) → rope_kv_write (RoPE + paged KV write) →
  paged attention (decode kernel for the q_len = 1 sequences, prefill kernel for the rest) →
  GEMM(o) [→ all-reduce] → fused_add_rms_norm → GEMM(gate_up, SwiGLU) → GEMM(down) [→ all-reduce]

Replaces the reference's per-layer flow (kernel/cuda/gollek-kernel-cuda/…/cuda/runner/
CudaRunner.java:475-569 and runner/safetensor/gollek-safetensor-engine/…/engine/forward/
DirectForwardPass.java:221-321) and its MoE loop (…/generation/moe/MoeForwardPass.java:39-128).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import numpy as np
import torch

from .. import ops
from ..config import ModelConfig
from ..utils import tracing
from .reference import layer_tensors, rope_cos_sin

# head sizes the attention kernels are built for; other sizes are stored zero-padded to the next one
_KERNEL_HEAD_DIMS = (32, 64, 128, 256)
# per-layer dense linear weights (quantized by ``quantize_fp8`` / ``quantize_int4``)
_DENSE_KEYS = ("w_qkv", "w_o", "w_gate_up", "w_down", "w_qa_kva", "w_q", "w_q_b", "w_kv_b", "w_sh_gu", "w_sh_down")


@dataclass
class AttnMetadata:
    """Per-step batch description built by the model runner.

    Tokens are ordered: the ``num_decode`` single-token (decode) sequences first, then the
    prefill / chunked-prefill sequences.
    """
    positions: torch.Tensor            # [T] int32
    slot_mapping: torch.Tensor         # [T] int32
    num_decode: int
    decode_block_tables: Optional[torch.Tensor] = None   # [nd, max_blocks] int32
    decode_seq_lens: Optional[torch.Tensor] = None       # [nd] int32
    decode_splits: int = 1
    decode_workspace: Optional[torch.Tensor] = None
    num_prefill_tokens: int = 0
    prefill_block_tables: Optional[torch.Tensor] = None  # [np, max_blocks] int32
    prefill_seq_lens: Optional[torch.Tensor] = None      # [np] int32
    prefill_query_start: Optional[torch.Tensor] = None   # [np + 1] int32 (relative)
    prefill_tiles: Optional[torch.Tensor] = None         # ops.prefill_schedule work list (int32)
    logits_indices: Optional[torch.Tensor] = None        # [B_out] int64 rows for the lm_head
    # hybrid GDN models: per sequence (batch order) its recurrent-state slot, whether the step starts
    # it from the zero state, and the token offsets of all sequences
    gdn_slots: Optional[torch.Tensor] = None             # [n] int32
    gdn_reset: Optional[torch.Tensor] = None             # [n] int32
    gdn_query_start: Optional[torch.Tensor] = None       # [n + 1] int32
    # split batch (tensor-parallel overlap): (rows of the first half, metadata of each half); each
    # half's collectives run while the other half computes
    halves: Optional[tuple] = None
    # multimodal prompts: batch rows whose embedding is replaced by projected image rows
    mm_rows: Optional[torch.Tensor] = None                # [k] int64
    mm_embeds: Optional[torch.Tensor] = None              # [k, hidden]

    @property
    def num_tokens(self) -> int:
        return self.num_decode + self.num_prefill_tokens


class TPComm:
    """Collectives used by the model under tensor parallelism (no-ops at tp_size 1).

    ``allreduce_add_rmsnorm`` is the one collective on the layer path: it follows each
    row-parallel GEMM (o_proj, down_proj) and folds in the residual add and the next RMSNorm.
    Implementations: this base class (single GPU), ``parallel.dist.NcclComm`` (NCCL all-reduce +
    the fused norm kernel; the baseline) and ``parallel.symm.FusedTPComm`` (one P2P kernel).
    """

    fused_ar = False

    def __init__(self, rank: int = 0, size: int = 1):
        self.rank, self.size = rank, size

    def partial_buffer(self, T: int) -> Optional[torch.Tensor]:
        """Where the next row-parallel GEMM should write its partial output (None = allocate)."""
        return None

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        return t

    def residual_rows(self, T: int) -> slice:
        """Rows of the residual stream that ``allreduce_add_rmsnorm`` keeps up to date on this rank
        (all of them, unless the implementation shards the residual by rows)."""
        return slice(0, T)

    # split batches (two halves whose collectives overlap the other half's compute)
    supports_split = False

    def half_partial_buffer(self, half: int, T: int) -> Optional[torch.Tensor]:
        return None

    def gathered_rows(self, T: int) -> Optional[torch.Tensor]:
        return None

    def allreduce_add_rmsnorm_half(self, half: int, row0: int, h: torch.Tensor, residual: torch.Tensor,
                                   w: torch.Tensor, eps: float) -> torch.Tensor:
        return ops.fused_add_rms_norm(self.all_reduce(h), residual, w, eps)

    def push_linear(self, a: torch.Tensor, w) -> Optional[torch.Tensor]:
        """Row-parallel GEMM fused with the data movement of the all-reduce that follows (the
        fused comm overrides this); None = run ``ops.linear`` into ``partial_buffer``."""
        return None

    def allreduce_add_rmsnorm(self, h: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                              eps: float) -> torch.Tensor:
        return ops.fused_add_rms_norm(self.all_reduce(h), residual, w, eps)

    def all_gather_last(self, t: torch.Tensor) -> torch.Tensor:
        return t

    def reserve_logits(self, v_local: int) -> None:
        """Set up the buffers of the vocab-parallel logits gather (collective where it allocates)."""

    def argmax_last(self, t: torch.Tensor, vocab_offset: int) -> torch.Tensor:
        """Greedy token ids from vocab-parallel logit shards (ties: lowest token id)."""
        return ops.argmax(t)


def _deinterleave_heads(w: torch.Tensor, n_heads: int, d: int) -> torch.Tensor:
    """Reorder each head's rows to (0, 2, 4, ..., 1, 3, 5, ...): RoPE on interleaved pairs
    (2i, 2i+1) of the original rows is rotate-half RoPE on pairs (i, i + d/2) of the reordered ones,
    and q . k is unchanged when q and k are reordered alike."""
    perm = torch.cat([torch.arange(0, d, 2), torch.arange(1, d, 2)]).to(w.device)
    return w.reshape(n_heads, d, *w.shape[1:]).index_select(1, perm).reshape(w.shape)


def _pad_heads(w: torch.Tensor, n_heads: int, d: int, d_pad: int, dim: int = 0) -> torch.Tensor:
    """Zero-pad each of ``n_heads`` head blocks of width ``d`` along ``dim`` to ``d_pad``."""
    if d == d_pad:
        return w
    if dim == 0:
        v = w.reshape(n_heads, d, *w.shape[1:])
        out = torch.zeros(n_heads, d_pad, *w.shape[1:], dtype=w.dtype, device=w.device)
        out[:, :d] = v
        return out.reshape(n_heads * d_pad, *w.shape[1:])
    v = w.reshape(w.shape[0], n_heads, d)
    out = torch.zeros(w.shape[0], n_heads, d_pad, dtype=w.dtype, device=w.device)
    out[:, :, :d] = v
    return out.reshape(w.shape[0], n_heads * d_pad)


def _pad_rows(w: torch.Tensor, rows: int) -> torch.Tensor:
    if w.shape[0] == rows:
        return w
    out = torch.zeros(rows, *w.shape[1:], dtype=w.dtype, device=w.device)
    out[: w.shape[0]] = w
    return out


def _pad_cols(w: torch.Tensor, cols: int) -> torch.Tensor:
    if w.shape[1] == cols:
        return w
    out = torch.zeros(w.shape[0], cols, dtype=w.dtype, device=w.device)
    out[:, : w.shape[1]] = w
    return out


def _copy_out(y: torch.Tensor, out: Optional[torch.Tensor]) -> torch.Tensor:
    if out is None:
        return y
    out.copy_(y)
    return out


class LlamaModel:
    """Llama / Mixtral decoder for serving (one TP rank)."""

    def __init__(self, cfg: ModelConfig, device: str = "cuda", dtype: torch.dtype = torch.bfloat16,
                 comm: Optional[TPComm] = None, expert_parallel: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.comm = comm or TPComm()
        tp, r = self.comm.size, self.comm.rank
        if cfg.num_attention_heads % tp:
            raise ValueError("num_attention_heads must be divisible by the TP size")
        self.H = cfg.num_attention_heads // tp
        if cfg.num_key_value_heads >= tp:
            if cfg.num_key_value_heads % tp:
                raise ValueError("num_key_value_heads must be divisible by the TP size")
            self.Hk = cfg.num_key_value_heads // tp
            self.kv_head0 = r * self.Hk
        else:  # replicate KV heads across ranks
            self.Hk = 1
            self.kv_head0 = r * cfg.num_key_value_heads // tp
        self.D_logical = cfg.head_dim
        self.D = next((d for d in _KERNEL_HEAD_DIMS if d >= cfg.head_dim), cfg.head_dim)
        if self.D != cfg.head_dim and cfg.qk_norm:
            raise ValueError(f"head_dim {cfg.head_dim} with QK-norm is not supported")
        if cfg.is_mla and (cfg.v_head_dim > self.D or cfg.head_dim > self.D):
            raise ValueError("MLA head dims above 256 are not supported")
        f_shard = cfg.intermediate_size // tp
        if cfg.intermediate_size % tp:
            raise ValueError("intermediate_size must be divisible by the TP size")
        self.F = f_shard
        self.F_pad = (f_shard + ops.SWIGLU_GROUP - 1) // ops.SWIGLU_GROUP * ops.SWIGLU_GROUP
        if cfg.vocab_size % tp:
            raise ValueError("vocab_size must be divisible by the TP size")
        self.V_local = cfg.vocab_size // tp
        # MoE placement. Tensor-parallel experts: every rank holds all experts with their FFN width
        # sharded. Expert parallel: rank r holds experts [r*E/tp, (r+1)*E/tp) at full width. In both
        # cases the activations entering the MoE are replicated (attention is tensor parallel), so the
        # rank's output is a partial sum completed by the all-reduce that follows.
        self.expert_parallel = bool(expert_parallel and cfg.is_moe)
        self.ep_a2a = None  # parallel.ep_a2a.EPAllToAll once enable_ep_all_to_all() succeeded
        self.split_sms = 16  # SMs the GEMMs leave free while a split batch's collective runs
        # fp8 e4m3 KV cache: per (layer, block, K/V, kv head, token) scales [L, NB, 2, Hk, bs] fp32
        self.kv_fp8 = False
        self.kv_scales: Optional[torch.Tensor] = None
        self.E_loc, self.e0, self.moe_F = 0, 0, self.F
        if cfg.is_moe:
            E = cfg.num_local_experts
            if cfg.moe_ffn % tp:
                raise ValueError("the expert FFN width must be divisible by the TP size")
            if self.expert_parallel:
                if E % tp:
                    raise ValueError("num_local_experts must be divisible by the expert-parallel size")
                self.E_loc, self.e0, self.moe_F = E // tp, r * (E // tp), cfg.moe_ffn
            else:
                self.E_loc, self.e0, self.moe_F = E, 0, cfg.moe_ffn // tp
        self.moe_F_pad = (self.moe_F + ops.SWIGLU_GROUP - 1) // ops.SWIGLU_GROUP * ops.SWIGLU_GROUP
        # shared experts (DeepSeek-V3): one dense SwiGLU of n_shared * expert width, sharded like the MLP
        self.sh_F = cfg.n_shared_experts * cfg.moe_ffn // tp if cfg.is_moe else 0
        self.sh_F_pad = (self.sh_F + ops.SWIGLU_GROUP - 1) // ops.SWIGLU_GROUP * ops.SWIGLU_GROUP
        self.scale = cfg.attn_scale
        n_pos = max(cfg.max_position_embeddings, 8192)
        self.cos_sin = rope_cos_sin(cfg, n_pos, device=self.device)
        self.cos_sin_local = (rope_cos_sin(cfg, n_pos, device=self.device, theta=cfg.rope_local_theta)
                              if cfg.rope_local_theta else None)
        self.cos_sin_none = None  # identity rotation (cos 1, sin 0) for layers without positions
        if cfg.rope_sliding_only:
            half = self.cos_sin.shape[1] // 2
            self.cos_sin_none = torch.cat([torch.ones(n_pos, half), torch.zeros(n_pos, half)], 1).to(self.cos_sin)
        self.windows = [cfg.layer_window(i) for i in range(cfg.num_hidden_layers)]
        # hybrid stacks: KV cache rows only for attention layers; GDN layers keep a recurrent state
        # [slots, Hg, 128, 128] fp32 per layer instead
        self.kv_index, self.gdn_index = [], []
        na = ng = 0
        for i in range(cfg.num_hidden_layers):
            g = cfg.is_gdn_layer(i)
            self.kv_index.append(-1 if g else na)
            self.gdn_index.append(ng if g else -1)
            na, ng = na + (not g), ng + g
        self.num_kv_layers, self.num_gdn_layers = na, ng
        self.Hg = 0
        if ng:
            if cfg.gdn_heads % tp:
                raise ValueError("GDN heads must be divisible by the TP size")
            self.Hg = cfg.gdn_heads // tp
        self.gdn_state: Optional[torch.Tensor] = None
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.embed: Optional[torch.Tensor] = None
        self.norm: Optional[torch.Tensor] = None
        self.lm_head: Optional[torch.Tensor] = None
        self.expert_perm: Dict[int, np.ndarray] = {}  # MoE layer -> physical slot -> logical expert (EP)
        self.lora = None  # optional MultiLoRA hook (gollek_b200.engine.lora)
        self.offload = None  # optional LayerOffload (weights of some layers streamed from host memory)

    def enable_offload(self, num_layers: int, depth: int = 2) -> None:
        """Keep the weights of the last ``num_layers`` layers in pinned host memory and stream them
        in ``depth`` layers ahead of use (CUDA only; the engine disables CUDA graphs)."""
        if num_layers <= 0 or self.device.type != "cuda":
            return
        from .offload import LayerOffload
        n = len(self.layers)
        self.offload = LayerOffload(self.layers, list(range(max(0, n - num_layers), n)), self.device, depth)
        torch.cuda.empty_cache()

    # ------------------------------------------------------------------ weights
    def load_weights(self, get: Callable[[str], torch.Tensor]) -> None:
        """Shard and fuse HF-named weights. ``get(name)`` returns a (CPU or GPU) tensor."""
        cfg, tp, r = self.cfg, self.comm.size, self.comm.rank
        H, Hk, D = self.H, self.Hk, self.D
        dev, dt = self.device, self.dtype

        from ..quant import int4 as I4
        from ..quant.gguf_weights import QWeight, cat_rows, interleave_rows
        quantized = (QWeight, I4.Int4Weight)

        def t(name):
            v = get(name)
            if type(v).__name__ == "QuantizedWeight":  # GGUF blocks stay quantized on the device
                return QWeight.from_quantized(v).to(dev)
            if isinstance(v, I4.Int4Weight):  # GPTQ / AWQ / NF4 stay 4-bit on the device
                return v.to(dev)
            return v.to(device=dev, dtype=dt)

        def dense(v):
            if isinstance(v, QWeight):
                return v.dequantize().to(device=dev, dtype=dt)
            if isinstance(v, I4.Int4Weight):
                return v.dequantize(dt).to(dev)
            return v

        def same_format(ws):
            return len({(type(w), getattr(w, "qtype", None), getattr(w, "K", None)) for w in ws}) == 1

        def cat(ws):
            if not same_format(ws):  # e.g. a GGUF mixture with a Q6_K v_proj beside Q4_K q/k: dense
                return torch.cat([dense(w) for w in ws], 0)
            if isinstance(ws[0], I4.Int4Weight):
                return I4.cat_rows(ws)
            return cat_rows(ws) if isinstance(ws[0], QWeight) else torch.cat(ws, 0)

        def gate_up(g, u, fpad=None):
            fpad = self.F_pad if fpad is None else fpad
            if not same_format([g, u]):
                g, u = dense(g), dense(u)
            if isinstance(g, quantized):
                if fpad != g.N:
                    raise ValueError("quantized FFN width must be a multiple of 64 per TP rank")
                return I4.interleave_rows(g, u) if isinstance(g, I4.Int4Weight) else interleave_rows(g, u)
            return ops.interleave_gate_up(_pad_rows(g, fpad), _pad_rows(u, fpad))

        def down(d, fpad=None):
            return d if isinstance(d, quantized) else _pad_cols(d, self.F_pad if fpad is None else fpad)

        Dl = self.D_logical

        def norm_w(x):
            # Gemma's RMSNorm scales by (1 + w): folded here so every norm kernel multiplies by w
            if cfg.norm_unit_offset:
                return (x.float() + 1.0).to(dt).contiguous()
            return x.contiguous()

        def ffn(L, c, p, i):
            if cfg.is_moe_layer(i):
                ds = cfg.moe_scoring == "sigmoid"  # DeepSeek-V3 names (mlp.*), else Mixtral's
                pe = p + ("mlp." if ds else "block_sparse_moe.")
                names = ("gate_proj", "up_proj", "down_proj") if ds else ("w1", "w3", "w2")
                L["router"] = t(pe + "gate.weight").contiguous()
                if ds:
                    L["router_bias"] = get(pe + "gate.e_score_correction_bias").to(dev, torch.float32).contiguous()
                    if cfg.n_shared_experts:
                        s0, s1 = r * self.sh_F, (r + 1) * self.sh_F
                        ps = pe + "shared_experts."
                        L["w_sh_gu"] = gate_up(t(ps + "gate_proj.weight")[s0:s1], t(ps + "up_proj.weight")[s0:s1],
                                               self.sh_F_pad).contiguous()
                        L["w_sh_down"] = down(t(ps + "down_proj.weight")[:, s0:s1], self.sh_F_pad).contiguous()
                experts = []
                f0, f1 = (0, self.moe_F) if self.expert_parallel else (r * self.moe_F, (r + 1) * self.moe_F)
                for e in range(self.e0, self.e0 + self.E_loc):
                    g = t(pe + f"experts.{e}.{names[0]}.weight")[f0:f1]
                    u = t(pe + f"experts.{e}.{names[1]}.weight")[f0:f1]
                    d = t(pe + f"experts.{e}.{names[2]}.weight")[:, f0:f1]
                    experts.append((gate_up(g, u, self.moe_F_pad).contiguous(),
                                    down(d, self.moe_F_pad).contiguous()))
                if all(isinstance(a, torch.Tensor) for a, _ in experts):
                    # dense experts stacked for the grouped GEMMs
                    L["moe_gu"] = torch.cat([a for a, _ in experts], 0)
                    L["moe_down"] = torch.cat([b for _, b in experts], 0)
                    del experts
                else:
                    L["experts"] = experts
            else:
                g = c["gate"][r * self.F:(r + 1) * self.F]
                u = c["up"][r * self.F:(r + 1) * self.F]
                d = c["down"][:, r * self.F:(r + 1) * self.F]
                L["w_gate_up"] = gate_up(g, u).contiguous()
                L["w_down"] = down(d).contiguous()

        self.embed = t("model.embed_tokens.weight").contiguous()
        self.norm = norm_w(t("model.norm.weight"))
        if cfg.logit_scale != 1.0:  # logits = norm(h) @ E^T * s: the scale folds into the final norm
            self.norm = (self.norm.float() * cfg.logit_scale).to(dt).contiguous()
        head_name = "model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"
        self.lm_head = t(head_name)[r * self.V_local:(r + 1) * self.V_local].contiguous()
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}."
            c = layer_tensors(t, cfg, i)
            if c.get("gdn") or cfg.is_mla:
                L = self._gdn_weights(c, norm_w) if c.get("gdn") else self._mla_weights(c, norm_w)
                ffn(L, c, p, i)
                self.layers.append(L)
                continue
            kv0, kv1 = self.kv_head0 * Dl, (self.kv_head0 + Hk) * Dl
            cq, ck = c["q"][r * H * Dl:(r + 1) * H * Dl], c["k"][kv0:kv1]
            if cfg.rope_interleaved:  # pairs (2i, 2i+1) -> (i, i + D/2): the NeoX kernel rotates them
                cq, ck = _deinterleave_heads(cq, H, Dl), _deinterleave_heads(ck, Hk, Dl)
            q = _pad_heads(cq, H, Dl, D)
            k = _pad_heads(ck, Hk, Dl, D)
            v = _pad_heads(c["v"][kv0:kv1], Hk, Dl, D)
            o = _pad_heads(c["o"][:, r * H * Dl:(r + 1) * H * Dl], H, Dl, D, dim=1)
            L = {
                "in_norm": norm_w(c["in_norm"]),
                "post_norm": norm_w(c["post_norm"]) if c["post_norm"] is not None else None,
                "w_qkv": cat([q, k, v]).contiguous(),
                "w_o": o.contiguous(),
            }
            if cfg.attention_bias:
                L["qkv_bias"] = torch.cat([_pad_heads(c["q_bias"][r * H * Dl:(r + 1) * H * Dl], H, Dl, D),
                                           _pad_heads(c["k_bias"][kv0:kv1], Hk, Dl, D),
                                           _pad_heads(c["v_bias"][kv0:kv1], Hk, Dl, D)]).contiguous()
            if cfg.qk_norm:
                L["q_norm"], L["k_norm"] = norm_w(c["q_norm"]), norm_w(c["k_norm"])
            if cfg.sandwich_norm:
                L["pre_ff_norm"], L["post_ff_norm"] = norm_w(c["pre_ff_norm"]), norm_w(c["post_ff_norm"])
            ffn(L, c, p, i)
            self.layers.append(L)

    def _gdn_weights(self, c: dict, norm_w) -> Dict[str, torch.Tensor]:
        """GDN layer: one fused input projection [q | k | v | g | a | b] of this rank's heads (rows
        padded to 128), the row-parallel output projection and the fp32 gate parameters."""
        r, Hg, GD = self.comm.rank, self.Hg, 128
        sl, hs = slice(r * Hg * GD, (r + 1) * Hg * GD), slice(r * Hg, (r + 1) * Hg)
        w_in = torch.cat([c["gq"][sl], c["gk"][sl], c["gv"][sl], c["gg"][sl], c["ga"][hs], c["gb"][hs]], 0)
        rows = (w_in.shape[0] + 127) // 128 * 128
        return {"gdn": True, "in_norm": norm_w(c["in_norm"]), "post_norm": norm_w(c["post_norm"]),
                "w_gdn_in": _pad_rows(w_in, rows).contiguous(), "w_o": c["o"][:, sl].contiguous(),
                "A_log": c["A_log"][hs].float().contiguous(), "dt_bias": c["dt_bias"][hs].float().contiguous(),
                "gdn_norm": c["gnorm"].contiguous()}

    def _mla_weights(self, c: dict, norm_w) -> Dict[str, torch.Tensor]:
        """Multi-head latent attention, decompressed into this rank's heads of the paged cache.

        Each head of q and k is laid out [rope (qk_rope) | nope (qk_nope) | 0] and padded to the
        kernel head size D, each v head [v | 0], so the fused RoPE + KV-write kernel rotates the
        first qk_rope dims (its partial-rotary mode) and the attention kernels run unchanged.
        Interleaved rope pairs are de-interleaved in the weight rows (NeoX rotation then gives
        the same scores). The latent projection ``w_qa_kva`` = [q_a ; kv_a] runs once per token
        (replicated over ranks); ``w_kv_b`` takes [norm(c) | k_rope] and carries k_rope into
        every key head through an identity block, so one GEMM writes the whole k and v of the
        rank's heads."""
        cfg, r, H, D = self.cfg, self.comm.rank, self.H, self.D
        nope, rd, vd, kvl = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
        for k in ("q_a", "q_b", "q", "kv_a", "kv_b", "o"):
            if k in c and not isinstance(c[k], torch.Tensor):
                raise ValueError("MLA layers need bf16 / fp16 / fp32 checkpoint weights")

        def deint(x):  # rows (2i, 2i+1) -> (i, rd/2 + i) along dim -2
            return torch.cat([x[..., 0::2, :], x[..., 1::2, :]], -2) if cfg.rope_interleaved else x

        def q_heads(wq):  # [nh * (nope + rd), K] -> [H * D, K]: this rank's heads, [rope | nope | 0]
            K = wq.shape[1]
            w = wq.view(-1, nope + rd, K)[r * H:(r + 1) * H]
            out = torch.zeros(H, D, K, dtype=wq.dtype, device=wq.device)
            out[:, :rd] = deint(w[:, nope:])
            out[:, rd:rd + nope] = w[:, :nope]
            return out.view(H * D, K)

        kv_a = c["kv_a"]
        kv_a = torch.cat([kv_a[:kvl], deint(kv_a[kvl:])], 0)
        kvb = c["kv_b"].view(-1, nope + vd, kvl)[r * H:(r + 1) * H]
        wk = torch.zeros(H, D, kvl + rd, dtype=kvb.dtype, device=kvb.device)
        wk[:, :rd, kvl:] = torch.eye(rd, dtype=kvb.dtype, device=kvb.device)
        wk[:, rd:rd + nope, :kvl] = kvb[:, :nope]
        wv = torch.zeros(H, D, kvl + rd, dtype=kvb.dtype, device=kvb.device)
        wv[:, :vd, :kvl] = kvb[:, nope:]
        L = {"mla": True, "in_norm": norm_w(c["in_norm"]), "post_norm": norm_w(c["post_norm"]),
             "kv_a_norm": c["kv_a_norm"].contiguous(),
             "w_kv_b": torch.cat([wk.view(H * D, -1), wv.view(H * D, -1)], 0).contiguous(),
             "w_o": _pad_heads(c["o"][:, r * H * vd:(r + 1) * H * vd], H, vd, D, dim=1).contiguous()}
        if cfg.q_lora_rank:
            L["w_qa_kva"] = torch.cat([c["q_a"], kv_a], 0).contiguous()
            L["q_a_norm"] = c["q_a_norm"].contiguous()
            L["w_q_b"] = q_heads(c["q_b"]).contiguous()
        else:
            L["w_qa_kva"] = kv_a.contiguous()
            L["w_q"] = q_heads(c["q"]).contiguous()
        return L

    def init_random(self, seed: int = 0, std: float = 0.02, fp8: bool = False) -> None:
        """Random-init this rank's shard directly on the device (benchmarks; no checkpoint)."""
        cfg = self.cfg
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1000 + self.comm.rank)
        dev, dt = self.device, self.dtype

        def rnd(*shape):
            x = torch.empty(*shape, dtype=dt, device=dev)
            x.normal_(0.0, std, generator=g)
            return x

        h = cfg.hidden_size
        Dl, D = self.D_logical, self.D
        ones = lambda n: torch.ones(n, dtype=dt, device=dev)  # noqa: E731
        self.embed = rnd(cfg.vocab_size, h)
        self.norm = ones(h)
        self.lm_head = rnd(self.V_local, h)
        self.layers = []
        for li in range(cfg.num_hidden_layers):
            if cfg.is_mla:
                H, D, kvl, rd = self.H, self.D, cfg.kv_lora_rank, cfg.qk_rope_head_dim
                L = {"mla": True, "in_norm": ones(h), "post_norm": ones(h), "kv_a_norm": ones(kvl),
                     "w_qa_kva": rnd(cfg.q_lora_rank + kvl + rd, h), "w_kv_b": rnd(2 * H * D, kvl + rd),
                     "w_o": rnd(h, H * D)}
                if cfg.q_lora_rank:
                    L["q_a_norm"], L["w_q_b"] = ones(cfg.q_lora_rank), rnd(H * D, cfg.q_lora_rank)
                else:
                    L["w_q"] = rnd(H * D, h)
            elif cfg.is_gdn_layer(li):
                hd = self.Hg * 128
                rows = (4 * hd + 2 * self.Hg + 127) // 128 * 128
                L = {"gdn": True, "in_norm": ones(h), "post_norm": ones(h), "w_gdn_in": rnd(rows, h),
                     "w_o": rnd(h, hd), "A_log": torch.full((self.Hg,), 1.0, device=dev),
                     "dt_bias": torch.zeros(self.Hg, device=dev), "gdn_norm": ones(128)}
            else:
                L = {
                    "in_norm": ones(h),
                    "post_norm": ones(h),
                    "w_qkv": _pad_heads(rnd((self.H + 2 * self.Hk) * Dl, h), self.H + 2 * self.Hk, Dl, D),
                    "w_o": _pad_heads(rnd(h, self.H * Dl), self.H, Dl, D, dim=1),
                }
            if cfg.attention_bias and "w_qkv" in L:
                L["qkv_bias"] = _pad_heads(rnd((self.H + 2 * self.Hk) * Dl), self.H + 2 * self.Hk, Dl, D)
            if cfg.qk_norm and "w_qkv" in L:
                L["q_norm"], L["k_norm"] = ones(D), ones(D)
            if cfg.sandwich_norm:
                L["pre_ff_norm"], L["post_ff_norm"] = ones(h), ones(h)
            if cfg.is_moe_layer(li):
                L["router"] = rnd(cfg.num_local_experts, h)
                if cfg.moe_scoring == "sigmoid":
                    L["router_bias"] = torch.zeros(cfg.num_local_experts, dtype=torch.float32, device=dev)
                if self.sh_F:
                    L["w_sh_gu"], L["w_sh_down"] = rnd(2 * self.sh_F_pad, h), rnd(h, self.sh_F_pad)
                fp = self.moe_F_pad
                if fp8:
                    L["experts"] = [(rnd(2 * fp, h), rnd(h, fp)) for _ in range(self.E_loc)]
                else:
                    L["moe_gu"] = rnd(self.E_loc * 2 * fp, h)
                    L["moe_down"] = rnd(self.E_loc * h, fp)
            else:
                L["w_gate_up"] = rnd(2 * self.F_pad, h)
                L["w_down"] = rnd(h, self.F_pad)
            if fp8:  # quantise this layer now so bf16 copies of all layers never coexist
                from ..quant.fp8 import quantize_weight
                for k in _DENSE_KEYS:
                    if k in L and L[k].shape[1] % 128 == 0:
                        L[k] = quantize_weight(L[k])
                if "experts" in L:
                    L["experts"] = [(quantize_weight(a), quantize_weight(b)) for a, b in L["experts"]]
            self.layers.append(L)

    def quantize_int4(self, kind: str = "int4", group: int = 128) -> None:
        """Quantize the dense linear weights (qkv, o, gate/up, down) to 4 bits at load: ``int4`` =
        round-to-nearest asymmetric int4 per ``group`` columns, ``nf4`` = NF4 with 64-column absmax
        blocks. Per-row quantization, so the fused/interleaved row layouts are unaffected."""
        from ..quant.int4 import quantize_nf4, quantize_rtn
        for L in self.layers:
            for k in _DENSE_KEYS:
                v = L.get(k)
                if isinstance(v, torch.Tensor):
                    K = v.shape[1]
                    g = next(x for x in (group, 128, 64, 32) if K % x == 0) if K % 32 == 0 else None
                    if g is None:
                        raise ValueError(f"4-bit quantization needs K divisible by 32 (got {K})")
                    L[k] = quantize_nf4(v, min(64, g)) if kind == "nf4" else quantize_rtn(v, g)
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def quantize_int8(self) -> None:
        """Weight-only int8: the dense linear weights become Q8_0 blocks (32 int8 values with one fp16
        scale, symmetric round-to-nearest), served by the Q8_0 dequant-fused GEMV for small batches
        and by in-L2 dequant + tcgen05 GEMM for large ones. Quantized on the host, layer by layer."""
        from ..native import host_ext
        from ..quant.gguf_weights import GGML_Q8_0, QWeight
        h = host_ext()
        for L in self.layers:
            for k in _DENSE_KEYS:
                v = L.get(k)
                if isinstance(v, torch.Tensor) and v.shape[1] % 32 == 0:
                    raw = h.quantize_q8_0(v.float().cpu().reshape(-1).contiguous())
                    L[k] = QWeight(raw.to(v.device), v.shape[0], v.shape[1], GGML_Q8_0)
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def quantize_fp8(self) -> None:
        """Convert the linear weights (qkv, o, gate/up, down; experts too) to block-scaled FP8, layer by
        layer so the bf16 copies are released as it goes. Embedding, norms and lm_head stay bf16."""
        from ..quant.fp8 import quantize_weight
        for L in self.layers:
            for k in _DENSE_KEYS:  # weights whose K is not a multiple of 128 stay bf16
                if k in L and isinstance(L[k], torch.Tensor) and L[k].shape[1] % 128 == 0:
                    L[k] = quantize_weight(L[k])
            if "moe_gu" in L:
                fp, h = self.moe_F_pad, self.cfg.hidden_size
                gu, dn = L.pop("moe_gu"), L.pop("moe_down")
                L["experts"] = [(gu[e * 2 * fp:(e + 1) * 2 * fp], dn[e * h:(e + 1) * h]) for e in range(self.E_loc)]
                del gu, dn
            if "experts" in L:
                L["experts"] = [(quantize_weight(a), quantize_weight(b)) for a, b in L["experts"]]
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def weight_bytes(self) -> int:
        def nb(x):
            return x.nbytes() if hasattr(x, "nbytes") and callable(x.nbytes) else x.numel() * x.element_size()

        n = sum(nb(x) for x in (self.embed, self.norm, self.lm_head))
        for L in self.layers:
            for k, v in L.items():
                if v is None or isinstance(v, (bool, int, float)):  # offloaded (host memory) or a layer flag
                    continue
                if k == "experts":
                    n += sum(nb(a) + nb(b) for a, b in v)
                else:
                    n += nb(v)
        if self.offload is not None:
            n += sum(nb(t) for slot in self.offload.slots for t in slot.values())
        return n

    # ------------------------------------------------------------------ KV cache
    def kv_cache_shape(self, num_blocks: int, block_size: int = 16) -> tuple:
        return (max(1, self.num_kv_layers), num_blocks, 2, self.Hk, block_size, self.D)

    def kv_bytes_per_block(self, block_size: int = 16) -> int:
        if self.kv_fp8:  # one byte per value + an fp32 scale per token and head
            return max(1, self.num_kv_layers) * 2 * self.Hk * block_size * (self.D + 4)
        return max(1, self.num_kv_layers) * 2 * self.Hk * block_size * self.D * torch.finfo(self.dtype).bits // 8

    def _kv_scales(self, li: int) -> Optional[torch.Tensor]:
        return self.kv_scales[self.kv_index[li]] if self.kv_scales is not None else None

    def gdn_state_bytes(self, num_slots: int) -> int:
        return self.num_gdn_layers * num_slots * self.Hg * 128 * 128 * 4

    def alloc_gdn_state(self, num_slots: int) -> None:
        """Recurrent states of the GDN layers: [gdn_layers, slots, Hg, 128, 128] fp32."""
        if self.num_gdn_layers:
            self.gdn_state = torch.zeros(self.num_gdn_layers, num_slots, self.Hg, 128, 128, dtype=torch.float32,
                                         device=self.device)

    # ------------------------------------------------------------------ forward
    def _attention(self, q: torch.Tensor, cache: torch.Tensor, meta: AttnMetadata, window: int = 0,
                   kv_scales: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = torch.empty_like(q)
        nd = meta.num_decode
        cap = self.cfg.attn_logit_softcapping
        if nd > 0:
            ops.paged_decode_attention(q[:nd], cache, meta.decode_block_tables, meta.decode_seq_lens, self.scale,
                                       meta.decode_splits, out=out[:nd], workspace=meta.decode_workspace,
                                       window=window, softcap=cap, kv_scales=kv_scales)
        if meta.num_prefill_tokens > 0:
            ops.paged_prefill_attention(q[nd:], cache, meta.prefill_block_tables, meta.prefill_seq_lens,
                                        meta.prefill_query_start, self.scale, tiles=meta.prefill_tiles,
                                        out=out[nd:], window=window, softcap=cap, kv_scales=kv_scales)
        return out

    def _row_linear(self, a: torch.Tensor, w, li: int, lora_kind: Optional[str] = None) -> torch.Tensor:
        """o_proj / down_proj (row-parallel): under the fused TP comm the GEMM pushes its tiles to
        every rank as it produces them; otherwise it writes the rank's partial for the collective."""
        if self.lora is None and not self.cfg.sandwich_norm:
            h = self.comm.push_linear(a, w)
            if h is not None:
                return h
        h = ops.linear(a, w, out=self.comm.partial_buffer(a.shape[0]))
        if self.lora is not None and lora_kind is not None:
            self.lora.apply(li, lora_kind, a, h)
        return h

    def _route(self, L: dict) -> dict:
        cfg = self.cfg
        if cfg.moe_scoring == "softmax":
            return {}
        return dict(scoring=cfg.moe_scoring, bias=L.get("router_bias"), n_group=cfg.n_group,
                    topk_group=cfg.topk_group, scale=cfg.routed_scaling_factor)

    def _moe(self, x: torch.Tensor, L: dict, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """This rank's share of the MoE FFN (its local experts, or its FFN shard of every expert),
        plus its shard of the shared experts when the family has them."""
        cfg = self.cfg
        if "w_sh_gu" in L:  # routed experts into a temporary, the shared expert's GEMM adds them
            hm = self._moe(x, {k: v for k, v in L.items() if k not in ("w_sh_gu", "w_sh_down")})
            return ops.linear(ops.linear_swiglu(x, L["w_sh_gu"]), L["w_sh_down"], residual=hm, out=out)
        renorm = cfg.norm_topk_prob
        if "moe_gu" in L:  # dense experts: route + permute + grouped tcgen05 GEMMs + combine
            rt = {} if "expert_load" in L else None
            y = ops.fused_moe(x, L["router"], L["moe_gu"], L["moe_down"], cfg.num_experts_per_tok,
                              self.e0, self.E_loc, renorm=renorm, out=out, routing=rt,
                              expert_map=L.get("expert_map"), **self._route(L))
            if rt is not None:  # per-expert token counts for the rebalancer (physical expert ids)
                ids = rt["ids"].reshape(-1).long()
                L["expert_load"].index_add_(0, ids, torch.ones(ids.shape[0], dtype=torch.float32, device=ids.device))
            return y
        # quantized experts (GGUF / FP8): one expert at a time
        topi, topw = ops.moe_route_ref(x, L["router"], cfg.num_experts_per_tok, renorm, **self._route(L))
        topw = topw.to(x.device)
        topi = topi.to(x.device)
        acc = torch.zeros(x.shape[0], cfg.hidden_size, dtype=torch.float32, device=x.device)
        for le, (w_gu, w_d) in enumerate(L["experts"]):
            e = self.e0 + le
            sel = (topi == e)
            rows = sel.any(-1).nonzero().flatten()
            if rows.numel() == 0:
                continue
            xe = x.index_select(0, rows).contiguous()
            ye = ops.linear(ops.linear_swiglu(xe, w_gu), w_d).float()
            we = (topw * sel).sum(-1).index_select(0, rows)
            acc.index_add_(0, rows, ye * we[:, None])
        return _copy_out(acc.to(x.dtype), out)

    # ------------------------------------------------------------------ expert-parallel rebalancing
    def enable_expert_load_tracking(self) -> None:
        """Count the tokens routed to each expert of every MoE layer (one small add per layer and
        step) so that ``rebalance_experts`` can move hot experts apart."""
        for L in self.layers:
            if "moe_gu" in L and "expert_load" not in L:
                L["expert_load"] = torch.zeros(self.cfg.num_local_experts, dtype=torch.float32, device=self.device)
            if "moe_gu" in L and "expert_map" not in L:  # created before any graph capture, updated in place
                L["expert_map"] = torch.arange(self.cfg.num_local_experts, dtype=torch.int32, device=self.device)

    def rebalance_experts(self, min_gain: float = 0.05, loads: Optional[Dict[int, np.ndarray]] = None) -> Dict[int, dict]:
        """Re-place the experts of each MoE layer over the expert-parallel ranks so that the ranks'
        routed-token loads even out (``parallel.ep_balance``). Collective: every rank calls it at
        the same point between steps. ``loads`` (logical expert -> tokens, per layer) overrides the
        tracked counters. A layer moves only when its max/mean rank load drops by ``min_gain``.
        Routing stays over the logical experts (router rows never move, so group-limited routing and
        tie-breaking are unchanged); the layer's logical -> physical expert map and the expert
        weights are rewritten in place (same device addresses, so captured CUDA graphs stay valid);
        returns {layer: {"before", "after", "moved"}}."""
        from ..parallel.ep_balance import imbalance, moves, plan_placement
        if not self.expert_parallel:
            return {}
        world = self.comm.size
        E = self.cfg.num_local_experts
        report = {}
        for li, L in enumerate(self.layers):
            if "moe_gu" not in L:
                continue
            perm = self.expert_perm.setdefault(li, np.arange(E))
            if loads is not None and li in loads:
                logical = np.asarray(loads[li], dtype=np.float64)
            elif "expert_load" in L:
                phys = L["expert_load"].double().cpu()
                if world > 1 and torch.distributed.is_initialized():  # every rank takes the same decision
                    t = phys.to(self.device) if torch.distributed.get_backend() == "nccl" else phys
                    torch.distributed.all_reduce(t)
                    phys = t.cpu() / world
                logical = np.zeros(E)
                logical[perm] = phys.numpy()
                L["expert_load"].zero_()
            else:
                continue
            before = imbalance(logical, perm, world)
            new = plan_placement(logical, perm, world)
            after = imbalance(logical, new, world)
            if after > before * (1.0 - min_gain):
                continue
            self._move_experts(L, perm, new)
            self.expert_perm[li] = new
            report[li] = {"before": before, "after": after, "moved": len(moves(perm, new, world))}
        return report

    def enable_ep_all_to_all(self, max_tokens: int) -> bool:
        """Switch the MoE layers to token-sharded expert parallelism over the NVLink all-to-all
        (parallel.ep_a2a). Needs expert parallelism, dense stacked experts without shared experts,
        RMSNorm pre-norm blocks and a TP comm with NVLS; the residual stream then stays sharded by
        rows in every layer. Collective: every rank calls it. Returns whether it is on."""
        cfg, comm = self.cfg, self.comm
        ok = (self.expert_parallel and comm.size > 1 and getattr(comm, "nvls", False)
              and not cfg.sandwich_norm and not cfg.parallel_block and not cfg.norm_center
              and self.lora is None and cfg.moe_scoring == "softmax"
              and all("moe_gu" in L and "w_sh_gu" not in L for li, L in enumerate(self.layers)
                      if cfg.is_moe_layer(li)))
        if not ok:
            return False
        from ..parallel.ep_a2a import EPAllToAll
        self.ep_a2a = EPAllToAll(comm.rank, comm.size, max_tokens, cfg.hidden_size, self.moe_F_pad,
                                 cfg.num_local_experts, cfg.num_experts_per_tok, cpu_group=comm.cpu_group,
                                 pg=comm.pg, timeout_s=comm.timeout_s)
        comm.nvls_one_shot_max = 0  # every collective keeps the row-sharded residual
        return True

    def _move_experts(self, L: dict, old: np.ndarray, new: np.ndarray) -> None:
        """Placement ``old`` -> ``new`` (physical slot -> logical expert): update the logical ->
        physical expert map, copy the experts that stay on this rank and exchange the others point to
        point (messages posted in destination-slot order on both sides)."""
        import torch.distributed as dist
        world, rank, cap = self.comm.size, self.comm.rank, self.E_loc
        to_old = torch.as_tensor(np.argsort(old))  # logical expert -> old physical slot
        sel = to_old[torch.as_tensor(new)]          # new physical slot -> old physical slot
        emap = torch.as_tensor(np.argsort(new), dtype=torch.int32)  # logical expert -> new physical slot
        if "expert_map" in L:
            L["expert_map"].copy_(emap.to(L["expert_map"].device))
        else:
            L["expert_map"] = emap.to(self.device)
        gu, dn = L["moe_gu"], L["moe_down"]
        rg, rd = gu.shape[0] // cap, dn.shape[0] // cap
        new_gu, new_dn = torch.empty_like(gu), torch.empty_like(dn)
        ops_ = []
        for p_new in range(rank * cap, (rank + 1) * cap):
            j, p_old = p_new - rank * cap, int(sel[p_new])
            src = p_old // cap
            if src == rank:
                i = p_old - rank * cap
                new_gu[j * rg:(j + 1) * rg].copy_(gu[i * rg:(i + 1) * rg])
                new_dn[j * rd:(j + 1) * rd].copy_(dn[i * rd:(i + 1) * rd])
            else:
                ops_.append(dist.P2POp(dist.irecv, new_gu[j * rg:(j + 1) * rg], src, tag=2 * p_new))
                ops_.append(dist.P2POp(dist.irecv, new_dn[j * rd:(j + 1) * rd], src, tag=2 * p_new + 1))
        for p_new in range(len(new)):
            p_old = int(sel[p_new])
            dst = p_new // cap
            if p_old // cap == rank and dst != rank:
                i = p_old - rank * cap
                ops_.append(dist.P2POp(dist.isend, gu[i * rg:(i + 1) * rg].contiguous(), dst, tag=2 * p_new))
                ops_.append(dist.P2POp(dist.isend, dn[i * rd:(i + 1) * rd].contiguous(), dst, tag=2 * p_new + 1))
        if ops_:
            for w in dist.batch_isend_irecv(ops_):
                w.wait()
        gu.copy_(new_gu)
        dn.copy_(new_dn)

    def _add_norm(self, h: torch.Tensor, residual: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """residual += all_reduce(h); returns norm(residual) * w (fused collective for RMSNorm;
        all-reduce then the LayerNorm kernel for centred norms)."""
        eps = self.cfg.rms_norm_eps
        if self.cfg.norm_center:
            return ops.fused_add_rms_norm(self.comm.all_reduce(h), residual, w, eps, center=True)
        return self.comm.allreduce_add_rmsnorm(h, residual, w, eps)

    def _gdn(self, x: torch.Tensor, L: Dict[str, torch.Tensor], meta: AttnMetadata, li: int) -> torch.Tensor:
        """Gated delta rule layer: fused projection, K14 scan over the batch's sequences (state slots
        per sequence), gated head norm; returns [T, Hg * 128] for the row-parallel output GEMM."""
        if self.gdn_state is None or meta.gdn_slots is None:
            raise RuntimeError("GDN layer without recurrent state / slot metadata")
        proj = ops.linear(x, L["w_gdn_in"])
        hd = self.Hg * 128
        o = ops.gdn_scan(proj, self.gdn_state[self.gdn_index[li]], meta.gdn_slots, meta.gdn_reset,
                         meta.gdn_query_start, L["A_log"], L["dt_bias"], self.Hg)
        return ops.gdn_gated_norm(o, proj[:, 3 * hd:4 * hd], L["gdn_norm"], self.cfg.rms_norm_eps)

    def _mla(self, x: torch.Tensor, L: Dict[str, torch.Tensor], meta: AttnMetadata, cache) -> torch.Tensor:
        """Multi-head latent attention of this rank's heads: latent GEMM, latent norms, q and kv
        up-projections written side by side into one [q | k | v] row, then the partial-rotary
        RoPE + paged KV write and the attention kernels (see ``_mla_weights`` for the layout)."""
        cfg, H, D, T = self.cfg, self.H, self.D, x.shape[0]
        eps, ql, kvl = cfg.rms_norm_eps, cfg.q_lora_rank, cfg.kv_lora_rank
        lat = ops.linear(x, L["w_qa_kva"])  # [T, q_lora + kv_lora + rope]
        ckv = lat[:, ql:]
        ops.rms_norm(ckv[:, :kvl], L["kv_a_norm"], eps, out=ckv[:, :kvl])  # in place: [norm(c) | k_rope]
        qkv = torch.empty(T, 3 * H * D, dtype=x.dtype, device=x.device)
        if ql:
            ops.linear(ops.rms_norm(lat[:, :ql], L["q_a_norm"], eps), L["w_q_b"], out=qkv[:, :H * D])
        else:
            ops.linear(x, L["w_q"], out=qkv[:, :H * D])
        ops.linear(ckv, L["w_kv_b"], out=qkv[:, H * D:])
        q = ops.rope_kv_write(qkv, meta.positions, self.cos_sin, cache, meta.slot_mapping, H, H, D)
        return self._attention(q, cache, meta, 0)

    def can_split_batch(self) -> bool:
        """Whether ``forward`` can run a step as two halves with overlapped collectives: dense
        pre-norm decoder layers (no MoE, GDN, MLA, LoRA, offload, sandwich or parallel blocks,
        centred norms) under a comm that supports it."""
        cfg = self.cfg
        return (getattr(self.comm, "supports_split", False) and self.comm.size > 1 and not cfg.is_moe
                and self.num_gdn_layers == 0 and not cfg.is_mla and self.lora is None and self.offload is None
                and not cfg.sandwich_norm and not cfg.parallel_block and not cfg.norm_center)

    def _plain_qkv(self, L: dict, kv_scales) -> bool:
        """The QKV projection can carry RoPE + the KV write in its GEMM epilogue: a plain bf16 weight,
        no bias / QK-norm / LoRA / fp8 cache (``ops.linear_rope_kv`` checks the shapes)."""
        return (self.lora is None and kv_scales is None and L.get("qkv_bias") is None and L.get("q_norm") is None
                and isinstance(L["w_qkv"], torch.Tensor) and L["w_qkv"].dtype == torch.bfloat16
                and L["w_qkv"].is_cuda)

    def _attn_block(self, x: torch.Tensor, L: dict, meta: AttnMetadata, kv_cache, li: int) -> torch.Tensor:
        """QKV GEMM, RoPE + paged KV write, attention of the rows of ``x`` ([T, H*D] output)."""
        cfg = self.cfg
        cache = kv_cache[self.kv_index[li]] if kv_cache is not None else None
        win = self.windows[li]
        cs = self.cos_sin_local if (self.cos_sin_local is not None and win > 0) else self.cos_sin
        if self.cos_sin_none is not None and win == 0:
            cs = self.cos_sin_none
        scl = self._kv_scales(li)
        if self._plain_qkv(L, scl):
            q = ops.linear_rope_kv(x, L["w_qkv"], meta.positions, cs, cache, meta.slot_mapping, self.H, self.Hk,
                                   self.D)
        else:
            qkv = ops.linear(x, L["w_qkv"])
            q = ops.rope_kv_write(qkv, meta.positions, cs, cache, meta.slot_mapping, self.H, self.Hk, self.D,
                                  bias=L.get("qkv_bias"), q_norm=L.get("q_norm"), k_norm=L.get("k_norm"),
                                  norm_eps=cfg.rms_norm_eps, kv_scales=scl)
        return self._attention(q, cache, meta, win, scl).view(x.shape[0], self.H * self.D)

    def _forward_split(self, input_ids: torch.Tensor, meta: AttnMetadata, kv_cache: Optional[torch.Tensor]):
        """The decoder layers over a step split in two halves (``meta.halves``): each half's
        row-parallel GEMM is followed by its all-reduce + residual + RMSNorm on a second
        (high-priority) stream, so one half's collective runs while the other half computes; the
        persistent GEMMs leave ``split_sms`` SMs free for it. Returns the final-norm rows [T, H]."""
        cfg = self.cfg
        eps = cfg.rms_norm_eps
        T = input_ids.shape[0]
        tA, mA, mB = meta.halves
        spans = [(0, tA, mA), (tA, T, mB)]
        h = self._embed_rows(input_ids, meta)
        residual = h
        x0 = ops.rms_norm(h, self.layers[0]["in_norm"], eps)
        xs = [x0[0:tA], x0[tA:T]]
        gathered = self.comm.gathered_rows(T)
        if gathered is None:  # no shared buffer (single process): the halves' rows land here
            gathered = torch.empty_like(h)
        cuda = input_ids.is_cuda
        comp = torch.cuda.current_stream() if cuda else None
        side = self._split_stream() if cuda else None
        ready = [None, None]  # event: the half's latest normalised rows are complete
        ext = None
        if cuda:
            from ..native import cuda_ext
            ext = cuda_ext()
            ops.set_gemm_sm_reserve(self.split_sms)
        n = len(self.layers)

        def collective(hi, r0, r1, part, w):
            if cuda:
                e = torch.cuda.Event()
                e.record(comp)
                with torch.cuda.stream(side):
                    side.wait_event(e)
                    out = self.comm.allreduce_add_rmsnorm_half(hi, r0, part, residual[r0:r1], w, eps)
                    ev = torch.cuda.Event()
                    ev.record(side)
                ready[hi] = ev
            else:
                out = self.comm.allreduce_add_rmsnorm_half(hi, r0, part, residual[r0:r1], w, eps)
                if out.data_ptr() != gathered[r0:r1].data_ptr():
                    gathered[r0:r1].copy_(out)
                    out = gathered[r0:r1]
            xs[hi] = out

        try:
            for li, L in enumerate(self.layers):
                nxt = self.layers[li + 1]["in_norm"] if li + 1 < n else self.norm
                for hi, (r0, r1, m) in enumerate(spans):
                    if ready[hi] is not None:
                        comp.wait_event(ready[hi])
                    a = self._attn_block(xs[hi], L, m, kv_cache, li)
                    part = ops.linear(a, L["w_o"], out=self.comm.half_partial_buffer(hi, r1 - r0))
                    collective(hi, r0, r1, part, L["post_norm"])
                for hi, (r0, r1, m) in enumerate(spans):
                    if ready[hi] is not None:
                        comp.wait_event(ready[hi])
                    g = ops.linear_swiglu(xs[hi], L["w_gate_up"], act=cfg.hidden_act)
                    part = ops.linear(g, L["w_down"], out=self.comm.half_partial_buffer(hi, r1 - r0))
                    collective(hi, r0, r1, part, nxt)
            for ev in ready:
                if ev is not None:
                    comp.wait_event(ev)
        finally:
            if ext is not None:
                ops.set_gemm_sm_reserve(0)
        return gathered

    def _embed_rows(self, input_ids: torch.Tensor, meta: AttnMetadata) -> torch.Tensor:
        """Token embeddings, with the rows of image placeholders replaced by projected image rows."""
        h = ops.embedding(input_ids, self.embed, scale=self.cfg.embed_scale)
        if meta.mm_rows is not None and meta.mm_rows.numel():
            h.index_copy_(0, meta.mm_rows, meta.mm_embeds.to(h.dtype))
        return h

    def _split_stream(self):
        st = getattr(self, "_side_stream", None)
        if st is None:
            st = self._side_stream = torch.cuda.Stream(priority=-1)
        return st

    def forward(self, input_ids: torch.Tensor, meta: AttnMetadata, kv_cache: Optional[torch.Tensor],
                hidden_only: bool = False, greedy: bool = False) -> torch.Tensor:
        """input_ids [T] int32 → logits [len(logits_indices), vocab] (gathered over TP), or with
        ``hidden_only`` the final-norm hidden states of every token [T, hidden]."""
        cfg = self.cfg
        eps = cfg.rms_norm_eps
        T = input_ids.shape[0]
        if meta.halves is not None and self.can_split_batch():
            x = self._forward_split(input_ids, meta, kv_cache)
            return self._head(x, meta, hidden_only, greedy)
        h = self._embed_rows(input_ids, meta)
        residual = h  # the embedding output buffer becomes the residual stream (updated in place)
        n = len(self.layers)
        ctr = cfg.norm_center
        x = ops.rms_norm(h, self.layers[0]["in_norm"], eps, center=ctr)
        nv = tracing.nvtx_enabled()
        off = self.offload
        if off is not None:
            off.begin_forward()
        for li, L in enumerate(self.layers):
            if off is not None:
                L = off.acquire(li)
            if nv:
                tracing.nvtx_push(f"layer{li}")
                tracing.nvtx_push("attn")
            if L.get("gdn"):
                a = self._gdn(x, L, meta, li)
            elif L.get("mla"):
                cache = kv_cache[self.kv_index[li]] if kv_cache is not None else None
                a = self._mla(x, L, meta, cache).view(T, self.H * self.D)
            else:
                cache = kv_cache[self.kv_index[li]] if kv_cache is not None else None
                win = self.windows[li]
                cs = self.cos_sin_local if (self.cos_sin_local is not None and win > 0) else self.cos_sin
                if self.cos_sin_none is not None and win == 0:
                    cs = self.cos_sin_none
                scl = self._kv_scales(li)
                if self._plain_qkv(L, scl):  # RoPE + KV write in the QKV GEMM's epilogue
                    q = ops.linear_rope_kv(x, L["w_qkv"], meta.positions, cs, cache, meta.slot_mapping, self.H,
                                           self.Hk, self.D)
                else:
                    qkv = ops.linear(x, L["w_qkv"])
                    if self.lora is not None:
                        self.lora.apply(li, "qkv", x, qkv)
                    q = ops.rope_kv_write(qkv, meta.positions, cs, cache, meta.slot_mapping, self.H, self.Hk, self.D,
                                          bias=L.get("qkv_bias"), q_norm=L.get("q_norm"), k_norm=L.get("k_norm"),
                                          norm_eps=eps, kv_scales=scl)
                a = self._attention(q, cache, meta, win, scl).view(T, self.H * self.D)
            if cfg.parallel_block:  # h = attn(x) + mlp(x): the down GEMM adds the attention partial
                ha = ops.linear(a, L["w_o"])
                if self.lora is not None:
                    self.lora.apply(li, "o", a, ha)
                g = ops.linear_swiglu(x, L["w_gate_up"], act=cfg.hidden_act)
                h = ops.linear(g, L["w_down"], residual=ha, out=self.comm.partial_buffer(T))
                nxt = self.layers[li + 1]["in_norm"] if li + 1 < n else self.norm
                x = self._add_norm(h, residual, nxt)
                if nv:
                    tracing.nvtx_pop()
                    tracing.nvtx_pop()
                if off is not None:
                    off.release(li)
                continue
            h = self._row_linear(a, L["w_o"], li, "o")
            if nv:
                tracing.nvtx_pop()
                tracing.nvtx_push("allreduce+norm")
            if self.ep_a2a is not None and cfg.is_moe_layer(li):
                # token-sharded MoE: reduce-scatter + norm of the owned rows, NVLink all-to-all through
                # the experts, combine + residual + next norm gathered on every rank
                from ..parallel.ep_a2a import owned_rows
                xo = self.comm.reduce_scatter_add_rmsnorm(h, residual, L["post_norm"], eps)
                r0, Tn = owned_rows(T, self.comm.rank, self.comm.size)
                nxt = self.layers[li + 1]["in_norm"] if li + 1 < n else self.norm
                x = self.ep_a2a.moe(xo[r0:r0 + Tn], residual, L["router"], L["moe_gu"], L["moe_down"], nxt, eps, T,
                                    renorm=cfg.norm_topk_prob, expert_map=L.get("expert_map"))
                if nv:
                    tracing.nvtx_pop()
                    tracing.nvtx_pop()
                if off is not None:
                    off.release(li)
                continue
            if cfg.sandwich_norm:  # norm(attn) + residual, then the pre-FFN norm
                h = ops.rms_norm(self.comm.all_reduce(h), L["post_norm"], eps)
                x = ops.fused_add_rms_norm(h, residual, L["pre_ff_norm"], eps)
            else:
                x = self._add_norm(h, residual, L["post_norm"])
            if nv:
                tracing.nvtx_pop()
                tracing.nvtx_push("moe" if cfg.is_moe_layer(li) else "ffn")
            if cfg.is_moe_layer(li):
                h = self._moe(x, L, out=self.comm.partial_buffer(T))
            else:
                h = self._row_linear(ops.linear_swiglu(x, L["w_gate_up"], act=cfg.hidden_act), L["w_down"], li)
            nxt = self.layers[li + 1]["in_norm"] if li + 1 < n else self.norm
            if nv:
                tracing.nvtx_pop()
                tracing.nvtx_push("allreduce+norm")
            if cfg.sandwich_norm:
                h = ops.rms_norm(self.comm.all_reduce(h), L["post_ff_norm"], eps)
                x = ops.fused_add_rms_norm(h, residual, nxt, eps)
            else:
                x = self._add_norm(h, residual, nxt)
            if nv:
                tracing.nvtx_pop()
                tracing.nvtx_pop()
            if off is not None:
                off.release(li)
        return self._head(x, meta, hidden_only, greedy)

    def _head(self, x: torch.Tensor, meta: AttnMetadata, hidden_only: bool, greedy: bool) -> torch.Tensor:
        """Final-norm rows → hidden states, greedy ids or logits."""
        cfg = self.cfg
        if hidden_only:
            if cfg.logit_scale != 1.0:
                return x / cfg.logit_scale
            # x may be a view of a shared buffer of the TP comm or the all-to-all, rewritten by its next call
            return x.clone() if (getattr(self.comm, "shares_x", False) or self.ep_a2a is not None) else x
        if meta.logits_indices is not None:
            x = x.index_select(0, meta.logits_indices)
        if greedy:  # token ids: argmax over the vocab shards without gathering the logits
            return self.comm.argmax_last(ops.linear(x, self.lm_head), self.comm.rank * self.V_local)
        logits = self.comm.all_gather_last(ops.linear(x, self.lm_head))
        if cfg.final_logit_softcapping:
            c = cfg.final_logit_softcapping
            logits = torch.tanh(logits.float() / c).mul_(c).to(logits.dtype)
        return logits
