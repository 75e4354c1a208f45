"""GGUF (v3) reader/writer, own implementation.

Layout: ``"GGUF"`` magic, u32 version, u64 tensor count, u64 metadata count; metadata
key/value pairs (typed, arrays allowed); tensor infos (name, n_dims, dims with ``ne[0]``
fastest-varying, ggml type, offset); padding to ``general.alignment`` (default 32); data.

Supported tensor types: F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K
(ggml block layouts; quantizers and dequantizers are in the host C++ module, checked bit for bit
against gguf-py). Q8_0 and Q4_K linear weights can stay quantized on the GPU (dequant-fused
kernels); the other types are dequantized to the serving dtype at load. Covers the reference's GGUF loader
(runner/gguf/gollek-gguf-core/…/gguf/core/GgmlType.java:8-42 type table;
runner/gguf/gollek-gguf-loader/…/gguf/loader/GGUFLoader.java:38-190 metadata + mmap +
Llama tensor mapping) and its converter's writer (runner/gguf/gollek-gguf-converter-java/…/
GgufWriter.java, LlamaArchMapper.java).

Llama Q/K weights in GGUF are stored row-permuted for llama.cpp's interleaved RoPE; on load we
undo that permutation so every checkpoint runs the same NeoX (rotate-half) RoPE kernel (the
reference's pure-Java path skips this and mixes RoPE conventions,
runner/gguf/gollek-gguf-loader/…/gguf/tensor/GGUFVectorOps.java:250-264).
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch

from ..config import ModelConfig, RopeScaling

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3

# metadata value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# ggml tensor types we handle: id -> (name, block elements, block bytes)
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_BF16 = 0, 1, 8, 12, 30
GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q2_K, GGML_Q3_K, GGML_Q5_K, GGML_Q6_K = 2, 3, 6, 7, 10, 11, 13, 14
GGML_TYPES = {
    GGML_F32: ("F32", 1, 4),
    GGML_F16: ("F16", 1, 2),
    GGML_Q4_0: ("Q4_0", 32, 18),
    GGML_Q4_1: ("Q4_1", 32, 20),
    GGML_Q5_0: ("Q5_0", 32, 22),
    GGML_Q5_1: ("Q5_1", 32, 24),
    GGML_Q8_0: ("Q8_0", 32, 34),
    GGML_Q2_K: ("Q2_K", 256, 84),
    GGML_Q3_K: ("Q3_K", 256, 110),
    GGML_Q4_K: ("Q4_K", 256, 144),
    GGML_Q5_K: ("Q5_K", 256, 176),
    GGML_Q6_K: ("Q6_K", 256, 210),
    GGML_BF16: ("BF16", 1, 2),
}
# types kept in their blocks on the GPU by the dequant-fused kernels
SERVED_QUANTIZED = (GGML_Q8_0, GGML_Q4_K, GGML_Q6_K)


def dequantize_blocks(raw: torch.Tensor, ggml_type: int, n: int) -> torch.Tensor:
    """fp32 values of ``n`` elements stored as ggml blocks of ``ggml_type`` (CPU uint8 ``raw``)."""
    from ..native import host_ext
    h = host_ext()
    raw = raw.cpu().contiguous()
    if ggml_type == GGML_Q8_0:
        return h.dequantize_q8_0(raw, n)
    if ggml_type == GGML_Q4_K:
        return h.dequantize_q4_k(raw, n)
    return h.gguf_dequantize(raw, ggml_type, n)


def quantize_blocks(t: torch.Tensor, ggml_type: int) -> torch.Tensor:
    """ggml blocks (uint8) of ``t``'s values in ``ggml_type``."""
    from ..native import host_ext
    h = host_ext()
    x = t.float().flatten().contiguous()
    if ggml_type == GGML_Q8_0:
        return h.quantize_q8_0(x)
    if ggml_type == GGML_Q4_K:
        return h.quantize_q4_k(x)
    return h.gguf_quantize(x, ggml_type)
TYPE_BY_NAME = {v[0]: k for k, v in GGML_TYPES.items()}


@dataclass
class GGUFTensorInfo:
    name: str
    shape: Tuple[int, ...]   # torch order (row-major): reversed ggml ne
    ggml_type: int
    offset: int              # absolute file offset of the data

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    @property
    def nbytes(self) -> int:
        _, be, bb = GGML_TYPES[self.ggml_type]
        return self.numel // be * bb


class GGUFFile:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._buf = np.frombuffer(self._mm, dtype=np.uint8)
        self._pos = 0
        if self._read(4) != GGUF_MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        (self.version,) = self._unpack("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{path}: unsupported GGUF version {self.version}")
        n_tensors, n_kv = self._unpack("<QQ")
        self.metadata: Dict[str, Any] = {}
        for _ in range(n_kv):
            key = self._read_str()
            (vt,) = self._unpack("<I")
            self.metadata[key] = self._read_value(vt)
        infos = []
        for _ in range(n_tensors):
            name = self._read_str()
            (nd,) = self._unpack("<I")
            ne = self._unpack("<" + "Q" * nd)
            gt, off = self._unpack("<IQ")
            if gt not in GGML_TYPES:
                raise ValueError(f"{path}: tensor {name} has unsupported ggml type {gt}")
            infos.append((name, tuple(reversed(ne)), gt, off))
        align = int(self.metadata.get("general.alignment", 32))
        data_start = (self._pos + align - 1) // align * align
        self.tensors: Dict[str, GGUFTensorInfo] = {
            n: GGUFTensorInfo(n, s, t, data_start + o) for n, s, t, o in infos}
        self.alignment = align

    # -- primitive readers
    def _read(self, n: int) -> bytes:
        b = self._mm[self._pos: self._pos + n]
        if len(b) != n:
            raise ValueError(f"{self.path}: truncated")
        self._pos += n
        return b

    def _unpack(self, fmt: str):
        n = struct.calcsize(fmt)
        return struct.unpack(fmt, self._read(n))

    def _read_str(self) -> str:
        (n,) = self._unpack("<Q")
        return self._read(n).decode("utf-8", errors="replace")

    def _read_value(self, vt: int):
        if vt in _SCALAR:
            return self._unpack(_SCALAR[vt])[0]
        if vt == T_STR:
            return self._read_str()
        if vt == T_ARR:
            et, n = self._unpack("<IQ")
            if et in _SCALAR and et != T_BOOL:
                fmt = _SCALAR[et]
                sz = struct.calcsize(fmt)
                arr = np.frombuffer(self._read(sz * n), dtype=np.dtype(fmt))
                return arr.tolist()
            return [self._read_value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {vt}")

    # -- tensors
    def raw(self, name: str) -> torch.Tensor:
        """Raw bytes of a tensor (uint8, zero-copy view of the mapping)."""
        ti = self.tensors[name]
        return torch.frombuffer(self._buf[ti.offset: ti.offset + ti.nbytes], dtype=torch.uint8)

    def get(self, name: str, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Dequantized tensor in torch (row-major) shape."""
        ti = self.tensors[name]
        raw = self.raw(name)
        if ti.ggml_type == GGML_F32:
            t = raw.view(torch.float32)
        elif ti.ggml_type == GGML_F16:
            t = raw.view(torch.float16)
        elif ti.ggml_type == GGML_BF16:
            t = raw.view(torch.bfloat16)
        else:
            t = dequantize_blocks(raw.clone(), ti.ggml_type, ti.numel)
        return t.reshape(ti.shape).to(dtype)

    def close(self):
        """Release the mapping; while zero-copy tensors returned by ``raw`` / ``get`` are alive the
        mapping stays open and is released when the last of them goes away."""
        self._buf = None
        try:
            self._mm.close()
        except BufferError:
            pass
        self._f.close()


# ----------------------------------------------------------------------------- writer
class GGUFWriter:
    def __init__(self, path: str, alignment: int = 32):
        self.path = path
        self.alignment = alignment
        self.kv: List[Tuple[str, int, Any, Optional[int]]] = []
        self.tensors: List[Tuple[str, Tuple[int, ...], int, bytes]] = []
        if alignment != 32:
            self.add("general.alignment", alignment, T_U32)

    def add(self, key: str, value: Any, vtype: Optional[int] = None, elem_type: Optional[int] = None):
        if vtype is None:
            if isinstance(value, bool):
                vtype = T_BOOL
            elif isinstance(value, int):
                vtype = T_U32 if 0 <= value < 2 ** 32 else T_I64
            elif isinstance(value, float):
                vtype = T_F32
            elif isinstance(value, str):
                vtype = T_STR
            elif isinstance(value, (list, tuple)):
                vtype = T_ARR
                if elem_type is None:
                    v0 = value[0] if value else ""
                    elem_type = T_STR if isinstance(v0, str) else (T_F32 if isinstance(v0, float) else T_I32)
            else:
                raise TypeError(f"cannot infer GGUF type of {key}")
        self.kv.append((key, vtype, value, elem_type))

    def add_tensor(self, name: str, t: torch.Tensor, ggml_type: int = GGML_F32):
        t = t.detach().cpu()
        if ggml_type == GGML_F32:
            data = t.float().contiguous().view(torch.uint8).numpy().tobytes()
        elif ggml_type == GGML_F16:
            data = t.half().contiguous().view(torch.uint8).numpy().tobytes()
        elif ggml_type == GGML_BF16:
            data = t.bfloat16().contiguous().view(torch.uint8).numpy().tobytes()
        else:
            data = quantize_blocks(t, ggml_type).numpy().tobytes()
        self.tensors.append((name, tuple(t.shape), ggml_type, data))

    @staticmethod
    def _pack_str(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def _pack_value(self, vt: int, v: Any, et: Optional[int]) -> bytes:
        if vt in _SCALAR:
            return struct.pack(_SCALAR[vt], v)
        if vt == T_STR:
            return self._pack_str(v)
        if vt == T_ARR:
            out = struct.pack("<IQ", et, len(v))
            return out + b"".join(self._pack_value(et, x, None) for x in v)
        raise ValueError(vt)

    def write(self):
        head = bytearray(GGUF_MAGIC + struct.pack("<IQQ", GGUF_VERSION, len(self.tensors), len(self.kv)))
        for k, vt, v, et in self.kv:
            head += self._pack_str(k) + struct.pack("<I", vt) + self._pack_value(vt, v, et)
        offsets, off = [], 0
        for name, shape, gt, data in self.tensors:
            offsets.append(off)
            off += (len(data) + self.alignment - 1) // self.alignment * self.alignment
        for (name, shape, gt, data), o in zip(self.tensors, offsets):
            ne = list(reversed(shape))
            head += self._pack_str(name) + struct.pack("<I", len(ne)) + struct.pack("<" + "Q" * len(ne), *ne)
            head += struct.pack("<IQ", gt, o)
        pad = (self.alignment - len(head) % self.alignment) % self.alignment
        with open(self.path, "wb") as f:
            f.write(head)
            f.write(b"\0" * pad)
            for name, shape, gt, data in self.tensors:
                f.write(data)
                f.write(b"\0" * ((self.alignment - len(data) % self.alignment) % self.alignment))


# ----------------------------------------------------------------------------- llama mapping
def permute_qk(w: torch.Tensor, n_head: int) -> torch.Tensor:
    """HF (rotate-half) row order → GGUF (interleaved-pair) row order for Q/K weights."""
    out = w.shape[0]
    return w.reshape(n_head, 2, out // n_head // 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape)


def unpermute_qk(w: torch.Tensor, n_head: int) -> torch.Tensor:
    out = w.shape[0]
    return w.reshape(n_head, out // n_head // 2, 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape)


_LAYER_MAP = {
    "input_layernorm.weight": "attn_norm.weight",
    "self_attn.q_proj.weight": "attn_q.weight",
    "self_attn.k_proj.weight": "attn_k.weight",
    "self_attn.v_proj.weight": "attn_v.weight",
    "self_attn.o_proj.weight": "attn_output.weight",
    "post_attention_layernorm.weight": "ffn_norm.weight",
    "mlp.gate_proj.weight": "ffn_gate.weight",
    "mlp.up_proj.weight": "ffn_up.weight",
    "mlp.down_proj.weight": "ffn_down.weight",
    "block_sparse_moe.gate.weight": "ffn_gate_inp.weight",
}
_EXPERT_MAP = {"w1": "ffn_gate", "w3": "ffn_up", "w2": "ffn_down"}


def hf_to_gguf_name(name: str) -> str:
    if name == "model.embed_tokens.weight":
        return "token_embd.weight"
    if name == "model.norm.weight":
        return "output_norm.weight"
    if name == "lm_head.weight":
        return "output.weight"
    parts = name.split(".")
    i = parts[2]
    rest = ".".join(parts[3:])
    if rest in _LAYER_MAP:
        return f"blk.{i}.{_LAYER_MAP[rest]}"
    if rest.startswith("block_sparse_moe.experts."):
        e, w = parts[5], parts[6]
        return f"blk.{i}.{_EXPERT_MAP[w]}.{e}.weight"
    raise KeyError(name)


def gguf_to_hf_name(name: str) -> str:
    inv = {v: k for k, v in _LAYER_MAP.items()}
    if name == "token_embd.weight":
        return "model.embed_tokens.weight"
    if name == "output_norm.weight":
        return "model.norm.weight"
    if name == "output.weight":
        return "lm_head.weight"
    parts = name.split(".")
    i = parts[1]
    rest = ".".join(parts[2:])
    if rest in inv:
        return f"model.layers.{i}.{inv[rest]}"
    if len(parts) == 5:  # blk.i.ffn_gate.E.weight
        w = {v: k for k, v in _EXPERT_MAP.items()}[parts[2]]
        return f"model.layers.{i}.block_sparse_moe.experts.{parts[3]}.{w}.weight"
    raise KeyError(name)


# Tensor-type mixtures named like llama.cpp's file types: a base k-quant for most linears, more
# bits for the tensors most sensitive to quantization (output, attention V, FFN down of the first
# and last eighth of the layers and every third layer between them).
MIXTURES = {"Q4_K_M": GGML_Q4_K, "Q5_K_M": GGML_Q5_K, "Q3_K_M": GGML_Q3_K, "Q4_K_S": GGML_Q4_K,
            "Q5_K_S": GGML_Q5_K, "Q3_K_S": GGML_Q3_K, "Q3_K_L": GGML_Q3_K}


def _more_bits(layer: int, n_layers: int) -> bool:
    return layer < n_layers // 8 or layer >= 7 * n_layers // 8 or (layer - n_layers // 8) % 3 == 2


def mixture_type(recipe: str, hf_name: str, n_layers: int) -> int:
    """ggml type of one 2-D tensor under a ``*_K_M`` mixture."""
    base = MIXTURES[recipe]
    if hf_name == "lm_head.weight":
        return GGML_Q6_K
    if hf_name == "model.embed_tokens.weight":
        return base
    layer = int(hf_name.split(".")[2]) if hf_name.startswith("model.layers.") else 0
    sensitive = hf_name.endswith(("v_proj.weight", "down_proj.weight", "w2.weight"))
    if recipe.endswith("_S"):  # small: only the output matrix gets more bits
        return base
    if recipe == "Q3_K_L":
        return GGML_Q5_K if sensitive or hf_name.endswith("o_proj.weight") else base
    if recipe == "Q3_K_M":
        if sensitive:
            return GGML_Q5_K if layer < 2 or hf_name.endswith("v_proj.weight") and _more_bits(layer, n_layers) \
                else GGML_Q4_K
        return GGML_Q4_K if hf_name.endswith("o_proj.weight") else base
    return GGML_Q6_K if sensitive and _more_bits(layer, n_layers) else base


def write_llama_gguf(path: str, cfg: ModelConfig, weights: Dict[str, torch.Tensor],
                     linear_type: Any = GGML_F32, embed_type: Optional[int] = None,
                     vocab: Optional[List[str]] = None, progress=None) -> None:
    """Write an HF-named Llama/Mixtral state dict as GGUF (norms always F32). ``linear_type`` is a
    ggml type id or a mixture name (``"Q4_K_M"``, ``"Q5_K_M"``, ``"Q3_K_M"``)."""
    w = GGUFWriter(path)
    arch = "llama"
    w.add("general.architecture", arch)
    w.add("general.name", "gollek-b200-export")
    w.add(f"{arch}.context_length", cfg.max_position_embeddings)
    w.add(f"{arch}.embedding_length", cfg.hidden_size)
    w.add(f"{arch}.block_count", cfg.num_hidden_layers)
    w.add(f"{arch}.feed_forward_length", cfg.intermediate_size)
    w.add(f"{arch}.attention.head_count", cfg.num_attention_heads)
    w.add(f"{arch}.attention.head_count_kv", cfg.num_key_value_heads)
    w.add(f"{arch}.attention.key_length", cfg.head_dim)
    w.add(f"{arch}.attention.value_length", cfg.head_dim)
    w.add(f"{arch}.rope.freq_base", float(cfg.rope_theta))
    w.add(f"{arch}.attention.layer_norm_rms_epsilon", float(cfg.rms_norm_eps))
    w.add(f"{arch}.vocab_size", cfg.vocab_size)
    if cfg.is_moe:
        w.add(f"{arch}.expert_count", cfg.num_local_experts)
        w.add(f"{arch}.expert_used_count", cfg.num_experts_per_tok)
    w.add("tokenizer.ggml.model", "llama")
    w.add("tokenizer.ggml.tokens", vocab if vocab is not None else [f"<t{i}>" for i in range(cfg.vocab_size)], T_ARR, T_STR)
    w.add("tokenizer.ggml.bos_token_id", cfg.bos_token_id)
    w.add("tokenizer.ggml.eos_token_id", cfg.eos_token_id)
    recipe = linear_type if isinstance(linear_type, str) else None
    if recipe is not None and recipe not in MIXTURES:
        raise ValueError(f"unknown mixture {recipe!r} (known: {sorted(MIXTURES)})")
    emb_t = linear_type if embed_type is None else embed_type
    names = list(weights)
    for idx, name in enumerate(names):
        if progress is not None:
            progress(idx, len(names), name)  # may raise to cancel the conversion
        t = weights[name]
        g = hf_to_gguf_name(name)
        if name.endswith("q_proj.weight"):
            t = permute_qk(t, cfg.num_attention_heads)
        elif name.endswith("k_proj.weight"):
            t = permute_qk(t, cfg.num_key_value_heads)
        if t.dim() == 1:
            gt = GGML_F32
        elif recipe is not None and not (embed_type is not None and name == "model.embed_tokens.weight"):
            gt = mixture_type(recipe, name, cfg.num_hidden_layers)
        elif name in ("model.embed_tokens.weight", "lm_head.weight"):
            gt = emb_t
        else:
            gt = linear_type
        bs = GGML_TYPES[gt][1]
        if t.dim() == 2 and t.shape[-1] % bs:
            gt = GGML_F16  # rows that are not a whole number of blocks stay unquantized
        w.add_tensor(g, t, gt)
    w.write()


def config_from_gguf(meta: Dict[str, Any]) -> ModelConfig:
    arch = meta.get("general.architecture", "llama")
    g = lambda k, d=None: meta.get(f"{arch}.{k}", d)  # noqa: E731
    nh = int(g("attention.head_count"))
    hs = int(g("embedding_length"))
    n_exp = int(g("expert_count", 0) or 0)
    vocab = g("vocab_size")
    if vocab is None:
        vocab = len(meta.get("tokenizer.ggml.tokens", [])) or 32000
    return ModelConfig(
        architecture="mixtral" if n_exp else "llama",
        vocab_size=int(vocab),
        hidden_size=hs,
        intermediate_size=int(g("feed_forward_length")),
        num_hidden_layers=int(g("block_count")),
        num_attention_heads=nh,
        num_key_value_heads=int(g("attention.head_count_kv", nh)),
        head_dim=int(g("attention.key_length", hs // nh)),
        rms_norm_eps=float(g("attention.layer_norm_rms_epsilon", 1e-5)),
        rope_theta=float(g("rope.freq_base", 10000.0)),
        rope_scaling=RopeScaling(),
        max_position_embeddings=int(g("context_length", 4096)),
        num_local_experts=n_exp,
        num_experts_per_tok=int(g("expert_used_count", 0) or 0),
        bos_token_id=int(meta.get("tokenizer.ggml.bos_token_id", 1)),
        eos_token_id=int(meta.get("tokenizer.ggml.eos_token_id", 2)),
    )


def load_llama_gguf(path: str, dtype: torch.dtype = torch.float32,
                    keep_quantized: bool = False) -> Tuple[ModelConfig, Dict[str, Any], GGUFFile]:
    """Load a Llama-family GGUF into an HF-named state dict.

    With ``keep_quantized`` the linear weights stay as ``QuantizedWeight`` (raw ggml blocks +
    shape) for the dequant-fused kernels; norms and embeddings are always dequantized.
    """
    f = GGUFFile(path)
    cfg = config_from_gguf(f.metadata)
    out: Dict[str, Any] = {}
    for name, ti in f.tensors.items():
        hf = gguf_to_hf_name(name)
        is_q = hf.endswith("q_proj.weight")
        is_k = hf.endswith("k_proj.weight")
        keep = keep_quantized and ti.ggml_type in SERVED_QUANTIZED and len(ti.shape) == 2
        if hf == "model.embed_tokens.weight" and ti.ggml_type != GGML_Q8_0:
            keep = False  # the quantized embedding gather supports Q8_0 tables
        if keep:
            raw = f.raw(name).clone()
            if is_q or is_k:  # blocks run along K, so the Q/K row permutation moves whole byte rows
                rows = raw.view(ti.shape[0], -1)
                heads = cfg.num_attention_heads if is_q else cfg.num_key_value_heads
                raw = unpermute_qk(rows, heads).contiguous().view(-1)
            out[hf] = QuantizedWeight(raw, ti.shape, ti.ggml_type)
            continue
        t = f.get(name, torch.float32)
        if is_q:
            t = unpermute_qk(t, cfg.num_attention_heads)
        elif is_k:
            t = unpermute_qk(t, cfg.num_key_value_heads)
        out[hf] = t.to(dtype)
    if "lm_head.weight" not in out:
        cfg.tie_word_embeddings = True
    return cfg, out, f


@dataclass
class QuantizedWeight:
    """A GGUF-quantized [N, K] weight kept in its ggml block format."""
    raw: torch.Tensor
    shape: Tuple[int, int]
    ggml_type: int

    def dequantize(self) -> torch.Tensor:
        n = self.shape[0] * self.shape[1]
        return dequantize_blocks(self.raw, self.ggml_type, n).view(self.shape)
