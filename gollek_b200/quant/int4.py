"""4-bit group-quantized weights: GPTQ / AWQ / round-to-nearest int4 and NF4 (QLoRA).

``Int4Weight`` holds an ``[N, K]`` matrix in one canonical layout (csrc/kernels/int4.cu):
``q`` uint8 [N, K/2] (low nibble = even k), ``scale`` [N, K/g] and, for int4, ``zero`` [N, K/g]
(w = (q - zero) * scale); NF4 uses w = NF4[q] * scale. Every source is converted into it:

* ``quantize_rtn``   round-to-nearest asymmetric int4 per group (min/max).
* ``quantize_gptq``  GPTQ (Frantar et al., "GPTQ: Accurate Post-Training Quantization for
                     Generative Pre-trained Transformers", 2022): columns quantized in order,
                     each one's rounding error propagated to the not-yet-quantized columns through
                     the Cholesky factor of the inverse Hessian H = 2 X Xᵀ of calibration inputs.
* ``quantize_nf4``   NF4 with per-block absmax scales (Dettmers et al., "QLoRA", 2023).
* ``from_awq``       AutoAWQ GEMM checkpoints: qweight int32 [K, N/8] (8 columns per word in the
                     order 0,2,4,6,1,3,5,7), qzeros int32 [K/g, N/8] (same order), scales [K/g, N].
* ``from_gptq``      AutoGPTQ checkpoints: qweight int32 [K/8, N] (8 consecutive k per word),
                     qzeros int32 [K/g, N/8] storing zero - 1, scales [K/g, N]; act-order
                     (non-monotonic g_idx) is dequantized to bf16 instead.

The reference ships GPTQ/AWQ/AutoRound quantizers in Java (core/quantizer/gollek-quantizer-*)
and an NF4 QLoRA path that decodes on the CPU (core/optimization/gollek-plugin-qlora/…/
QLoraCpuFallback.java:18-119).
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

NF4_LEVELS = torch.tensor([-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
                           -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
                           0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
                           0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
                           0.7229568362236023, 1.0])

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)  # column position of the i-th nibble of an AWQ word


class Int4Weight:
    def __init__(self, q: torch.Tensor, scale: torch.Tensor, zero: Optional[torch.Tensor], N: int, K: int,
                 group: int, nf4: bool = False):
        if K % group or group % 32:
            raise ValueError(f"group size {group} must divide K={K} and be a multiple of 32")
        self.q = q.reshape(N, K // 2)
        self.scale = scale.reshape(N, K // group)
        self.zero = None if zero is None else zero.reshape(N, K // group)
        self.N, self.K, self.group, self.nf4 = N, K, group, nf4

    @property
    def shape(self):
        return (self.N, self.K)

    @property
    def device(self):
        return self.q.device

    def nbytes(self) -> int:
        n = self.q.numel() + self.scale.numel() * self.scale.element_size()
        return n + (0 if self.zero is None else self.zero.numel() * self.zero.element_size())

    def to(self, device=None, dtype=None) -> "Int4Weight":
        z = None if self.zero is None else self.zero.to(device, torch.bfloat16).contiguous()
        return Int4Weight(self.q.to(device).contiguous(), self.scale.to(device, torch.bfloat16).contiguous(), z,
                          self.N, self.K, self.group, self.nf4)

    def contiguous(self) -> "Int4Weight":
        return self.to(self.q.device)

    def __getitem__(self, idx) -> "Int4Weight":
        if isinstance(idx, tuple):  # [:, k0:k1]
            rows, cols = idx
            out = self if rows == slice(None) else self[rows]
            return out.kslice(cols.start or 0, cols.stop if cols.stop is not None else self.K)
        q = self.q[idx]
        return Int4Weight(q, self.scale[idx], None if self.zero is None else self.zero[idx], q.shape[0], self.K,
                          self.group, self.nf4)

    def kslice(self, k0: int, k1: int) -> "Int4Weight":
        g = self.group
        if k0 % g or k1 % g:
            raise ValueError("K slices must fall on quantization group boundaries")
        z = None if self.zero is None else self.zero[:, k0 // g:k1 // g].contiguous()
        return Int4Weight(self.q[:, k0 // 2:k1 // 2].contiguous(), self.scale[:, k0 // g:k1 // g].contiguous(), z,
                          self.N, k1 - k0, g, self.nf4)

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        """[N, K] (GPU kernel on CUDA, torch on the CPU)."""
        if self.q.is_cuda:
            from ..native import cuda_ext
            out = torch.empty(self.N, self.K, dtype=torch.bfloat16, device=self.q.device)
            cuda_ext().int4_dequant(out, self.q.contiguous(), self.scale.contiguous(),
                                    None if self.zero is None else self.zero.contiguous(), self.N, self.K, self.group,
                                    self.nf4)
            return out.to(dtype)
        lo = (self.q & 0xF).long()
        hi = (self.q >> 4).long()
        codes = torch.stack([lo, hi], -1).reshape(self.N, self.K)
        s = self.scale.float().repeat_interleave(self.group, 1)
        if self.nf4:
            w = NF4_LEVELS[codes] * s
        else:
            w = (codes.float() - self.zero.float().repeat_interleave(self.group, 1)) * s
        return w.to(dtype)


def _pack(codes: torch.Tensor) -> torch.Tensor:
    """[N, K] ints in [0, 15] -> uint8 [N, K/2] (low nibble = even k)."""
    c = codes.to(torch.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).contiguous()


def cat_rows(ws: Sequence[Int4Weight]) -> Int4Weight:
    if len({(w.K, w.group, w.nf4) for w in ws}) != 1:
        raise ValueError("row concatenation needs equal K, group size and format")
    z = None if ws[0].zero is None else torch.cat([w.zero for w in ws], 0)
    q = torch.cat([w.q for w in ws], 0)
    return Int4Weight(q, torch.cat([w.scale for w in ws], 0), z, q.shape[0], ws[0].K, ws[0].group, ws[0].nf4)


def interleave_rows(g: Int4Weight, u: Int4Weight, group: int = 64) -> Int4Weight:
    if g.N % group:
        raise ValueError("gate/up rows must be a multiple of the interleave group")

    def il(a, b):
        return torch.stack([a.view(g.N // group, group, -1), b.view(u.N // group, group, -1)], 1).reshape(2 * g.N, -1)
    z = None if g.zero is None else il(g.zero, u.zero)
    return Int4Weight(il(g.q, u.q), il(g.scale, u.scale), z, 2 * g.N, g.K, g.group, g.nf4)


# ---------------------------------------------------------------------------- quantizers
def quantize_rtn(w: torch.Tensor, group: int = 128) -> Int4Weight:
    """Round-to-nearest asymmetric int4 per group of ``group`` columns."""
    N, K = w.shape
    x = w.float().reshape(N, K // group, group)
    mn, mx = x.amin(-1), x.amax(-1)
    scale = ((mx - mn) / 15.0).clamp_min(1e-8)
    zero = torch.round(-mn / scale).clamp(0, 15)
    codes = torch.round(x / scale[..., None] + zero[..., None]).clamp(0, 15).reshape(N, K)
    return Int4Weight(_pack(codes), scale.to(torch.bfloat16), zero.to(torch.bfloat16), N, K, group)


def quantize_nf4(w: torch.Tensor, block: int = 64) -> Int4Weight:
    """NF4 with one absmax scale per ``block`` columns (QLoRA's data type, single quantization)."""
    N, K = w.shape
    x = w.float().reshape(N, K // block, block)
    absmax = x.abs().amax(-1).clamp_min(1e-8)
    xn = x / absmax[..., None]
    codes = (xn[..., None] - NF4_LEVELS.to(x.device)).abs().argmin(-1).reshape(N, K)
    return Int4Weight(_pack(codes), absmax.to(torch.bfloat16), None, N, K, block, nf4=True)


def quantize_gptq(w: torch.Tensor, H: torch.Tensor, group: int = 128, damp: float = 0.01,
                  block: int = 128) -> Int4Weight:
    """GPTQ with asymmetric int4 groups (scales/zeros of a group fixed when its first column is
    reached, from the error-updated weights). ``H`` = 2 X Xᵀ over calibration inputs X [K, n]."""
    W = w.float().clone()
    N, K = W.shape
    H = H.float().clone()
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += damp * torch.mean(torch.diag(H)) * torch.eye(K, device=H.device)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    codes = torch.zeros(N, K, dtype=torch.long, device=W.device)
    scale = torch.zeros(N, K // group, device=W.device)
    zero = torch.zeros(N, K // group, device=W.device)
    for b0 in range(0, K, block):
        b1 = min(K, b0 + block)
        W1 = W[:, b0:b1].clone()
        Err = torch.zeros_like(W1)
        Hb = Hinv[b0:b1, b0:b1]
        for i in range(b1 - b0):
            k = b0 + i
            if k % group == 0:  # group parameters from the current (error-compensated) weights
                seg = torch.cat([W1[:, i:], W[:, b1:]], 1)[:, :group]
                mn, mx = seg.amin(1), seg.amax(1)
                s = ((mx - mn) / 15.0).clamp_min(1e-8)
                scale[:, k // group], zero[:, k // group] = s, torch.round(-mn / s).clamp(0, 15)
            s, z = scale[:, k // group], zero[:, k // group]
            col = W1[:, i]
            c = torch.round(col / s + z).clamp(0, 15)
            codes[:, k] = c.long()
            qv = (c - z) * s
            e = (col - qv) / Hb[i, i]
            W1[:, i:] -= e[:, None] * Hb[i, i:][None, :]
            Err[:, i] = e
        W[:, b1:] -= Err @ Hinv[b0:b1, b1:]
    return Int4Weight(_pack(codes), scale.to(torch.bfloat16), zero.to(torch.bfloat16), N, K, group)


# ---------------------------------------------------------------------------- checkpoint formats
def _unpack_words(words: torch.Tensor, order=None) -> torch.Tensor:
    """int32 [..., C] -> int [..., 8C] nibbles; nibble i of word c goes to 8c + order[i]."""
    w = words.to(torch.int64) & 0xFFFFFFFF
    nib = torch.stack([(w >> (4 * i)) & 0xF for i in range(8)], -1)  # [..., C, 8] by nibble index
    if order is not None:
        out = torch.empty_like(nib)
        out[..., list(order)] = nib
        nib = out
    return nib.reshape(*words.shape[:-1], words.shape[-1] * 8)


def _pack_words(vals: torch.Tensor, order=None) -> torch.Tensor:
    """Inverse of ``_unpack_words`` (used by tests and the exporter)."""
    v = vals.to(torch.int64).reshape(*vals.shape[:-1], vals.shape[-1] // 8, 8)
    if order is not None:
        v = v[..., list(order)]
    word = torch.zeros(v.shape[:-1], dtype=torch.int64)
    for i in range(8):
        word |= (v[..., i] & 0xF) << (4 * i)
    return torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)


def from_awq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group: int) -> Int4Weight:
    K = qweight.shape[0]
    codes = _unpack_words(qweight, AWQ_ORDER)          # [K, N]
    zeros = _unpack_words(qzeros, AWQ_ORDER).float()   # [K/g, N]
    N = codes.shape[1]
    return Int4Weight(_pack(codes.t().contiguous()), scales.t().to(torch.bfloat16).contiguous(),
                      zeros.t().to(torch.bfloat16).contiguous(), N, K, group)


def from_gptq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group: int,
              g_idx: Optional[torch.Tensor] = None) -> "Int4Weight | torch.Tensor":
    """AutoGPTQ tensors -> Int4Weight, or a bf16 [N, K] matrix for act-order checkpoints."""
    K = qweight.shape[0] * 8
    codes = _unpack_words(qweight.t().contiguous()).t()  # [K, N]: nibble i of word r is k = 8r + i
    zeros = _unpack_words(qzeros).float() + 1.0          # stored as zero - 1
    N = codes.shape[1]
    if g_idx is not None and not torch.equal(g_idx.long(), torch.arange(K) // group):
        s = scales.float()[g_idx.long()]                  # [K, N]
        z = zeros[g_idx.long()]
        return ((codes.float() - z) * s).t().to(torch.bfloat16).contiguous()
    return Int4Weight(_pack(codes.t().contiguous()), scales.t().to(torch.bfloat16).contiguous(),
                      zeros.t().to(torch.bfloat16).contiguous(), N, K, group)


QUANT_METHODS = ("awq", "gptq", "auto-round", "autoround", "intel/auto-round", "quip", "bitsandbytes", "squeezellm",
                 "modelopt", "mxfp4")


def checkpoint_quant_config(d: str) -> dict:
    """The quantization config of checkpoint directory ``d``: config.json's ``quantization_config``,
    else ModelOpt's hf_quant_config.json (``{"quantization": {"quant_algo": …}}``)."""
    import json
    import os
    with open(os.path.join(d, "config.json")) as fh:
        qc = json.load(fh).get("quantization_config") or {}
    mo = os.path.join(d, "hf_quant_config.json")
    if not qc and os.path.exists(mo):
        with open(mo) as fh:
            q = json.load(fh).get("quantization") or {}
        if q.get("quant_algo"):
            qc = {"quant_method": "modelopt", **q}
    return qc


def quantized_checkpoint_getter(ck, quant_config: dict):
    """Wrap a checkpoint reader so that ``get("….weight")`` of a quantized linear returns an
    ``Int4Weight`` (or bf16 for act-order GPTQ): GPTQ / AWQ from qweight / qzeros / scales; AutoRound
    from its native weight / scale / zp tensors or from GPTQ-named ones; QuIP (``quant/quip.py``) from
    its lattice codes, dequantized to bf16 here; NVFP4 / FP8 ModelOpt and MXFP4 through ``quant/fp4.py``."""
    method = quant_config.get("quant_method")
    if method in ("modelopt", "mxfp4"):
        from .fp4 import fp4_getter
        return fp4_getter(ck, quant_config)
    if method == "bitsandbytes":
        from .bnb import bnb_getter
        return bnb_getter(ck)
    if method == "squeezellm":
        from .squeezellm import squeezellm_getter
        return squeezellm_getter(ck)
    if method == "quip":
        from .quip import QuipWeight
        stages, seed = int(quant_config.get("stages", 1)), int(quant_config.get("seed", 0))
        keys_q = set(ck.keys())

        def get_quip(name: str):
            base = name[:-7] if name.endswith(".weight") else name
            if base + ".quip_scales" in keys_q:
                sc = ck.get(base + ".quip_scales")
                codes = [ck.get(f"{base}.quip_codes{i}") for i in range(stages)]
                N, K = sc.shape[0], codes[0].shape[1] * 8
                return QuipWeight(codes, sc, N, K, seed).dequantize(torch.float32).to(torch.bfloat16)
            return ck.get(name)
        return get_quip
    if method in ("auto-round", "autoround", "intel/auto-round"):
        from .autoround import from_autoround
        group_ar = int(quant_config.get("group_size", 128))
        if int(quant_config.get("bits", 4)) != 4:
            raise ValueError(f"{method}: only 4-bit checkpoints are supported")
        keys_ar = set(ck.keys())

        def get_ar(name: str):
            if name.endswith(".weight"):
                base = name[:-7]
                if base + ".scale" in keys_ar:  # native naming: the packed int32 words under .weight
                    zp = ck.get(base + ".zp") if base + ".zp" in keys_ar else None
                    return from_autoround(ck.get(name), ck.get(base + ".scale"), zp, group_ar)
                if base + ".qweight" in keys_ar:
                    g_idx = ck.get(base + ".g_idx") if base + ".g_idx" in keys_ar else None
                    return from_gptq(ck.get(base + ".qweight"), ck.get(base + ".qzeros"), ck.get(base + ".scales"),
                                     group_ar, g_idx)
            return ck.get(name)
        return get_ar
    bits = int(quant_config.get("bits", quant_config.get("w_bit", 4)))
    group = int(quant_config.get("group_size", quant_config.get("q_group_size", 128)))
    if bits != 4:
        raise ValueError(f"{method}: only 4-bit checkpoints are supported (got {bits} bits)")
    keys = set(ck.keys())

    def get(name: str):
        if name.endswith(".weight") and name[:-7] + ".qweight" in keys:
            base = name[:-7]
            qw, qz, sc = ck.get(base + ".qweight"), ck.get(base + ".qzeros"), ck.get(base + ".scales")
            if method == "awq":
                return from_awq(qw, qz, sc, group)
            g_idx = ck.get(base + ".g_idx") if base + ".g_idx" in keys else None
            return from_gptq(qw, qz, sc, group, g_idx)
        return ck.get(name)
    return get
