"""GGUF-quantized weight matrices resident on the device in their ggml block format.

A ``QWeight`` is an ``[N, K]`` matrix stored as ``N`` rows of ``K / block`` ggml blocks (Q4_K:
256 weights in 144 bytes; Q8_0: 32 weights in 34 bytes). Because blocks never straddle rows, the
operations the serving graph needs are byte-row operations that never dequantize:

* row slices (column-parallel shards of q/k/v/gate/up, vocab shards of lm_head),
* K slices on block boundaries (row-parallel shards of o_proj/down_proj),
* row concatenation (fused ``w_qkv``) and row interleaving (SwiGLU gate/up groups of 64).

Matmuls with ≤ 16 activation rows run the fused dequant GEMV kernel (csrc/kernels/gguf.cu);
larger ones dequantize into a bf16 scratch matrix and run the tcgen05 GEMM.
"""
from __future__ import annotations

from typing import List, Sequence

import torch

GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 8, 12, 14
BLOCK = {GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210)}


class QWeight:
    def __init__(self, raw: torch.Tensor, N: int, K: int, qtype: int):
        be, bb = BLOCK[qtype]
        if K % be:
            raise ValueError(f"K={K} is not a multiple of the ggml block ({be})")
        self.N, self.K, self.qtype = N, K, qtype
        self.row_bytes = K // be * bb
        self.raw = raw.reshape(N, self.row_bytes)

    @staticmethod
    def from_quantized(qw) -> "QWeight":
        """From ``loaders.gguf.QuantizedWeight`` (raw blocks + shape)."""
        N, K = qw.shape
        return QWeight(qw.raw, N, K, qw.ggml_type)

    @property
    def shape(self):
        return (self.N, self.K)

    @property
    def device(self):
        return self.raw.device

    def nbytes(self) -> int:
        return self.raw.numel()

    def to(self, device=None, dtype=None) -> "QWeight":  # dtype ignored: stays quantized
        return QWeight(self.raw.to(device).contiguous(), self.N, self.K, self.qtype)

    def contiguous(self) -> "QWeight":
        return QWeight(self.raw.contiguous(), self.N, self.K, self.qtype)

    def __getitem__(self, idx) -> "QWeight":
        if isinstance(idx, tuple):  # [:, k0:k1]
            rows, cols = idx
            out = self if rows == slice(None) else self[rows]
            return out.kslice(cols.start or 0, cols.stop if cols.stop is not None else self.K)
        r = self.raw[idx]
        return QWeight(r, r.shape[0], self.K, self.qtype)

    def kslice(self, k0: int, k1: int) -> "QWeight":
        be, bb = BLOCK[self.qtype]
        if k0 % be or k1 % be:
            raise ValueError("K slices must fall on ggml block boundaries")
        r = self.raw[:, k0 // be * bb: k1 // be * bb]
        return QWeight(r.contiguous(), self.N, k1 - k0, self.qtype)

    def dequantize(self) -> torch.Tensor:
        """bf16 [N, K] (on the weight's device; GPU kernel on CUDA, host C++ on CPU)."""
        if self.raw.is_cuda:
            from ..native import cuda_ext
            out = torch.empty(self.N, self.K, dtype=torch.bfloat16, device=self.raw.device)
            cuda_ext().gguf_dequant(out, self.raw.contiguous(), self.qtype)
            return out
        from ..loaders.gguf import dequantize_blocks
        return dequantize_blocks(self.raw.contiguous().view(-1), self.qtype, self.N * self.K).view(self.N, self.K)


def cat_rows(ws: Sequence[QWeight]) -> QWeight:
    if len({(w.K, w.qtype) for w in ws}) != 1:
        raise ValueError("row concatenation needs equal K and type")
    raw = torch.cat([w.raw for w in ws], 0)
    return QWeight(raw, raw.shape[0], ws[0].K, ws[0].qtype)


def interleave_rows(g: QWeight, u: QWeight, group: int = 64) -> QWeight:
    if g.N % group:
        raise ValueError("gate/up rows must be a multiple of the interleave group")
    rg = g.raw.view(g.N // group, group, -1)
    ru = u.raw.view(u.N // group, group, -1)
    raw = torch.stack([rg, ru], 1).reshape(2 * g.N, -1)
    return QWeight(raw, 2 * g.N, g.K, g.qtype)
