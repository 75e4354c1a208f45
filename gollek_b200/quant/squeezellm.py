"""SqueezeLLM: dense-and-sparse non-uniform weight quantization.

After Kim et al., "SqueezeLLM: Dense-and-Sparse Quantization", 2023 (the reference dequantizes this
format on the CPU: core/quantizer/gollek-quantizer-turboquant/…/turboquant/SqueezeLLMDequantizer.java):

* sparse: the ``outlier_frac`` largest-magnitude weights of the matrix are kept exactly (fp16) in a
  CSR matrix (row pointers, column indices, values);
* dense: every output channel of the rest gets its own 2^bits-entry codebook from a 1-D weighted
  k-means (Lloyd iterations from quantile seeds; the weights are per-input-channel importances,
  e.g. the mean squared calibration activation, else uniform); each weight stores its code.

w[n, k] = lookup_table[n, code[n, k]] + sparse[n, k].

Checkpoint tensors of a linear ``<name>``: ``qweight`` int32 [K / 8, N] (4-bit codes of 8 consecutive
input rows per word, code i in bits 4i..4i+3), ``lookup_table`` [N, 16], and for the sparse part
``dense_ptr`` int32 [N + 1], ``dense_idx`` int32 [nnz] (input column), ``weight_nnz`` fp16 [nnz].
Loading dequantizes to bf16.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch


@dataclass
class SqueezeWeight:
    codes: torch.Tensor     # uint8 [N, K]
    lut: torch.Tensor       # float16 [N, 2^bits]
    ptr: torch.Tensor       # int32 [N + 1]
    idx: torch.Tensor       # int32 [nnz]
    val: torch.Tensor       # float16 [nnz]

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        N, K = self.codes.shape
        w = self.lut.float().gather(1, self.codes.long())
        if self.val.numel():
            rows = torch.repeat_interleave(torch.arange(N), (self.ptr[1:] - self.ptr[:-1]).long())
            w[rows, self.idx.long()] += self.val.float()
        return w.to(dtype)


def quantize_squeezellm(w: torch.Tensor, bits: int = 4, outlier_frac: float = 0.0045,
                        importance: Optional[torch.Tensor] = None, iters: int = 30) -> SqueezeWeight:
    W = w.detach().float().cpu()
    N, K = W.shape
    n_out = int(round(outlier_frac * W.numel()))
    sparse = torch.zeros_like(W, dtype=torch.bool)
    if n_out:
        thr = W.abs().flatten().kthvalue(W.numel() - n_out).values
        sparse = W.abs() > thr
    dense = torch.where(sparse, torch.zeros_like(W), W)
    imp = torch.ones(K) if importance is None else importance.float().cpu().clamp_min(1e-12)
    wt = imp[None, :].expand(N, K) * (~sparse)                           # outliers do not pull centroids
    L = 1 << bits
    qs = torch.linspace(0.5 / L, 1 - 0.5 / L, L)
    c = torch.quantile(dense, qs, dim=1).t().contiguous()               # [N, L] seeds
    for _ in range(iters):
        code = (dense[..., None] - c[:, None, :]).abs().argmin(-1)      # [N, K]
        num = torch.zeros(N, L).scatter_add_(1, code, wt * dense)
        den = torch.zeros(N, L).scatter_add_(1, code, wt)
        c = torch.where(den > 0, num / den.clamp_min(1e-30), c)
    c16 = c.to(torch.float16)
    code = (dense[..., None] - c16.float()[:, None, :]).abs().argmin(-1).to(torch.uint8)
    rows, cols = sparse.nonzero(as_tuple=True)
    counts = torch.bincount(rows, minlength=N)
    ptr = torch.cat([torch.zeros(1, dtype=torch.int64), counts.cumsum(0)]).to(torch.int32)
    return SqueezeWeight(code, c16, ptr, cols.to(torch.int32), W[rows, cols].to(torch.float16))


def to_tensors(q: SqueezeWeight) -> Dict[str, torch.Tensor]:
    """4-bit SqueezeWeight -> checkpoint tensors (suffixes of ``<name>.``)."""
    N, K = q.codes.shape
    if q.lut.shape[1] != 16 or K % 8:
        raise ValueError("the checkpoint form holds 4-bit codes with K a multiple of 8")
    v = q.codes.t().to(torch.int64).reshape(K // 8, 8, N)
    word = torch.zeros(K // 8, N, dtype=torch.int64)
    for i in range(8):
        word |= v[:, i] << (4 * i)
    word = torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)
    return {"qweight": word, "lookup_table": q.lut, "dense_ptr": q.ptr, "dense_idx": q.idx, "weight_nnz": q.val}


def from_tensors(qweight: torch.Tensor, lut: torch.Tensor, ptr: Optional[torch.Tensor] = None,
                 idx: Optional[torch.Tensor] = None, val: Optional[torch.Tensor] = None) -> SqueezeWeight:
    x = qweight.to(torch.int64) & 0xFFFFFFFF                            # [K/8, N]
    codes = torch.stack([(x >> (4 * i)) & 0xF for i in range(8)], 1).reshape(-1, x.shape[1]).t()
    N = codes.shape[0]
    if ptr is None:
        ptr, idx, val = torch.zeros(N + 1, dtype=torch.int32), torch.zeros(0, dtype=torch.int32), torch.zeros(0)
    return SqueezeWeight(codes.to(torch.uint8).contiguous(), lut.to(torch.float16), ptr, idx, val)


def squeezellm_getter(ck):
    """``get("….weight")`` for a SqueezeLLM checkpoint: dense-and-sparse linears as bf16."""
    keys = set(ck.keys())

    def get(name: str):
        base = name[:-7] if name.endswith(".weight") else name
        if base + ".qweight" in keys and base + ".lookup_table" in keys:
            sp = base + ".dense_ptr" in keys
            q = from_tensors(ck.get(base + ".qweight"), ck.get(base + ".lookup_table"),
                             ck.get(base + ".dense_ptr") if sp else None, ck.get(base + ".dense_idx") if sp else None,
                             ck.get(base + ".weight_nnz") if sp else None)
            return q.dequantize(torch.float32).to(torch.bfloat16)
        return ck.get(name)
    return get
