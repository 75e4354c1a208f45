"""TurboQuant: data-oblivious vector quantization of KV vectors (random rotation + Lloyd-Max scalar
codes), its unbiased inner-product form, and a 2.5-bit KV format with outlier channels.

After Zandieh et al., "TurboQuant: Online Vector Quantization with Near-optimal Distortion Rate",
2025; the reference's Java version: core/quantizer/gollek-quantizer-turboquant/…/turboquant/
TurboQuantKVCache.java:13-50, TurboQuantEngine.java, LloydMaxCodebook.java.

* MSE quantizer (``TurboQuantMSE``): x = |x| u. A fixed random rotation R makes every coordinate of
  sqrt(d) R u follow the same known density f(t) ~ (1 - t^2 / d)^((d - 3) / 2) on |t| < sqrt(d)
  (close to N(0, 1)); each coordinate gets the b-bit Lloyd-Max code of that density (centroids
  computed here by Lloyd iterations on the exact density). |x| is kept in fp16. Reconstruction:
  |x| R^T c / sqrt(d). No calibration, so tokens are quantized online, one at a time.
* Inner-product quantizer (``TurboQuantProd``): the MSE quantizer at b - 1 bits plus a 1-bit
  sketch of the residual r: sign(S r) with a Gaussian S, and |r|. For any query y,
  <y, x_mse> + |r| sqrt(pi / 2) / d <S y, sign(S r)> is an unbiased estimate of <y, x>.
* KV format (``quantize_kv`` / ``dequantize_kv``): per head, the ``outliers`` channels with the
  largest RMS over the given tokens get their own MSE quantizer at b + 1 bits, the rest b bits
  (head_dim 128, 32 channels at 3 bits + 96 at 2 bits + two fp16 norms = 2.5 bits per value).
  Used to compress prefix-cache snapshots (``engine/persistence.py``, ``compress="turboquant"``).

Rotations: a random-sign Hadamard transform for power-of-two sizes, else a seeded random orthogonal
matrix (QR of a Gaussian matrix).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from functools import lru_cache
from typing import Dict, Optional

import torch


@lru_cache(maxsize=None)
def lloyd_max(bits: int, dim: int, iters: int = 300) -> torch.Tensor:
    """Centroids [2^bits] (ascending) of the MSE-optimal scalar quantizer for one coordinate of
    sqrt(dim) times a uniformly random unit vector in R^dim."""
    L = min(math.sqrt(dim), 9.0)
    t = torch.linspace(-L, L, 40001, dtype=torch.float64)
    if dim > 3:
        dens = torch.clamp(1.0 - t * t / dim, min=0.0) ** ((dim - 3) / 2.0)
    else:
        dens = torch.ones_like(t)
    dens = dens / dens.sum()
    cdf = dens.cumsum(0)
    n = 1 << bits
    c = torch.stack([t[int(torch.searchsorted(cdf, torch.tensor((i + 0.5) / n, dtype=torch.float64)))]
                     for i in range(n)])
    for _ in range(iters):
        edges = (c[1:] + c[:-1]) / 2
        cell = torch.bucketize(t, edges)
        num = torch.zeros(n, dtype=torch.float64).index_add_(0, cell, dens * t)
        den = torch.zeros(n, dtype=torch.float64).index_add_(0, cell, dens)
        c = torch.where(den > 0, num / den.clamp_min(1e-300), c)
    return c.float()


def _rotation(dim: int, seed: int) -> torch.Tensor:
    """Orthogonal [dim, dim] matrix (rows: the rotated coordinates)."""
    g = torch.Generator().manual_seed(seed)
    if dim & (dim - 1) == 0:
        h = torch.ones(1, 1)
        while h.shape[0] < dim:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
        signs = (torch.randint(0, 2, (dim,), generator=g) * 2 - 1).float()
        return h / math.sqrt(dim) * signs[None, :]
    q, r = torch.linalg.qr(torch.randn(dim, dim, generator=g, dtype=torch.float64))
    return (q * torch.sign(torch.diagonal(r))[None, :]).float()


def _pack(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """uint8 codes [n, m] (< 2^bits) -> uint8 [n, ceil(m * bits / 8)]."""
    n, m = codes.shape
    sh = torch.arange(bits, device=codes.device)
    b = ((codes.to(torch.int64)[..., None] >> sh) & 1).reshape(n, m * bits)
    pad = (-b.shape[1]) % 8
    if pad:
        b = torch.cat([b, torch.zeros(n, pad, dtype=b.dtype, device=b.device)], 1)
    return (b.view(n, -1, 8) << torch.arange(8, device=codes.device)).sum(-1).to(torch.uint8)


def _unpack(packed: torch.Tensor, bits: int, m: int) -> torch.Tensor:
    n = packed.shape[0]
    b = (packed.to(torch.int64)[..., None] >> torch.arange(8, device=packed.device)) & 1
    b = b.reshape(n, -1)[:, :m * bits].view(n, m, bits)
    return (b << torch.arange(bits, device=packed.device)).sum(-1).to(torch.uint8)


class TurboQuantMSE:
    """b-bit MSE quantizer of vectors in R^dim."""

    def __init__(self, dim: int, bits: int, seed: int = 0):
        self.dim, self.bits, self.seed = dim, bits, seed
        self.R = _rotation(dim, seed)
        self.c = lloyd_max(bits, dim)

    def quantize(self, x: torch.Tensor) -> Dict[str, torch.Tensor]:
        xf = x.float().reshape(-1, self.dim)
        norm = xf.norm(dim=1)
        y = (xf / norm.clamp_min(1e-30)[:, None]) @ self.R.to(xf.device).t() * math.sqrt(self.dim)
        c = self.c.to(xf.device)
        idx = torch.bucketize(y, (c[1:] + c[:-1]) / 2).to(torch.uint8)
        return {"codes": _pack(idx, self.bits), "norm": norm.to(torch.float16)}

    def dequantize(self, q: Dict[str, torch.Tensor]) -> torch.Tensor:
        idx = _unpack(q["codes"], self.bits, self.dim).long()
        y = self.c.to(idx.device)[idx] / math.sqrt(self.dim)
        return (y @ self.R.to(idx.device)) * q["norm"].float()[:, None]


class TurboQuantProd:
    """b-bit quantizer with unbiased inner products: MSE at b - 1 bits + 1-bit residual sketch."""

    def __init__(self, dim: int, bits: int, seed: int = 0):
        if bits < 2:
            raise ValueError("the inner-product form needs at least 2 bits")
        self.dim, self.bits = dim, bits
        self.mse = TurboQuantMSE(dim, bits - 1, seed)
        self.S = torch.randn(dim, dim, generator=torch.Generator().manual_seed(seed + 7919))

    def quantize(self, x: torch.Tensor) -> Dict[str, torch.Tensor]:
        xf = x.float().reshape(-1, self.dim)
        q = self.mse.quantize(xf)
        r = xf - self.mse.dequantize(q)
        sign = (r @ self.S.to(xf.device).t() >= 0).to(torch.uint8)
        return {**q, "qjl": _pack(sign, 1), "rnorm": r.norm(dim=1).to(torch.float16)}

    def inner(self, y: torch.Tensor, q: Dict[str, torch.Tensor]) -> torch.Tensor:
        """Estimates [m, n] of <y_i, x_j> for queries y [m, dim] and the n quantized vectors."""
        yf = y.float().reshape(-1, self.dim)
        base = yf @ self.mse.dequantize(q).t()
        s = _unpack(q["qjl"], 1, self.dim).float() * 2 - 1                       # [n, dim] in {-1, 1}
        proj = yf @ self.S.to(yf.device).t()                                     # [m, dim]
        return base + math.sqrt(math.pi / 2) / self.dim * (proj @ s.t()) * q["rnorm"].float()[None, :]


@dataclass
class KVQuantized:
    """Vectors [n, dim] of one head in the outlier-split form."""
    outlier_idx: torch.Tensor      # int16 [k] channels coded with the finer quantizer
    hi: Dict[str, torch.Tensor]
    lo: Dict[str, torch.Tensor]
    dim: int
    bits: int

    def nbytes(self) -> int:
        return 2 * self.outlier_idx.numel() + sum(t.numel() * t.element_size()
                                                  for d in (self.hi, self.lo) for t in d.values())


def quantize_kv(x: torch.Tensor, bits: int = 2, outliers: int = 32, seed: int = 0,
                outlier_idx: Optional[torch.Tensor] = None) -> KVQuantized:
    """x [n, dim] (one head's keys or values over n tokens): the ``outliers`` channels of largest RMS
    (or the given ones) at bits + 1, the others at ``bits``."""
    n, dim = x.shape
    xf = x.float()
    if outlier_idx is None:
        outlier_idx = xf.pow(2).mean(0).topk(outliers).indices.sort().values
    mask = torch.zeros(dim, dtype=torch.bool, device=x.device)
    mask[outlier_idx.long().to(x.device)] = True
    hi = TurboQuantMSE(outliers, bits + 1, seed).quantize(xf[:, mask])
    lo = TurboQuantMSE(dim - outliers, bits, seed + 1).quantize(xf[:, ~mask])
    return KVQuantized(outlier_idx.to(torch.int16).cpu(), hi, lo, dim, bits)


def dequantize_kv(q: KVQuantized, seed: int = 0) -> torch.Tensor:
    k = q.outlier_idx.numel()
    dev = q.lo["norm"].device
    mask = torch.zeros(q.dim, dtype=torch.bool, device=dev)
    mask[q.outlier_idx.long().to(dev)] = True
    out = torch.empty(q.lo["norm"].shape[0], q.dim, device=dev)
    out[:, mask] = TurboQuantMSE(k, q.bits + 1, seed).dequantize(q.hi)
    out[:, ~mask] = TurboQuantMSE(q.dim - k, q.bits, seed + 1).dequantize(q.lo)
    return out
