"""Incoherence processing + E8 lattice vector quantization of weight matrices (QuIP#-style).

Method (after Tseng et al., "QuIP#: Even Better LLM Quantization with Hadamard Incoherence and
Lattice Codebooks", 2024; the reference's Java version: core/quantizer/gollek-quantizer-quip/…/quip/
QuipQuantizer.java:8-60, E8Codebook.java, RandomHadamard.java):

1. Incoherence. W~ = H_L diag(s_L) W diag(s_R) H_R^T, with random +-1 sign vectors s_L, s_R and
   orthonormal Hadamard transforms H applied block-diagonally (blocks of the largest power of two,
   at most 4096, that divides the dimension, so that shapes like 14336 = 7 x 2048 need no padding).
   The transform spreads outliers, so every 8-weight block looks roughly Gaussian.
2. Lattice vector quantization of W~ in blocks of 8 consecutive weights of a row, with one fp16 scale
   per 64 weights: block / scale goes to its nearest point of the E8 lattice (Conway & Sloane's
   decoder: E8 = D8 u (D8 + 1/2), D8 = integer vectors with an even sum), kept inside the ball of
   squared norm 10, whose 56,881 lattice points fit a 16-bit index: 2 bits per weight for the codes
   + 0.25 for the scales. ``stages=2`` quantizes the residual again at a third of the scale (the E8
   covering radius is 1, so a residual of a point decoded at scale s has squared norm <= s^2, inside
   the ball at s / 3): 4.25 bits per weight.
3. Dequantization: W~ = sum over stages of scale * point, then W = diag(s_L) H_L W~ H_R diag(s_R)
   (H symmetric and orthonormal).

No calibration data is needed. Serving dequantizes to bf16 at load time (as the reference does).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

BALL = 10.0          # squared-norm bound of the codebook points
GROUP = 64           # weights per scale
STAGE_SHRINK = 3.0   # scale ratio between consecutive residual stages


def _enumerate_ball() -> torch.Tensor:
    """All E8 points with squared norm <= BALL, as doubled integer coordinates [P, 8] (int8)."""
    pts = []
    for half in (False, True):
        vals = torch.tensor([-5, -3, -1, 1, 3, 5] if half else [-6, -4, -2, 0, 2, 4, 6], dtype=torch.int16)
        grid = torch.cartesian_prod(*([vals] * 8))                  # doubled coordinates
        n2 = (grid.float() ** 2).sum(1) / 4.0
        keep = n2 <= BALL + 1e-6
        grid = grid[keep]
        s = grid.sum(1)
        # integer coset: coordinates even (doubled), coordinate sum even <=> doubled sum % 4 == 0;
        # half-integer coset: the coordinate sum (doubled sum / 2) even <=> doubled sum % 4 == 0
        grid = grid[(s % 4) == 0]
        pts.append(grid)
    return torch.cat(pts).to(torch.int8)


_BOOK: Optional[torch.Tensor] = None
_KEYS: Optional[torch.Tensor] = None
_ORDER: Optional[torch.Tensor] = None


def codebook() -> torch.Tensor:
    """[P, 8] float32 lattice points of the ball (P = 56,881), in index order."""
    global _BOOK, _KEYS, _ORDER
    if _BOOK is None:
        dbl = _enumerate_ball()
        _BOOK = dbl.float() / 2.0
        keys = _key(dbl.long())
        _KEYS, _ORDER = torch.sort(keys)
    return _BOOK


def _key(dbl: torch.Tensor) -> torch.Tensor:
    """Doubled coordinates in [-6, 6] -> a unique int64 key (base-16 digits)."""
    k = torch.zeros(dbl.shape[:-1], dtype=torch.int64, device=dbl.device)
    for i in range(8):
        k = k * 16 + (dbl[..., i] + 8)
    return k


def _index(points: torch.Tensor) -> torch.Tensor:
    """Lattice points (inside the ball) -> codebook indices."""
    codebook()
    keys = _key(torch.round(points * 2).long())
    ks, order = _KEYS.to(points.device), _ORDER.to(points.device)
    pos = torch.searchsorted(ks, keys).clamp_max(ks.numel() - 1)
    if not bool((ks[pos] == keys).all()):
        raise RuntimeError("point outside the E8 codebook ball")
    return order[pos]


def _nearest_d8(x: torch.Tensor) -> torch.Tensor:
    r = torch.round(x)
    odd = (r.sum(-1) % 2) != 0
    if bool(odd.any()):
        err = x - r
        i = err.abs().argmax(-1, keepdim=True)
        step = torch.where(err.gather(-1, i) >= 0, 1.0, -1.0)
        r = torch.where(odd[..., None], r.scatter_add(-1, i, step), r)
    return r


def nearest_e8(x: torch.Tensor) -> torch.Tensor:
    """Nearest E8 lattice point of each row of x [..., 8] (Conway & Sloane)."""
    a = _nearest_d8(x)
    b = _nearest_d8(x - 0.5) + 0.5
    da = ((x - a) ** 2).sum(-1, keepdim=True)
    db = ((x - b) ** 2).sum(-1, keepdim=True)
    return torch.where(da <= db, a, b)


def _nearest_in_ball(x: torch.Tensor) -> torch.Tensor:
    p = nearest_e8(x)
    out = (p * p).sum(-1) > BALL + 1e-6
    shrink = 1.0
    while bool(out.any()):  # rare: pull the block towards the origin until its point is inside
        shrink *= 0.9
        p[out] = nearest_e8(x[out] * shrink)
        out = (p * p).sum(-1) > BALL + 1e-6
    return p


def hadamard_block(n: int) -> int:
    """Largest power of two <= 4096 that divides n."""
    b = 1
    while b < 4096 and n % (2 * b) == 0:
        b *= 2
    return b


def _fwht(x: torch.Tensor) -> torch.Tensor:
    """Orthonormal fast Walsh-Hadamard transform over the last dimension (a power of two)."""
    n = x.shape[-1]
    y = x.reshape(-1, n)
    h = 1
    while h < n:
        y = y.view(-1, n // (2 * h), 2, h)
        a, b = y[:, :, 0, :], y[:, :, 1, :]
        y = torch.stack([a + b, a - b], 2).reshape(-1, n)
        h *= 2
    return (y / (n ** 0.5)).reshape(x.shape)


def block_hadamard(x: torch.Tensor, block: int) -> torch.Tensor:
    """Block-diagonal orthonormal Hadamard transform of the last dimension (its own inverse)."""
    *lead, n = x.shape
    return _fwht(x.reshape(*lead, n // block, block)).reshape(*lead, n)


def random_signs(n: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(0, 2, (n,), generator=g) * 2 - 1).float()


def incoherent(w: torch.Tensor, seed: int) -> torch.Tensor:
    """W~ = H_L diag(s_L) W diag(s_R) H_R for the given seed."""
    N, K = w.shape
    sl, sr = random_signs(N, seed).to(w.device), random_signs(K, seed + 1).to(w.device)
    x = sl[:, None] * w.float() * sr[None, :]
    x = block_hadamard(x, hadamard_block(K))
    return block_hadamard(x.t(), hadamard_block(N)).t()


def coherent(wt: torch.Tensor, seed: int) -> torch.Tensor:
    """Inverse of ``incoherent``."""
    N, K = wt.shape
    sl, sr = random_signs(N, seed).to(wt.device), random_signs(K, seed + 1).to(wt.device)
    w = block_hadamard(wt, hadamard_block(K))
    w = block_hadamard(w.t(), hadamard_block(N)).t()
    return sl[:, None] * w * sr[None, :]


@dataclass
class QuipWeight:
    """An [N, K] matrix in the incoherent basis of ``seed``: per stage, int16 lattice indices
    [N, K / 8] (the uint16 index stored in int16) and fp16 scales [N, K / 64] of the first stage."""
    codes: List[torch.Tensor]
    scales: torch.Tensor
    N: int
    K: int
    seed: int

    def nbytes(self) -> int:
        return sum(c.numel() * 2 for c in self.codes) + 2 * self.scales.numel()

    def bits_per_weight(self) -> float:
        return 8.0 * self.nbytes() / (self.N * self.K)

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        cb = codebook().to(self.scales.device)
        s = self.scales.float().repeat_interleave(GROUP // 8, 1)[..., None]     # [N, K/8, 1]
        wt = torch.zeros(self.N, self.K // 8, 8, device=self.scales.device)
        for st, c in enumerate(self.codes):
            wt += cb[c.long() & 0xFFFF] * (s / STAGE_SHRINK ** st)
        return coherent(wt.reshape(self.N, self.K), self.seed).to(dtype)


def quantize_quip(w: torch.Tensor, stages: int = 1, seed: int = 0, scale_grid=(0.9, 1.05, 1.2, 1.35),
                  chunk_rows: int = 256) -> QuipWeight:
    """Quantize an [N, K] matrix (K a multiple of 64): ``stages`` = 1 (2.25 bits per weight) or 2
    (4.25). Each 64-weight group's scale is rms(group) times the factor of ``scale_grid`` with the
    least first-stage squared error."""
    N, K = w.shape
    if K % GROUP:
        raise ValueError(f"K={K} must be a multiple of {GROUP}")
    codebook()
    wt = incoherent(w, seed)
    nb = K // 8
    codes = [torch.empty(N, nb, dtype=torch.int16, device=wt.device) for _ in range(stages)]
    scales = torch.empty(N, K // GROUP, dtype=torch.float16, device=wt.device)
    for r0 in range(0, N, chunk_rows):
        x = wt[r0:r0 + chunk_rows]
        R = x.shape[0]
        g = x.reshape(R, K // GROUP, GROUP)
        rms = g.pow(2).mean(-1).sqrt().clamp_min(1e-12)                          # [R, K/64]
        blocks = x.reshape(R, nb, 8)
        best_err, best_s = None, None
        for f in scale_grid:  # per-group choice of the scale factor
            s = (rms * f).to(torch.float16).float()
            sb = s.repeat_interleave(GROUP // 8, 1)[..., None]
            p = _nearest_in_ball(blocks / sb)
            err = ((blocks - p * sb) ** 2).sum(-1).reshape(R, K // GROUP, GROUP // 8).sum(-1)
            if best_err is None:
                best_err, best_s = err, s
            else:
                better = err < best_err
                best_err = torch.where(better, err, best_err)
                best_s = torch.where(better, s, best_s)
        scales[r0:r0 + R] = best_s.to(torch.float16)
        sb = best_s.repeat_interleave(GROUP // 8, 1)[..., None]
        resid = blocks
        for st in range(stages):
            ss = sb / STAGE_SHRINK ** st
            p = _nearest_in_ball(resid / ss)
            idx = _index(p.reshape(-1, 8)).view(R, nb)
            codes[st][r0:r0 + R] = torch.where(idx >= 32768, idx - 65536, idx).to(torch.int16)
            resid = resid - p * ss
    return QuipWeight(codes, scales, N, K, seed)
