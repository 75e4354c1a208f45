"""AutoRound: signed-gradient optimization of the rounding of 4-bit group-quantized weights, and the
AutoRound checkpoint formats.

Quantizer (after Cheng et al., "Optimize Weight Rounding via Signed Gradient Descent for the
Quantization of LLMs", 2023): asymmetric int4 with one (scale, zero) per group of ``group`` input
columns. Besides the round-to-nearest grid, three tensors are learned per layer:

* V in [-0.5, 0.5], one per weight, added before rounding: q = clamp(round(W / s + V) + z, 0, 15);
* alpha, beta in [0.5, 1], one each per group, shrinking the group's max and min before the scale
  and zero are derived from them: s = (alpha max - beta min) / 15, z = round(-beta min / s).

The objective is the layer's output reconstruction error on calibration inputs X [n, K]:
mean((X W^T - X Wq^T)^2). Rounding passes gradients straight through; every parameter takes
signed steps lr * sign(grad) with lr decaying linearly to 0 over ``iters`` steps, and the
parameters of the best loss seen are kept. The result is an ``Int4Weight`` (canonical layout), so
the int4 GEMV / dequant + GEMM kernels serve it.

Checkpoint formats (the reference reads them in core/quantizer/gollek-quantizer-autoround/…/autoround/
AutoRoundConfig.java:33-60, AutoRoundDequantizer.java:10-60):

* native: ``<layer>.weight`` int32 [N / 8, K] (word [r, k] holds rows 8r..8r+7 of column k, nibble i
  = row 8r + i), ``<layer>.scale`` float32 [N, K / g], ``<layer>.zp`` int32 [N, K / g] (plain
  integers; absent for symmetric checkpoints, whose zero point is 8);
* GPTQ naming (``qweight`` / ``qzeros`` / ``scales``): the AutoGPTQ layout, read by ``from_gptq``.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from .int4 import Int4Weight, _pack


def _ste_round(x: torch.Tensor) -> torch.Tensor:
    return x + (torch.round(x) - x).detach()


def _fake_quant(wg: torch.Tensor, mn0: torch.Tensor, mx0: torch.Tensor, v: torch.Tensor, a: torch.Tensor,
                b: torch.Tensor):
    mx = mx0 * a.clamp(0.5, 1.0)
    mn = mn0 * b.clamp(0.5, 1.0)
    s = ((mx - mn) / 15.0).clamp_min(1e-8)
    z = torch.clamp(_ste_round(-mn / s), 0, 15)
    q = torch.clamp(_ste_round(wg / s[..., None] + v) + z[..., None], 0, 15)
    return (q - z[..., None]) * s[..., None], q, s, z


def quantize_autoround(w: torch.Tensor, X: torch.Tensor, group: int = 128, iters: int = 200,
                       lr: Optional[float] = None, batch: int = 512, seed: int = 0) -> Int4Weight:
    """Quantize ``w`` [N, K] with calibration inputs ``X`` [n, K] (rows are tokens)."""
    N, K = w.shape
    if K % group:
        raise ValueError(f"group size {group} must divide K={K}")
    W = w.detach().float()
    Xf = X.detach().float().to(W.device)
    wg = W.reshape(N, K // group, group)
    mn0 = wg.amin(-1).clamp_max(0.0)   # keep 0 representable (as round-to-nearest does in practice)
    mx0 = wg.amax(-1).clamp_min(0.0)
    v = torch.zeros_like(wg, requires_grad=True)
    a = torch.ones(N, K // group, device=W.device, requires_grad=True)
    b = torch.ones(N, K // group, device=W.device, requires_grad=True)
    lr0 = lr if lr is not None else 1.0 / iters
    g = torch.Generator(device="cpu").manual_seed(seed)
    ref_full = Xf @ W.t()
    best = None
    for t in range(iters + 1):
        if Xf.shape[0] > batch:
            rows = torch.randint(0, Xf.shape[0], (batch,), generator=g).to(W.device)
            xb, ref = Xf[rows], ref_full[rows]
        else:
            xb, ref = Xf, ref_full
        wq, _, _, _ = _fake_quant(wg, mn0, mx0, v, a, b)
        loss = ((xb @ wq.reshape(N, K).t() - ref) ** 2).mean()
        lv = float(loss.detach())
        if best is None or lv < best[0]:
            best = (lv, v.detach().clone(), a.detach().clone(), b.detach().clone())
        if t == iters:
            break
        for p in (v, a, b):
            p.grad = None
        loss.backward()
        step = lr0 * (1.0 - t / iters)
        with torch.no_grad():
            v -= step * torch.sign(v.grad)
            v.clamp_(-0.5, 0.5)
            a -= step * torch.sign(a.grad)
            a.clamp_(0.5, 1.0)
            b -= step * torch.sign(b.grad)
            b.clamp_(0.5, 1.0)
    _, v, a, b = best
    with torch.no_grad():
        _, q, s, z = _fake_quant(wg, mn0, mx0, v, a, b)
    codes = q.reshape(N, K).round().clamp(0, 15)
    return Int4Weight(_pack(codes), s.to(torch.bfloat16), z.to(torch.bfloat16), N, K, group)


# ---------------------------------------------------------------------------- native checkpoint format
def _unpack_rows(words: torch.Tensor) -> torch.Tensor:
    """int32 [N / 8, K] -> int [N, K]: nibble i of word [r, k] is row 8r + i."""
    x = words.to(torch.int64) & 0xFFFFFFFF
    nib = torch.stack([(x >> (4 * i)) & 0xF for i in range(8)], 1)       # [N/8, 8, K]
    return nib.reshape(words.shape[0] * 8, words.shape[1])


def _pack_rows(codes: torch.Tensor) -> torch.Tensor:
    N, K = codes.shape
    c = codes.to(torch.int64).reshape(N // 8, 8, K)
    word = torch.zeros(N // 8, K, dtype=torch.int64)
    for i in range(8):
        word |= (c[:, i] & 0xF) << (4 * i)
    return torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)


def from_autoround(weight: torch.Tensor, scale: torch.Tensor, zp: Optional[torch.Tensor], group: int) -> Int4Weight:
    """AutoRound native tensors -> Int4Weight (zp None: symmetric, zero point 8)."""
    codes = _unpack_rows(weight)
    N, K = codes.shape
    z = torch.full(scale.shape, 8.0) if zp is None else zp.float()
    return Int4Weight(_pack(codes), scale.float().to(torch.bfloat16), z.to(torch.bfloat16), N, K, group)


def to_autoround(w: Int4Weight) -> Dict[str, torch.Tensor]:
    """Int4Weight -> AutoRound native tensors {"weight", "scale", "zp"} (asymmetric int4)."""
    if w.nf4 or w.zero is None:
        raise ValueError("only asymmetric int4 weights have an AutoRound form")
    q = w.q.to(torch.int64)
    codes = torch.stack([q & 0xF, q >> 4], -1).reshape(w.N, w.K)
    return {"weight": _pack_rows(codes.cpu()), "scale": w.scale.float().cpu().contiguous(),
            "zp": w.zero.float().round().to(torch.int32).cpu().contiguous()}
