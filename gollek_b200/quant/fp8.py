"""Block-scaled FP8 (e4m3) weights and activations.

Weights: 128 x 128 blocks, one fp32 scale per block (amax / 448). Activations: quantised on the
fly per token and 128-column group (1 x 128), one fp32 scale per group. The GEMM
(csrc/kernels/gemm_fp8.cu) applies ``sa[m, kb] * sb[n/128, kb]`` per 128-deep K block. Covers the
reference's FP8 quantisation (runner/safetensor/gollek-safetensor-quantization/…/quantizer/FP8Quantizer.java)
with the block granularity the 70B serving config asks for.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch

FP8_MAX = 448.0


class FP8Weight:
    def __init__(self, q: torch.Tensor, scale: torch.Tensor, N: int, K: int):
        self.q, self.scale, self.N, self.K = q, scale, N, K

    @property
    def shape(self):
        return (self.N, self.K)

    @property
    def device(self):
        return self.q.device

    def nbytes(self) -> int:
        return self.q.numel() + self.scale.numel() * 4

    def contiguous(self) -> "FP8Weight":
        return self

    def dequantize(self) -> torch.Tensor:
        s = self.scale.repeat_interleave(128, 0)[: self.N].repeat_interleave(128, 1)[:, : self.K]
        return (self.q.float() * s).to(torch.bfloat16)


def quantize_weight(w: torch.Tensor) -> FP8Weight:
    """bf16 [N, K] → FP8Weight (GPU kernel on CUDA; plain torch on CPU)."""
    N, K = w.shape
    if K % 128:
        raise ValueError("fp8 weights need K % 128 == 0")
    nb = (N + 127) // 128
    if w.is_cuda:
        from ..native import cuda_ext
        q = torch.empty(N, K, dtype=torch.float8_e4m3fn, device=w.device)
        s = torch.empty(nb, K // 128, dtype=torch.float32, device=w.device)
        cuda_ext().weight_quant_fp8(q, s, w.contiguous().bfloat16())
        return FP8Weight(q, s, N, K)
    wf = w.float()
    pad = torch.zeros(nb * 128, K)
    pad[:N] = wf
    blk = pad.view(nb, 128, K // 128, 128)
    s = (blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / FP8_MAX)
    q = (blk / s[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(nb * 128, K)[:N]
    return FP8Weight(q.contiguous(), s, N, K)


def quantize_act(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] → (e4m3 [M, K], fp32 scales [M, K/128]) with 1 x 128 groups."""
    M, K = x.shape
    if x.is_cuda:
        from ..native import cuda_ext
        q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(M, K // 128, dtype=torch.float32, device=x.device)
        cuda_ext().act_quant_fp8(q, s, x)
        return q, s
    g = x.float().view(M, K // 128, 128)
    s = g.abs().amax(-1).clamp_min(1e-10) / FP8_MAX
    q = (g / s[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(M, K)
    return q, s


def reference_gemm(xq: torch.Tensor, sa: torch.Tensor, w: FP8Weight) -> torch.Tensor:
    """fp32 oracle of the block-scaled GEMM: (x8 * sa) @ (w8 * sb)^T."""
    M, K = xq.shape
    xa = xq.float().view(M, K // 128, 128) * sa[..., None]
    return xa.view(M, K) @ w.dequantize().float().t()


def quantize_checkpoint_fp8(src: str, dst: str) -> None:
    """safetensors checkpoint → safetensors with e4m3 linear weights + ``<name>_scale`` block scales."""
    import json
    import os
    import shutil
    from ..loaders.safetensors import SafetensorsCheckpoint, save_file
    ck = SafetensorsCheckpoint(src)
    out = {}
    for k in ck.keys():
        t = ck.get(k)
        if t.dim() == 2 and "proj" in k and t.shape[1] % 128 == 0:
            fw = quantize_weight(t.bfloat16())
            out[k] = fw.q
            out[k + "_scale"] = fw.scale
        else:
            out[k] = t
    os.makedirs(dst, exist_ok=True)
    save_file(out, os.path.join(dst, "model.safetensors"), {"quantization": "fp8-e4m3-block128"})
    cfgp = os.path.join(src if os.path.isdir(src) else os.path.dirname(src), "config.json")
    if os.path.exists(cfgp):
        shutil.copy(cfgp, os.path.join(dst, "config.json"))
