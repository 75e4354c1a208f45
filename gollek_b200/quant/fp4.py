"""FP4 (e2m1) weights: NVFP4 and OCP MXFP4 block formats, their checkpoint layouts, and the fp32
oracle of a block-scaled FP4 matmul.

The reference exposes one FP4 entry point, ``gollek_blackwell_matmul_fp4(C, A, B, M, K, N, alpha,
beta)`` (kernel/blackwell/gollek-kernel-blackwell/…/blackwell/binding/BlackwellBinding.java:67,353-361),
whose CPU fallback is a plain fp32 matmul; it names no storage format. The formats here are the
two that Blackwell's block-scaled tensor-core MMA consumes:

* e2m1 element: sign, 2 exponent bits, 1 mantissa bit; magnitudes {0, 0.5, 1, 1.5, 2, 3, 4, 6};
  encoding rounds to nearest with ties to the even code and saturates at 6;
* NVFP4: one e4m3 scale per 16 consecutive elements of a row, times one fp32 scale per tensor
  chosen so that the largest block scale lands on e4m3's maximum (amax / (6 * 448));
* MXFP4 (OCP Microscaling v1.0): one e8m0 scale (a power of two, biased by 127) per 32 elements,
  2^(floor(log2 amax) - 2), so the block maximum falls in [4, 8) before saturation.

Codes are packed two per byte, element 2i in the low nibble. Checkpoint tensors of a linear
``<name>.weight`` [N, K]:

* NVFP4 (ModelOpt naming, ``quantization_config = {"quant_method": "modelopt", "quant_algo":
  "NVFP4"}``): ``<name>.weight`` uint8 [N, K / 2], ``<name>.weight_scale`` float8_e4m3fn [N, K / 16],
  ``<name>.weight_scale_2`` fp32 scalar, optionally ``<name>.input_scale`` (activation scale for
  W4A4 execution; unused by weight-only loading). ModelOpt FP8 checkpoints (``quant_algo":
  "FP8"``) hold ``<name>.weight`` e4m3 with a per-tensor or per-channel ``<name>.weight_scale``;
* MXFP4 (``{"quant_method": "mxfp4"}``): ``<name>.weight_blocks`` uint8 [N, K / 32, 16] and
  ``<name>.weight_scales`` uint8 [N, K / 32] (e8m0).

Loading dequantizes to bf16; the block-scaled FP4 tensor-core GEMM (``tcgen05.mma`` kind::mxf4nvf4)
is not built, so FP4 checkpoints serve through the bf16 GEMMs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

E2M1_MAX = 6.0
E4M3_MAX = 448.0
# magnitude of codes 0..7; codes 8..15 are the negatives (sign in bit 3)
E2M1_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
E2M1_VALUES = torch.cat([E2M1_MAG, -E2M1_MAG])
_MID = (E2M1_MAG[1:] + E2M1_MAG[:-1]) / 2  # decision points between neighbouring magnitudes


def encode_e2m1(x: torch.Tensor) -> torch.Tensor:
    """Nearest e2m1 code (uint8 0..15) of each element of x; ties go to the even code, magnitudes
    above 6 saturate to 6, NaN encodes as +0."""
    a = torch.nan_to_num(x.float().abs(), nan=0.0)
    lo = torch.bucketize(a, _MID, right=False)   # the lower neighbour where a sits on a midpoint
    hi = torch.bucketize(a, _MID, right=True)    # the upper neighbour there
    code = torch.where((lo != hi) & (hi % 2 == 0), hi, lo)
    neg = (x.float() < 0) & (code > 0)
    return (code + 8 * neg.to(code.dtype)).to(torch.uint8)


def decode_e2m1(code: torch.Tensor) -> torch.Tensor:
    return E2M1_VALUES[code.long()]


def pack_nibbles(code: torch.Tensor) -> torch.Tensor:
    """[..., 2m] codes -> [..., m] bytes, element 2i in the low nibble."""
    c = code.to(torch.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).contiguous()


def unpack_nibbles(b: torch.Tensor) -> torch.Tensor:
    b = b.to(torch.uint8)
    return torch.stack([b & 0xF, b >> 4], -1).flatten(-2)


@dataclass
class FP4Weight:
    """Block-scaled e2m1 weight [N, K]: ``codes`` uint8 [N, K] (unpacked), ``scale`` per block
    (fp32 values of the e4m3 / e8m0 scales), ``global_scale`` (NVFP4; 1 for MXFP4)."""
    codes: torch.Tensor
    scale: torch.Tensor
    global_scale: float
    block: int
    fmt: str  # "nvfp4" | "mxfp4"

    @property
    def shape(self):
        return tuple(self.codes.shape)

    def nbytes(self) -> int:
        return self.codes.numel() // 2 + self.scale.numel() + (4 if self.fmt == "nvfp4" else 0)

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        s = self.scale.float().repeat_interleave(self.block, 1)[:, : self.codes.shape[1]]
        return (decode_e2m1(self.codes) * s * self.global_scale).to(dtype)


def quantize_nvfp4(w: torch.Tensor, global_scale: Optional[float] = None) -> FP4Weight:
    W = w.detach().float().cpu()
    N, K = W.shape
    if K % 16:
        raise ValueError("NVFP4 needs K % 16 == 0")
    if global_scale is None:
        global_scale = max(float(W.abs().max()), 1e-30) / (E2M1_MAX * E4M3_MAX)
    blk = W.view(N, K // 16, 16)
    sb = (blk.abs().amax(-1) / E2M1_MAX / global_scale).clamp(max=E4M3_MAX)
    sq = sb.to(torch.float8_e4m3fn).float()       # the stored e4m3 block scale
    eff = torch.where(sq > 0, sq * global_scale, torch.ones_like(sq))
    codes = encode_e2m1(blk / eff[..., None]).view(N, K)
    return FP4Weight(codes, sq, float(global_scale), 16, "nvfp4")


def quantize_mxfp4(w: torch.Tensor) -> FP4Weight:
    W = w.detach().float().cpu()
    N, K = W.shape
    if K % 32:
        raise ValueError("MXFP4 needs K % 32 == 0")
    blk = W.view(N, K // 32, 32)
    amax = blk.abs().amax(-1)
    e = torch.where(amax > 0, torch.floor(torch.log2(amax.clamp_min(1e-38))) - 2, torch.full_like(amax, -127.0))
    e = e.clamp(-127, 127)
    scale = torch.exp2(e)
    codes = encode_e2m1(blk / scale[..., None]).view(N, K)
    return FP4Weight(codes, scale, 1.0, 32, "mxfp4")


def to_tensors(q: FP4Weight) -> Dict[str, torch.Tensor]:
    """FP4Weight -> checkpoint tensors, keyed by suffix of ``<name>.weight``."""
    N, K = q.codes.shape
    if q.fmt == "nvfp4":
        return {"": pack_nibbles(q.codes), "_scale": q.scale.to(torch.float8_e4m3fn),
                "_scale_2": torch.tensor(q.global_scale, dtype=torch.float32)}
    e8 = (torch.log2(q.scale).round() + 127).clamp(0, 254).to(torch.uint8)
    return {"_blocks": pack_nibbles(q.codes).view(N, K // 32, 16), "_scales": e8}


def from_nvfp4(packed: torch.Tensor, scale: torch.Tensor, scale_2: torch.Tensor) -> FP4Weight:
    codes = unpack_nibbles(packed)
    return FP4Weight(codes, scale.float(), float(scale_2.float().reshape(-1)[0]), 16, "nvfp4")


def from_mxfp4(blocks: torch.Tensor, scales: torch.Tensor) -> FP4Weight:
    N = blocks.shape[0]
    codes = unpack_nibbles(blocks.reshape(N, -1))
    scale = torch.exp2(scales.to(torch.int32).float() - 127.0).view(N, -1)
    return FP4Weight(codes, scale, 1.0, 32, "mxfp4")


def fp4_matmul_reference(x: torch.Tensor, w: FP4Weight, quantize_activations: bool = True) -> torch.Tensor:
    """fp32 oracle of the block-scaled FP4 GEMM y = x @ w^T: with ``quantize_activations`` the rows
    of x are quantized to the weight's format first (W4A4, as the tensor cores consume it)."""
    xf = x.float()
    if quantize_activations:
        qa = quantize_nvfp4(xf) if w.fmt == "nvfp4" else quantize_mxfp4(xf)
        xf = qa.dequantize()
    return xf @ w.dequantize().t()


def fp4_getter(ck, quant_config: dict):
    """``get("….weight")`` for an NVFP4 / FP8 ModelOpt or an MXFP4 checkpoint: quantized linears
    dequantized to bf16, everything else as stored."""
    keys = set(ck.keys())

    def get(name: str):
        if name + "_blocks" in keys and name + "_scales" in keys:
            return from_mxfp4(ck.get(name + "_blocks"), ck.get(name + "_scales")).dequantize().to(torch.bfloat16)
        if name.endswith(".weight") and name + "_scale" in keys:
            t = ck.get(name)
            if name + "_scale_2" in keys and t.dtype == torch.uint8:
                return from_nvfp4(t, ck.get(name + "_scale"), ck.get(name + "_scale_2")).dequantize().to(torch.bfloat16)
            if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
                s = ck.get(name + "_scale").float()
                s = s.reshape(-1, *([1] * (t.dim() - 1))) if s.numel() > 1 else s.reshape(())
                return (t.float() * s).to(torch.bfloat16)
        return ck.get(name)
    return get
