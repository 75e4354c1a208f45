"""AWQ: activation-aware per-input-channel scaling before 4-bit group quantization.

After Lin et al., "AWQ: Activation-aware Weight Quantization for LLM Compression and Acceleration",
2023. Weights on input channels that see large activations matter most; scaling such a channel up by
s_k before quantization (and the activation down by 1 / s_k, folded into the producer of the input)
shrinks its relative rounding error. With mean |x_k| over calibration inputs, s = mean|x|^alpha,
normalized so that sqrt(max s * min s) = 1, and alpha searched on a grid in [0, 1) for the least
output error of all linears that read the same input (q/k/v, or gate/up):
    sum_i || X W_i^T - (X diag(1/s)) Q(W_i diag(s))^T ||^2.
Q is round-to-nearest asymmetric int4 per group of input columns (``quantize_rtn``).

``to_awq`` writes the AutoAWQ GEMM tensors (qweight / qzeros / scales), which ``from_awq`` reads. The
reference converts such checkpoints (core/quantizer/gollek-quantizer-awq/…/awq/AWQDequantizer.java,
AWQSafetensorConverter.java) but ships no scale search.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .int4 import AWQ_ORDER, Int4Weight, _pack_words, quantize_rtn


def awq_search(ws: Sequence[torch.Tensor], X: torch.Tensor, group: int = 128, grid: int = 20,
               tie: Optional[Tuple[int, int]] = None) -> Tuple[torch.Tensor, List[Int4Weight]]:
    """Per-input-channel scales s [K] for linears ``ws`` ([N_i, K]) that read inputs X [n, K], and
    their int4 weights Q(W_i diag(s)); the caller divides the inputs by s (folds 1/s upstream).
    ``tie`` = (G, D): channel h * D + d shares its scale with every head h' of the same group of G
    heads (geometric mean), so that 1/s can be folded into a GQA value projection."""
    Xf = X.detach().float()
    Wf = [w.detach().float() for w in ws]
    ref = [Xf @ w.t() for w in Wf]
    xmean = Xf.abs().mean(0).clamp_min(1e-8)
    best = None
    for i in range(grid):
        alpha = i / grid
        s = xmean.pow(alpha)
        if tie is not None:
            G, D = tie
            ls = s.log().view(-1, G, D).mean(1, keepdim=True).expand(-1, G, D)
            s = ls.reshape(-1).exp()
        s = s / (s.max() * s.min()).sqrt()
        qs = [quantize_rtn(w * s[None, :], group) for w in Wf]
        err = sum(float(((Xf @ (q.dequantize() / s[None, :]).t() - r) ** 2).sum()) for q, r in zip(qs, ref))
        if best is None or err < best[0]:
            best = (err, s, qs)
    return best[1], best[2]


def to_awq(w: Int4Weight) -> Dict[str, torch.Tensor]:
    """Int4Weight (asymmetric int4) -> AutoAWQ GEMM tensors {"qweight", "qzeros", "scales"}."""
    if w.nf4 or w.zero is None:
        raise ValueError("only asymmetric int4 weights have an AWQ form")
    q = w.q.to(torch.int64).cpu()
    codes = torch.stack([q & 0xF, q >> 4], -1).reshape(w.N, w.K)          # [N, K]
    return {"qweight": _pack_words(codes.t().contiguous(), AWQ_ORDER),    # [K, N/8]
            "qzeros": _pack_words(w.zero.float().round().t().contiguous().cpu(), AWQ_ORDER),  # [K/g, N/8]
            "scales": w.scale.t().contiguous().to(torch.float16).cpu()}   # [K/g, N]
