"""Hot-op entry points.

Every function dispatches on the device of its inputs: CUDA tensors go to the sm_100a
kernels of ``gollek_b200_C`` (``csrc/kernels``), CPU tensors to the plain-PyTorch
restatement in ``gollek_b200.ops.reference`` (the numerics oracle). There is no silent
fallback: a CUDA tensor with the extension missing raises.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch

from . import reference as ref
from ..native import cuda_ext

EPI_NONE, EPI_RESIDUAL, EPI_SWIGLU, EPI_GEGLU = 0, 1, 2, 3
SWIGLU_GROUP = 64


class _LaunchCounter:
    """Counts sm_100a kernel launches issued through this module (graph replays add their
    captured count via ``add``); the benchmark reports it for its timed region."""

    def __init__(self):
        self.n = 0

    def add(self, k: int = 1) -> None:
        self.n += k

    def reset(self) -> int:
        n, self.n = self.n, 0
        return n


LAUNCHES = _LaunchCounter()


def _C(k: int = 1):
    LAUNCHES.add(k)
    return cuda_ext()


class BoundsCheck:
    """Device bounds checking of the indices kernels read from memory (block-table entries, KV
    slots, token ids): while enabled, an index outside its pool records a status bit and the first
    bad index in a device word, reads use a valid index instead and KV writes are skipped, so a
    corrupt table gives wrong numbers and a readable report instead of a memory fault.

        with ops.BoundsCheck() as bc:
            ...                     # launches
        bc.status()                 # (flags, first bad index or None); flag 4 = out of bounds
    """
    BOUNDS = 1 << 2

    def __init__(self, device: Optional[torch.device] = None):
        self.buf = torch.tensor([0, -1], dtype=torch.int32, device=device or "cuda")

    def __enter__(self) -> "BoundsCheck":
        cuda_ext().set_bounds_status(self.buf)
        return self

    def __exit__(self, *exc) -> None:
        torch.cuda.synchronize(self.buf.device)
        cuda_ext().set_bounds_status(None)

    def status(self):
        flags, idx = (int(v) for v in self.buf.cpu())
        return flags, (None if idx == -1 else idx & 0xFFFFFFFF)

    def reset(self) -> None:
        self.buf.copy_(torch.tensor([0, -1], dtype=torch.int32))


def _cpu(result: torch.Tensor, out: Optional[torch.Tensor]) -> torch.Tensor:
    """CPU path: honour a caller-provided output buffer."""
    if out is None:
        return result
    out.copy_(result)
    return out


# ----------------------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None,
             center: bool = False) -> torch.Tensor:
    """RMSNorm(x) * w; ``center``: bias-free LayerNorm (x - mean) * rsqrt(var + eps) * w."""
    if not x.is_cuda:
        return _cpu(ref.rms_norm(x, w, eps, center=center), out)
    out = torch.empty_like(x) if out is None else out
    _C().rms_norm(out, x, w, float(eps), bool(center))
    return out


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                       out: Optional[torch.Tensor] = None, center: bool = False) -> torch.Tensor:
    """residual += x (in place); returns rms_norm(residual) * w (LayerNorm with ``center``)."""
    if not x.is_cuda:
        return _cpu(ref.fused_add_rms_norm(x, residual, w, eps, center=center), out)
    out = torch.empty_like(x) if out is None else out
    _C().fused_add_rms_norm(out, x, residual, w, float(eps), bool(center))
    return out


# ----------------------------------------------------------------------------- rope + kv
def rope_kv_write(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                  kv_cache: Optional[torch.Tensor], slot_mapping: Optional[torch.Tensor],
                  num_heads: int, num_kv_heads: int, head_dim: int,
                  q_out: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                  q_norm: Optional[torch.Tensor] = None, k_norm: Optional[torch.Tensor] = None,
                  norm_eps: float = 1e-6, kv_scales: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Split fused QKV (+ projection bias), per-head RMSNorm of q and k (QK-norm) when weights
    are given, NeoX RoPE of q and k, paged KV-cache write; returns q [T, H, D]. With ``kv_scales``
    the cache is fp8 e4m3 (uint8 storage): the step's K/V rows go through a bf16 scratch and are
    quantized into their slots with one scale per token and head (``kv_quant_fp8``)."""
    if kv_scales is not None and kv_cache is not None:
        T = qkv.shape[0]
        step = torch.empty(T, 2, num_kv_heads, 1, head_dim, dtype=torch.bfloat16 if qkv.is_cuda else qkv.dtype,
                           device=qkv.device)
        ident = torch.arange(T, dtype=torch.int32, device=qkv.device)
        q = rope_kv_write(qkv, positions, cos_sin, step, ident, num_heads, num_kv_heads, head_dim, q_out, bias,
                          q_norm, k_norm, norm_eps)
        kv_quant_fp8(step.view(T, 2, num_kv_heads, head_dim), slot_mapping, kv_cache, kv_scales)
        return q
    if not qkv.is_cuda:
        return _cpu(ref.rope_kv_write(qkv, positions, cos_sin, kv_cache, slot_mapping,
                                      num_heads, num_kv_heads, head_dim, bias, q_norm, k_norm, norm_eps), q_out)
    T = qkv.shape[0]
    q_out = torch.empty(T, num_heads, head_dim, dtype=qkv.dtype, device=qkv.device) if q_out is None else q_out
    _C().rope_kv_write(q_out, qkv, positions, cos_sin, kv_cache, slot_mapping,
                       num_heads, num_kv_heads, head_dim, bias, q_norm, k_norm, float(norm_eps))
    return q_out


ROPE_FUSED = os.environ.get("GOLLEK_ROPE_FUSED", "1") != "0"


def linear_rope_kv(x: torch.Tensor, w_qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                   kv_cache: Optional[torch.Tensor], slot_mapping: Optional[torch.Tensor], num_heads: int,
                   num_kv_heads: int, head_dim: int) -> torch.Tensor:
    """q = RoPE(x @ Wq^T); RoPE(x @ Wk^T) and x @ Wv^T written into the paged KV cache; returns q
    [T, H, D]. On the GPU with a plain bf16 weight, head_dim 128, full rotary and a bf16 cache this is
    one tcgen05 GEMM whose epilogue rotates q/k and stores q and the cache rows (the [T, (H + 2Hk) D]
    projection is never written); otherwise the projection GEMM followed by ``rope_kv_write``."""
    fused = (ROPE_FUSED and x.is_cuda and isinstance(w_qkv, torch.Tensor) and w_qkv.dtype == torch.bfloat16
             and head_dim == 128 and cos_sin.shape[1] == 128 and x.stride(1) == 1 and x.stride(0) % 8 == 0
             and (kv_cache is None or kv_cache.dtype == torch.bfloat16))
    if not fused:
        qkv = linear(x, w_qkv)
        return rope_kv_write(qkv, positions, cos_sin, kv_cache, slot_mapping, num_heads, num_kv_heads, head_dim)
    q = torch.empty(x.shape[0], num_heads, head_dim, dtype=x.dtype, device=x.device)
    _C().gemm_rope_kv(q, x, w_qkv, positions, cos_sin, kv_cache if slot_mapping is not None else None,
                      slot_mapping if kv_cache is not None else None, num_heads, num_kv_heads)
    return q


# ----------------------------------------------------------------------------- attention
def decode_splits(num_seqs: int, num_kv_heads: int, max_seq_len: int, num_sms: int = 148,
                  block_size: int = 16) -> int:
    """Split-KV factor for the decode kernel: fill ~2 waves of CTAs, keep >= 8 blocks per split."""
    ctas = max(1, num_seqs * num_kv_heads)
    if ctas >= 2 * num_sms:
        return 1
    want = (2 * num_sms + ctas - 1) // ctas
    max_by_len = max(1, (max_seq_len + block_size - 1) // block_size // 8)
    return int(max(1, min(want, max_by_len, 32)))


def paged_decode_attention(q: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                           seq_lens: torch.Tensor, scale: float, num_splits: int = 1,
                           out: Optional[torch.Tensor] = None,
                           workspace: Optional[torch.Tensor] = None, tensor_cores: bool = True,
                           window: int = 0, softcap: float = 0.0,
                           kv_scales: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One query token per sequence: q [B, H, D]. head_dim 128 runs the tensor-core kernel
    (``tensor_cores=False`` selects the CUDA-core kernel, used for other head sizes).
    ``window`` > 0: sliding-window attention; ``softcap`` > 0: tanh soft-capped scores.
    ``kv_scales`` (fp32 [NB, 2, Hk, bs]): ``kv_cache`` holds fp8 e4m3 values (uint8 storage), value =
    e4m3 * scale of its token and head (head_dim 128)."""
    if kv_scales is not None and not q.is_cuda:
        kv_cache = kv_dequant_fp8(kv_cache, kv_scales)
        kv_scales = None
    if not q.is_cuda:
        B = q.shape[0]
        qsl = torch.arange(B + 1, dtype=torch.int32)
        return _cpu(ref.paged_attention(q, kv_cache, block_tables, seq_lens, qsl, scale, window, softcap), out)
    out = torch.empty_like(q) if out is None else out
    if num_splits > 1 and workspace is None:
        B, H, D = q.shape
        workspace = torch.empty(B * H * num_splits * (D + 2), dtype=torch.float32, device=q.device)
    _C(2 if num_splits > 1 else 1).paged_decode_attention(out, q, kv_cache, block_tables, seq_lens, float(scale),
                                                          int(num_splits), workspace, bool(tensor_cores),
                                                          int(window), float(softcap), kv_scales)
    return out


# ---------------------------------------------------------------------------- fp8 KV cache
FP8_E4M3_MAX = 448.0


def kv_dequant_fp8(cache: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 values of an fp8 e4m3 cache (uint8 storage [..., bs, D]) with per-token scales [..., bs]."""
    return cache.view(torch.float8_e4m3fn).float() * scales.unsqueeze(-1)


def kv_quant_fp8(kv: torch.Tensor, slots: torch.Tensor, cache: torch.Tensor, scales: torch.Tensor) -> None:
    """Write the step's K/V rows kv [T, 2, Hk, D] into an fp8 e4m3 cache (uint8 [NB, 2, Hk, bs, D])
    at ``slots``: per (token, K/V, head) scale = absmax / 448, values round-to-nearest saturating."""
    if kv.is_cuda:
        _C().kv_quant_fp8(kv.contiguous(), slots, cache, scales)
        return
    T, _, Hk, D = kv.shape
    bs = cache.shape[3]
    x = kv.float()
    amax = x.abs().amax(-1)
    scl = torch.where(amax > 0, amax / FP8_E4M3_MAX, torch.ones_like(amax))
    q = (x / scl.unsqueeze(-1)).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        cache[s // bs, :, :, s % bs] = q[t]
        scales[s // bs, :, :, s % bs] = scl[t]


def kv_dequant_blocks(cache: torch.Tensor, scales: torch.Tensor, block_tables: torch.Tensor):
    """bf16 copy of the blocks an fp8 cache's ``block_tables`` [n, mb] reference, as a [n * mb]-block
    cache, with the matching [n, mb] table (prefill attention over an fp8 cache)."""
    n, mb = block_tables.shape
    ids = block_tables.reshape(-1).contiguous()
    if not cache.is_cuda:
        NB = cache.shape[0]
        safe = ids.long().clamp(0, NB - 1)
        tmp = kv_dequant_fp8(cache[safe], scales[safe])
    else:
        tmp = torch.empty(n * mb, *cache.shape[1:], dtype=torch.bfloat16, device=cache.device)
        _C().kv_dequant_blocks(cache, scales, ids, tmp)
    table = torch.arange(n * mb, dtype=torch.int32, device=cache.device).view(n, mb)
    return tmp, table


def prefill_block_m(head_dim: int, tensor_cores: bool = True) -> int:
    """Query rows per CTA of the prefill kernel (128 on the tcgen05 path for head_dim 64 / 128, 64 on
    the mma.sync path)."""
    return 128 if (tensor_cores and head_dim in (64, 128)) else 64


def prefill_tiles(query_start: list, block_m: int = 64) -> torch.Tensor:
    """(sequence, query offset) pairs of the 64-row query tiles the prefill kernel runs."""
    tiles = []
    for b in range(len(query_start) - 1):
        ql = query_start[b + 1] - query_start[b]
        for off in range(0, ql, block_m):
            tiles.append((b, off))
    return torch.tensor(tiles, dtype=torch.int32).view(-1, 2)


# Share of the softmax exponentials the two-tile prefill kernel evaluates on the FMA pipe instead of
# MUFU: 0 none, 1 every fourth column, 2 every second column.
PREFILL_EMU = int(os.environ.get("GOLLEK_PREFILL_EMU", "1"))


def prefill_schedule(query_start: list, seq_lens: list, H: int, Hk: int, head_dim: int,
                     tensor_cores: bool = True, form: Optional[str] = None) -> torch.Tensor:
    """Work list of the prefill kernel for one batch.

    head_dim 64 / 128 on tensor cores: int32 [n, 4] rows (sequence, query offset of slot 0, of slot 1 or
    -1, (pair << 16) | head), one per CTA of the two-tile kernel, heaviest first. Two forms:
    head pairs (pair = 1: heads h, h+1 of one GQA group over the same 128 query rows, each K/V tile
    loaded once for both; needs an even group size) and row-tile pairs (pair = 0: one head, two
    consecutive query tiles, which stay active over nearly the same KV tiles). Head pairs are used
    whenever the group size allows: measured on B200 they are faster at every prompt shape. A KV
    tile costs nearly as much with one active slot as with two, so pairing tile i with tile n-1-i
    (every item the same n+1 KV tiles) lost even on a short single prompt (1 x 1088 tokens,
    32 / 8 heads: 0.0389 vs 0.0348 ms). ``form`` ("pairs" / "rows") forces a form. Otherwise: the [n, 2] (sequence, offset) 64-row tiles of the mma.sync kernel."""
    if not (tensor_cores and head_dim in (64, 128)):
        return prefill_tiles(query_start, 64)
    seqs = []
    for b in range(len(query_start) - 1):
        ql = query_start[b + 1] - query_start[b]
        L = int(seq_lens[b])
        ctx0 = L - ql
        offs = list(range(0, ql, 128))
        cost = [(min(L, ctx0 + o + 128) + 127) // 128 for o in offs]
        seqs.append((b, offs, cost))
    pairable = (H // Hk) % 2 == 0
    pair = pairable and form != "rows"
    items = []
    for b, offs, cost in seqs:
        if pair:
            for o, c in zip(offs, cost):
                for h in range(0, H, 2):
                    items.append((2 * c, b, o, o, (1 << 16) | h))
        else:
            for k in range(0, len(offs), 2):
                j = k + 1 if k + 1 < len(offs) else k
                c = max(cost[k], cost[j])  # the two slots advance together: the longer one sets the time
                o1 = offs[j] if j != k else -1
                for h in range(H):
                    items.append((c, b, offs[k], o1, h))
    items.sort(key=lambda t: -t[0])
    return torch.tensor([t[1:] for t in items], dtype=torch.int32).view(-1, 4)


def paged_prefill_attention(q: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                            seq_lens: torch.Tensor, query_start: torch.Tensor, scale: float,
                            tiles: Optional[torch.Tensor] = None,
                            out: Optional[torch.Tensor] = None, tensor_cores: bool = True,
                            window: int = 0, softcap: float = 0.0, emu: Optional[int] = None,
                            kv_scales: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Varlen causal attention of new tokens q [T, H, D] over the paged KV (prefix + new).
    head_dim 64 / 128 runs on tcgen05/TMEM (the two-tile kernel when ``tiles`` is a ``prefill_schedule``
    work list); other sizes on mma.sync (64-row tiles). ``window`` > 0: sliding-window attention;
    ``softcap`` > 0: tanh soft-capped scores. With ``kv_scales`` (fp8 cache) the referenced blocks
    are dequantized into a bf16 copy first."""
    if kv_scales is not None:
        kv_cache, block_tables = kv_dequant_blocks(kv_cache, kv_scales, block_tables)
    if not q.is_cuda:
        return _cpu(ref.paged_attention(q, kv_cache, block_tables, seq_lens, query_start, scale, window, softcap),
                    out)
    out = torch.empty_like(q) if out is None else out
    if tiles is None:
        tiles = prefill_schedule(query_start.tolist(), seq_lens.tolist(), q.shape[1], kv_cache.shape[2],
                                 q.shape[2], tensor_cores).to(q.device)
    _C().paged_prefill_attention(out, q, kv_cache, block_tables, seq_lens, query_start, tiles, float(scale),
                                 bool(tensor_cores), int(window), float(softcap),
                                 PREFILL_EMU if emu is None else int(emu))
    return out


# ----------------------------------------------------------------------------- GEMM
_PLAN_CACHE: dict = {}


def gemm_plan(M: int, N: int, K: int, epi: int = EPI_NONE) -> tuple:
    """(tile width, split-K factor) the tcgen05 GEMM uses for this shape."""
    key = (M, N, K, epi)
    p = _PLAN_CACHE.get(key)
    if p is None:
        p = tuple(cuda_ext().gemm_plan(M, N, K, epi))
        _PLAN_CACHE[key] = p
    return p


_SM_RESERVE = [0]


def set_gemm_sm_reserve(n: int) -> None:
    """SMs the persistent GEMM grids leave free (for a collective running beside them)."""
    _SM_RESERVE[0] = int(n)
    cuda_ext().set_gemm_sm_reserve(int(n))


def _gemm(out, a, w, residual, epi, bn):
    M, K = a.shape
    N = w.shape[0]
    splits, ws = 1, None
    if bn == 0:
        bn, splits = gemm_plan(M, N, K, epi)
    if splits > 1:  # fp32 partial sums, reduced (with the epilogue) by a second kernel
        ws = torch.empty(splits * M * N, dtype=torch.float32, device=a.device)
    _C(2 if splits > 1 else 1).gemm_bf16(out, a, w, residual, epi, bn, None, 0, splits, ws)


GGUF_GEMV_MAX_TOKENS = 4
Q4K_FUSED = os.environ.get("GOLLEK_Q4K_FUSED", "1") != "0"
GGUF_CHUNK_BYTES = 48 << 20  # bf16 scratch per chunk: stays resident in the 126 MB L2


def _qlinear(a: torch.Tensor, w, out: Optional[torch.Tensor], swiglu: bool) -> torch.Tensor:
    """Matmul with a GGUF-quantized weight.

    <= GGUF_GEMV_MAX_TOKENS rows: fused dequant GEMV (weights decoded in registers).
    More rows, Q4_K: the tcgen05 GEMM decodes the super-blocks into its shared-memory B tiles.
    More rows, other types: the weight is dequantized in row chunks of <= 48 MB of bf16 into a scratch buffer
    that stays in L2, and each chunk is multiplied by the tcgen05 GEMM right away, so HBM sees
    the quantized bytes once plus the activations.
    """
    M = a.shape[0]
    N = w.N
    n_out = N // 2 if swiglu else N
    if not a.is_cuda:
        wd = w.dequantize().to(a.dtype)
        y = ref.gemm_swiglu(a, wd, SWIGLU_GROUP) if swiglu else ref.gemm(a, wd)
        return _cpu(y, out)
    out = torch.empty(M, n_out, dtype=a.dtype, device=a.device) if out is None else out
    if M <= GGUF_GEMV_MAX_TOKENS and (not swiglu or w.qtype == 12):
        _C().gguf_gemv(out, a, w.raw, w.qtype, N, w.K, swiglu)
        return out
    if w.qtype == 12 and Q4K_FUSED and N % 128 == 0 and w.K % 256 == 0 and a.stride(1) == 1 and a.stride(0) % 8 == 0:
        # Q4_K: super-blocks decoded inside the tcgen05 GEMM (HBM reads 0.5625 bytes per weight)
        ext = cuda_ext()
        splits = ext.gemm_q4k_splits(M, N, w.K)
        ws = torch.empty(splits * M * N, dtype=torch.float32, device=a.device) if splits > 1 else None
        _C(2 if splits > 1 else 1).gemm_q4k(out, a, w.raw, N, w.K, EPI_SWIGLU if swiglu else EPI_NONE, splits, ws)
        return out
    rows = max(128, GGUF_CHUNK_BYTES // (2 * w.K) // 128 * 128)
    scratch = torch.empty(min(rows, N), w.K, dtype=torch.bfloat16, device=a.device)
    ext = cuda_ext()
    for n0 in range(0, N, rows):
        n1 = min(N, n0 + rows)
        wd = scratch[: n1 - n0]
        _C().gguf_dequant(wd, w.raw[n0:n1], w.qtype)
        if swiglu:
            _gemm(out[:, n0 // 2: n1 // 2], a, wd, None, EPI_SWIGLU, 0)
        else:
            _gemm(out[:, n0:n1], a, wd, None, EPI_NONE, 0)
    return out


INT4_GEMV_MAX_TOKENS = 8


def _is_int4(w) -> bool:
    return type(w).__name__ == "Int4Weight"


def _int4_linear(a: torch.Tensor, w, out: Optional[torch.Tensor], swiglu: bool) -> torch.Tensor:
    """Matmul with a 4-bit group-quantized weight (GPTQ / AWQ / NF4): fused dequant GEMV for up
    to 8 tokens; otherwise L2-sized row chunks dequantized to bf16 and fed to the tcgen05 GEMM."""
    M, N = a.shape[0], w.N
    n_out = N // 2 if swiglu else N
    if not a.is_cuda:
        wd = w.dequantize(a.dtype)
        y = ref.gemm_swiglu(a, wd, SWIGLU_GROUP) if swiglu else ref.gemm(a, wd)
        return _cpu(y, out)
    out = torch.empty(M, n_out, dtype=a.dtype, device=a.device) if out is None else out
    if M <= INT4_GEMV_MAX_TOKENS:
        _C().int4_gemv(out, a, w.q, w.scale, w.zero, N, w.K, w.group, w.nf4, swiglu)
        return out
    rows = max(128, GGUF_CHUNK_BYTES // (2 * w.K) // 128 * 128)
    scratch = torch.empty(min(rows, N), w.K, dtype=torch.bfloat16, device=a.device)
    for n0 in range(0, N, rows):
        n1 = min(N, n0 + rows)
        wd = scratch[: n1 - n0]
        _C().int4_dequant(wd, w.q[n0:n1], w.scale[n0:n1], None if w.zero is None else w.zero[n0:n1], n1 - n0, w.K,
                          w.group, w.nf4)
        if swiglu:
            _gemm(out[:, n0 // 2: n1 // 2], a, wd, None, EPI_SWIGLU, 0)
        else:
            _gemm(out[:, n0:n1], a, wd, None, EPI_NONE, 0)
    return out


def _is_q(w) -> bool:
    return type(w).__name__ == "QWeight"


def _is_fp8(w) -> bool:
    return type(w).__name__ == "FP8Weight"


def linear_fp8(a: torch.Tensor, w, out: Optional[torch.Tensor] = None, swiglu: bool = False) -> torch.Tensor:
    """bf16 activations × block-scaled FP8 weight: quantise a per (token, 128 group), FP8 GEMM."""
    from ..quant import fp8 as F8
    M = a.shape[0]
    n_out = w.N // 2 if swiglu else w.N
    if not a.is_cuda:
        xq, sa = F8.quantize_act(a)
        y = F8.reference_gemm(xq, sa, w)
        if swiglu:
            y = y.view(M, -1, 2, SWIGLU_GROUP)
            y = (torch.nn.functional.silu(y[:, :, 0]) * y[:, :, 1]).reshape(M, -1)
        return _cpu(y.to(a.dtype), out)
    out = torch.empty(M, n_out, dtype=torch.bfloat16, device=a.device) if out is None else out
    xq, sa = F8.quantize_act(a)
    LAUNCHES.add(1)
    epi = EPI_SWIGLU if swiglu else EPI_NONE
    ext = cuda_ext()
    splits = ext.gemm_fp8_splits(M, w.N, w.K, epi)
    ws = cnt = None
    if splits > 1:  # fp32 split partials, summed by each tile's last unit (zeroed tile counters)
        ws = torch.empty(splits * M * w.N, dtype=torch.float32, device=a.device)
        cnt = torch.zeros(((M + 127) // 128) * (w.N // 128), dtype=torch.int32, device=a.device)
    _C().gemm_fp8(out, xq, sa, w.q, w.scale, epi, splits, ws, cnt)
    return out


def linear(a: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None, bn: int = 0) -> torch.Tensor:
    """a [M, K] @ w[N, K]^T (+ residual), bf16 in/out, fp32 accumulate (tcgen05 on GPU).
    ``w`` may be a GGUF-quantized ``QWeight`` (see gollek_b200.quant.gguf_weights)."""
    if _is_fp8(w):
        y = linear_fp8(a, w, out)
        if residual is not None:
            y.add_(residual)
        return y
    if _is_q(w) or _is_int4(w):
        y = (_qlinear if _is_q(w) else _int4_linear)(a, w, out, False)
        if residual is not None:
            y.add_(residual)
        return y
    if not a.is_cuda:
        return _cpu(ref.gemm(a, w, residual), out)
    M, N = a.shape[0], w.shape[0]
    out = torch.empty(M, N, dtype=a.dtype, device=a.device) if out is None else out
    epi = EPI_RESIDUAL if residual is not None else EPI_NONE
    _gemm(out, a, w, residual, epi, bn)
    return out


def linear_swiglu(a: torch.Tensor, w_gate_up: torch.Tensor, out: Optional[torch.Tensor] = None,
                  bn: int = 0, act: str = "silu") -> torch.Tensor:
    """act(a @ Wg^T) * (a @ Wu^T) with gate/up rows interleaved by ``interleave_gate_up``;
    ``act`` is ``silu`` (SwiGLU, Llama) or ``gelu_tanh`` (GeGLU, Gemma), fused in the GEMM epilogue."""
    if act != "silu" and (_is_q(w_gate_up) or _is_fp8(w_gate_up) or _is_int4(w_gate_up)):
        # quantized GeGLU: plain product, gate activation on the host-side graph
        y = linear(a, w_gate_up)
        return _copy_into(ref.glu_interleaved(y, SWIGLU_GROUP, act).to(a.dtype), out)
    if _is_q(w_gate_up):
        return _qlinear(a, w_gate_up, out, True)
    if _is_int4(w_gate_up):
        return _int4_linear(a, w_gate_up, out, True)
    if _is_fp8(w_gate_up):
        return linear_fp8(a, w_gate_up, out, swiglu=True)
    if not a.is_cuda:
        return _cpu(ref.gemm_swiglu(a, w_gate_up, SWIGLU_GROUP, act), out)
    M, N = a.shape[0], w_gate_up.shape[0]
    out = torch.empty(M, N // 2, dtype=a.dtype, device=a.device) if out is None else out
    _gemm(out, a, w_gate_up, None, EPI_SWIGLU if act == "silu" else EPI_GEGLU, bn)
    return out


def _copy_into(y: torch.Tensor, out: Optional[torch.Tensor]) -> torch.Tensor:
    if out is None:
        return y
    out.copy_(y)
    return out


interleave_gate_up = ref.interleave_gate_up


def silu_mul(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not x.is_cuda:
        return _cpu(ref.silu_mul(x), out)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device) if out is None else out
    _C().silu_mul(out, x)
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None,
              scale: float = 1.0) -> torch.Tensor:
    """Row gather (x ``scale``: Gemma multiplies embeddings by sqrt(hidden))."""
    if _is_q(table):
        if not table.raw.is_cuda:
            return _cpu(table.dequantize()[ids.long()].to(torch.float32) * scale, out)
        if table.qtype != 8:
            return embedding(ids, table.dequantize(), out, scale)
        out = torch.empty(ids.shape[0], table.K, dtype=torch.bfloat16, device=table.device) if out is None else out
        _C().embedding_q8_0(out, ids, table.raw, table.N)
        if scale != 1.0:
            out.mul_(scale)
        return out
    if not table.is_cuda:
        return _cpu(ref.embedding(ids, table) * scale, out)
    out = torch.empty(ids.shape[0], table.shape[1], dtype=table.dtype, device=table.device) if out is None else out
    _C().embedding(out, ids, table, float(scale))
    return out


# ----------------------------------------------------------------------------- sampling
def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not logits.is_cuda:
        return _cpu(logits.float().argmax(-1), out)
    out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device) if out is None else out
    _C().argmax(out, logits)
    return out


def apply_penalties(logits: torch.Tensor, triples: torch.Tensor, repetition: torch.Tensor,
                    frequency: torch.Tensor, presence: torch.Tensor) -> torch.Tensor:
    """In-place penalties on fp32 logits from unique (row, token, count) triples."""
    if not logits.is_cuda:
        return ref.apply_penalties_triples(logits, triples, repetition, frequency, presence)
    _C().apply_penalties(logits, triples, repetition, frequency, presence)
    return logits


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           min_p: torch.Tensor, seeds: torch.Tensor, offsets: torch.Tensor,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not logits.is_cuda:
        return _cpu(ref.sample(logits, temperature, top_k, top_p, min_p, seeds, offsets), out)
    out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device) if out is None else out
    _C().sample(out, logits, temperature, top_k, top_p, min_p, seeds, offsets)
    return out


def attention_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


# ---------------------------------------------------------------------------- MoE (K12)
_MOE_WS = {}


def _moe_workspace(device: torch.device, ints: int) -> torch.Tensor:
    """Per-device int32 routing workspace, zero-filled once (the plan kernel re-zeroes its counters
    after each use, so the same buffer serves every layer, step and CUDA-graph replay)."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    ws = _MOE_WS.get(key)
    if ws is None or ws.numel() < ints:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("MoE workspace must be created before CUDA-graph capture (run one eager step)")
        ws = torch.zeros(max(ints, 1 << 16), dtype=torch.int32, device=device)
        _MOE_WS[key] = ws
    return ws


def moe_route_ref(x: torch.Tensor, router: torch.Tensor, top_k: int, renorm: bool = True, **route):
    """fp32 top-k routing: (ids [T, k] int64, weights [T, k] fp32); ``route`` holds the scoring
    options of ``ops.reference.moe_route`` (scoring, bias, n_group, topk_group, scale)."""
    return ref.moe_route(x.float() @ router.float().t(), top_k, renorm, **route)


MOE_TC_ROUTER_MIN_EXPERTS = 32


def fused_moe(x: torch.Tensor, router: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor, top_k: int,
              e0: int = 0, e_loc: Optional[int] = None, renorm: bool = True,
              out: Optional[torch.Tensor] = None, scoring: str = "softmax", bias: Optional[torch.Tensor] = None,
              n_group: int = 1, topk_group: int = 1, scale: float = 1.0,
              routing: Optional[dict] = None, expert_map: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Mixture-of-experts FFN over the local experts [e0, e0 + e_loc) of ``router.shape[0]``.

    w_gu [e_loc * 2F, H]: per expert, gate/up rows interleaved in groups of 64 (SwiGLU epilogue);
    w_down [e_loc * H, F]. Returns Σ over the token's top-k experts that are local of
    weight · down(silu(gate) · up) — under expert parallelism a partial sum that the following
    tensor-parallel all-reduce completes. Routing: softmax top-k (Mixtral), or with
    ``scoring="sigmoid"`` DeepSeek-V3's bias-corrected, group-limited choice (``bias`` fp32 [E],
    ``n_group`` / ``topk_group``) with weights times ``scale``. A ``routing`` dict receives the
    chosen expert ids and weights ("ids" [T, k], "wts" [T, k]). ``expert_map`` (int32 [E]) places
    logical expert e (router row e) in physical slot expert_map[e]: routing is computed over the
    logical experts, the weights and the returned ids are physical (expert-parallel re-placement)."""
    route = dict(scoring=scoring, bias=bias, n_group=n_group, topk_group=topk_group, scale=scale)
    T, H = x.shape
    E = router.shape[0]
    e_loc = E if e_loc is None else e_loc
    F_ = w_down.shape[1]
    if not x.is_cuda:
        ids, w = moe_route_ref(x, router, top_k, renorm, **route)
        if expert_map is not None:
            ids = expert_map.to(ids.device).long()[ids]
        if routing is not None:
            routing.update(ids=ids, wts=w)
        acc = torch.zeros(T, H, dtype=torch.float32)
        for le in range(e_loc):
            sel = ids == (e0 + le)
            rows = sel.any(-1).nonzero().flatten()
            if rows.numel() == 0:
                continue
            xe = x.index_select(0, rows)
            he = ref.gemm_swiglu(xe, w_gu[le * 2 * F_:(le + 1) * 2 * F_])
            ye = ref.gemm(he, w_down[le * H:(le + 1) * H]).float()
            acc.index_add_(0, rows, ye * (w * sel).sum(-1).index_select(0, rows)[:, None])
        return _cpu(acc.to(x.dtype), out)
    C = _C()
    out = torch.empty_like(x) if out is None else out
    if T == 0:
        return out
    cap = C.moe_capacity_rows(T, top_k, e_loc)
    ws = _moe_workspace(x.device, C.moe_ws_ints(T, top_k, e_loc))
    dev = x.device
    ids = torch.empty(T * top_k, dtype=torch.int32, device=dev)
    dest = torch.empty(T * top_k, dtype=torch.int32, device=dev)
    wts = torch.empty(T * top_k, dtype=torch.float32, device=dev)
    xp = torch.empty(cap, H, dtype=x.dtype, device=dev)
    hp = torch.empty(cap, F_, dtype=x.dtype, device=dev)
    _, _, splits = C.moe_plan(T, top_k, E, e_loc, H, F_)
    # many experts: the router GEMM (T x E x H) runs on tensor cores into an fp32 scratch first
    logits = (torch.empty(C.moe_logit_splits(T, E, H), T, E, dtype=torch.float32, device=dev)
              if E >= MOE_TC_ROUTER_MIN_EXPERTS else None)
    if splits > 1:  # down projection split over K: fp32 partials summed by the combine kernel
        yp = None
        ypart = torch.empty(splits * cap * H, dtype=torch.float32, device=dev)
    else:
        yp = torch.empty(cap, H, dtype=x.dtype, device=dev)
        ypart = None
    C.moe_forward(out, x, router, w_gu, w_down, ws, ids, wts, dest, xp, hp, xp if yp is None else yp, ypart,
                  top_k, renorm, e0, e_loc, 0 if scoring == "softmax" else 1, bias, n_group, topk_group, float(scale),
                  expert_map, logits)
    LAUNCHES.add(7 if logits is not None else 6)
    if routing is not None:
        routing.update(ids=ids.view(T, top_k), wts=wts.view(T, top_k))
    return out


# ---------------------------------------------------------------------------- KV block transfer
def kv_gather_blocks(cache: torch.Tensor, block_ids: torch.Tensor) -> torch.Tensor:
    """packed [L, n, 2, Hk, bs, D] = cache[:, block_ids] (P/D hand-off of one sequence's KV)."""
    if not cache.is_cuda:
        return cache[:, block_ids.long()].contiguous()
    L = cache.shape[0]
    packed = torch.empty(L, block_ids.numel(), *cache.shape[2:], dtype=cache.dtype, device=cache.device)
    _C().kv_blocks(cache, packed, block_ids.to(cache.device, torch.int32), True)
    return packed


# ---------------------------------------------------------------------------- gated delta rule (K14)
def gdn_scan(proj: torch.Tensor, state: torch.Tensor, slots: torch.Tensor, reset: torch.Tensor,
             query_start: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor, Hg: int,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gated delta rule over the varlen token batch. proj [T, >= 4*Hg*D + 2*Hg] holds q | k | v | g |
    a | b per token; state [slots, Hg, D, D] fp32 (this layer) is read (unless ``reset``) and
    updated per sequence; returns raw o [T, Hg, D]."""
    if not proj.is_cuda:
        return _cpu(ref.gdn_scan(proj, state, slots, reset, query_start, a_log, dt_bias, Hg).to(proj.dtype), out)
    T, D = proj.shape[0], state.shape[-1]
    out = torch.empty(T, Hg, D, dtype=proj.dtype, device=proj.device) if out is None else out
    _C().gdn_scan(proj, out, state, slots, reset, query_start, a_log, dt_bias, Hg)
    return out


def gdn_gated_norm(o: torch.Tensor, g: torch.Tensor, w: torch.Tensor, eps: float,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y [T, Hg*D] = RMSNorm_head(o) * w * silu(g) for o [T, Hg, D] and g a [T, Hg*D] view."""
    if not o.is_cuda:
        return _cpu(ref.gdn_gated_norm(o, g, w, eps), out)
    T, Hg, D = o.shape
    out = torch.empty(T, Hg * D, dtype=o.dtype, device=o.device) if out is None else out
    _C().gdn_gated_norm(out, o, g, w, Hg, float(eps))
    return out


def kv_key_norms(cache: torch.Tensor, block_ids: torch.Tensor) -> torch.Tensor:
    """Mean key L2 norm of each listed block over layers, KV heads and tokens (KV eviction scoring)."""
    ids = block_ids.to(cache.device, torch.int32)
    if not cache.is_cuda:
        k = cache[:, ids.long(), 0].float()                 # [L, n, Hk, bs, D]
        return torch.linalg.vector_norm(k, dim=-1).mean(dim=(0, 2, 3))
    return _C().kv_key_norms(cache, ids)


def kv_scatter_blocks(cache: torch.Tensor, block_ids: torch.Tensor, packed: torch.Tensor) -> None:
    """cache[:, block_ids] = packed (the receiving side of a hand-off)."""
    if not cache.is_cuda:
        cache[:, block_ids.long()] = packed.to(cache.dtype)
        return
    _C().kv_blocks(cache, packed.to(cache.device, cache.dtype).contiguous(), block_ids.to(cache.device, torch.int32),
                   False)
