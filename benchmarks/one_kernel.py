"""Run one hot kernel a few times on one shape (small, self-terminating case for ncu captures).

    python benchmarks/one_kernel.py gemm --M 8192 --N 28672 --K 4096 [--swiglu] [--reps 3]
    python benchmarks/one_kernel.py decode --B 256 --ctx 1200
    python benchmarks/one_kernel.py prefill --nseq 4 --L 2048
    python benchmarks/one_kernel.py moe --T 256 --e-loc 1      (Mixtral-8x7B layer, one EP=8 shard)
    python benchmarks/one_kernel.py gdn --nseq 256 --L 1       (gated delta rule decode, 32 heads)
    python benchmarks/one_kernel.py decode_fp8 --B 64 --ctx 4096  (decode over an fp8 e4m3 KV cache)
    python benchmarks/one_kernel.py q6k --M 1 --N 28672 --K 4096  (Q6_K decode GEMV)
    python benchmarks/one_kernel.py fp8gemm --M 64 --N 1280 --K 8192 (block-scaled fp8 GEMM)
    python benchmarks/one_kernel.py norm --M 1344 --K 4096 --residual (residual add + RMSNorm)
The last three also print a CUDA-event time (the repetitions captured as one CUDA graph, so host
launch cost is excluded) and the achieved fraction of the measured HBM copy bandwidth or sustained
bf16 peak (fp8 GEMM: of twice it, the nominal fp8/bf16 ratio). Weights smaller than 256 MB are
cycled through several copies so that the repetitions read HBM, not L2 (126 MB).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from gollek_b200 import ops  # noqa: E402


def _n_copies(weight_bytes: int) -> int:
    """Weight copies cycled through so that consecutive launches stream > 256 MB (twice L2)."""
    return max(1, -(-(256 << 20) // max(1, weight_bytes)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["gemm", "decode", "prefill", "moe", "moe_ds", "gdn", "decode_fp8",
                                     "decode_bf16", "q6k", "q4k", "int4", "fp8gemm", "gemm_bf16", "qkv_rope",
                                     "norm"])
    ap.add_argument("--T", type=int, default=256)
    ap.add_argument("--e-loc", type=int, default=8)
    ap.add_argument("--M", type=int, default=8192)
    ap.add_argument("--N", type=int, default=28672)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--bn", type=int, default=0)
    ap.add_argument("--splits", type=int, default=1, help="gemm_bf16: split-K factor (with --bn or the planned width)")
    ap.add_argument("--swiglu", action="store_true")
    ap.add_argument("--residual", action="store_true")
    ap.add_argument("--B", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=1200)
    ap.add_argument("--nseq", type=int, default=4)
    ap.add_argument("--L", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--emu", type=int, default=None, help="prefill: FMA-pipe exponential share (0, 1, 2)")
    a = ap.parse_args()
    dev = "cuda"
    if a.kind == "gemm":
        x = torch.randn(a.M, a.K, device=dev).bfloat16()
        w = (torch.randn(a.N, a.K, device=dev) * 0.02).bfloat16()
        for _ in range(a.reps):
            (ops.linear_swiglu(x, w, bn=a.bn) if a.swiglu else ops.linear(x, w, bn=a.bn))
    elif a.kind == "moe":
        H, F, E = 4096, 14336, 8
        x = torch.randn(a.T, H, device=dev).bfloat16()
        router = (torch.randn(E, H, device=dev) * 0.02).bfloat16()
        gu = (torch.randn(a.e_loc * 2 * F, H, device=dev) * 0.02).bfloat16()
        dn = (torch.randn(a.e_loc * H, F, device=dev) * 0.02).bfloat16()
        for _ in range(a.reps):
            ops.fused_moe(x, router, gu, dn, 2, e0=0, e_loc=a.e_loc)
    elif a.kind == "moe_ds":
        # one expert-parallel rank (EP8) of a DeepSeek-V3 MoE layer: 32 of 256 experts, H 7168, expert
        # FFN 2048, top-8 sigmoid routing with correction bias inside the 4 best of 8 expert groups
        H, F, E, k = 7168, 2048, 256, 8
        el = a.e_loc if a.e_loc != 8 else 32
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(a.T, H, device=dev, generator=g).bfloat16()
        router = (torch.randn(E, H, device=dev, generator=g) * 0.02).bfloat16()
        bias = torch.randn(E, device=dev, generator=g) * 0.01
        gu = (torch.randn(el * 2 * F, H, device=dev, generator=g) * 0.02).bfloat16()
        dn = (torch.randn(el * H, F, device=dev, generator=g) * 0.02).bfloat16()
        opt = dict(scoring="sigmoid", bias=bias, n_group=8, topk_group=4, scale=2.5)
        rt = {}
        ops.fused_moe(x, router, gu, dn, k, e0=0, e_loc=el, routing=rt, **opt)
        rows = int(((rt["ids"] >= 0) & (rt["ids"] < el)).sum())
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(a.reps):
            ops.fused_moe(x, router, gu, dn, k, e0=0, e_loc=el, **opt)
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / a.reps
        wbytes = (gu.numel() + dn.numel()) * 2
        print(json.dumps({"kind": "moe_ds", "T": a.T, "e_loc": el, "local_rows": rows, "ms": round(ms, 4),
                          "weight_GBps": round(wbytes / ms / 1e6, 1),
                          "expert_TFLOPs": round(6 * rows * H * F / ms / 1e9, 1)}))
    elif a.kind == "gdn":
        Hg, D = 32, 128
        T = a.nseq * a.L
        proj = torch.randn(T, 4 * Hg * D + 2 * Hg, device=dev).bfloat16()
        state = torch.zeros(a.nseq, Hg, D, D, device=dev)
        slots = torch.arange(a.nseq, dtype=torch.int32, device=dev)
        reset = torch.zeros(a.nseq, dtype=torch.int32, device=dev)
        qs = torch.arange(0, T + 1, a.L, dtype=torch.int32, device=dev)
        for _ in range(a.reps):
            ops.gdn_scan(proj, state, slots, reset, qs, torch.zeros(Hg, device=dev), torch.zeros(Hg, device=dev), Hg)
    elif a.kind in ("decode_fp8", "decode_bf16", "q6k", "q4k", "int4", "fp8gemm", "gemm_bf16", "qkv_rope", "norm"):
        # measured copy bandwidth, sustained and burst bf16 GEMM peaks
        HBM_GBS, BF16_TFLOPS, BF16_BURST = 6534.5, 1400.9, 1672.7
        if a.kind == "qkv_rope":
            # Llama-3-8B QKV projection + RoPE + paged KV write for M tokens: fused epilogue
            # (GOLLEK_ROPE_FUSED=1, default) or projection GEMM then rope_kv_write (=0)
            H, Hk, D = 32, 8, 128
            w = (torch.randn((H + 2 * Hk) * D, a.K, device=dev) * 0.02).bfloat16()
            copies = [w.clone() for _ in range(_n_copies(w.numel() * 2))]
            x = torch.randn(a.M, a.K, device=dev).bfloat16()
            pos = torch.randint(0, 2048, (a.M,), device=dev).int()
            inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device=dev).float() / D))
            ang = torch.arange(8192, device=dev).float()[:, None] * inv[None]
            cos_sin = torch.cat([ang.cos(), ang.sin()], 1).contiguous()
            NB = (a.M + 15) // 16 + 8
            cache = torch.zeros(NB, 2, Hk, 16, D, dtype=torch.bfloat16, device=dev)
            slots = torch.randperm(NB * 16, device=dev)[:a.M].int()
            turn = [0]

            def fn():
                wi = copies[turn[0] % len(copies)]
                turn[0] += 1
                ops.linear_rope_kv(x, wi, pos, cos_sin, cache, slots, H, Hk, D)
            nbytes = w.numel() * 2 + a.M * a.K * 2
            flops = 2.0 * a.M * w.shape[0] * a.K
        elif a.kind == "norm":
            # residual += x; out = RMSNorm(residual) * w for M rows of width K (--residual: fused add)
            n = _n_copies(a.M * a.K * 2 * (2 if a.residual else 1))
            xs = [torch.randn(a.M, a.K, device=dev).bfloat16() for _ in range(n)]
            rs = [torch.randn(a.M, a.K, device=dev).bfloat16() for _ in range(n)] if a.residual else None
            wn = torch.rand(a.K, device=dev).bfloat16()
            outs = [torch.empty(a.M, a.K, device=dev, dtype=torch.bfloat16) for _ in range(n)]
            turn = [0]

            def fn():
                i = turn[0] % n
                turn[0] += 1
                if a.residual:
                    ops.fused_add_rms_norm(xs[i], rs[i], wn, 1e-5, out=outs[i])
                else:
                    ops.rms_norm(xs[i], wn, 1e-5, out=outs[i])
            nbytes = a.M * a.K * 2 * (4 if a.residual else 2)
            flops = None
        elif a.kind == "gemm_bf16":
            # --swiglu: gate/up with the fused SwiGLU epilogue (N = 2 x FFN); --residual: + residual
            w = (torch.randn(a.N, a.K, device=dev) * 0.02).bfloat16()
            copies = [w.clone() for _ in range(_n_copies(a.N * a.K * 2))]
            x = torch.randn(a.M, a.K, device=dev).bfloat16()
            res = torch.randn(a.M, a.N, device=dev).bfloat16() if a.residual else None
            turn = [0]

            if a.splits > 1 or a.bn:  # an explicit tile width / split-K factor (fp32 partials + reduce)
                from gollek_b200.native import cuda_ext
                epi = ops.EPI_SWIGLU if a.swiglu else (ops.EPI_RESIDUAL if a.residual else ops.EPI_NONE)
                yo = torch.empty(a.M, a.N // 2 if a.swiglu else a.N, device=dev, dtype=torch.bfloat16)
                ws = torch.empty(max(1, a.splits) * a.M * a.N, device=dev) if a.splits > 1 else None
                bn = a.bn or ops.gemm_plan(a.M, a.N, a.K, epi)[0]

                def fn():
                    wi = copies[turn[0] % len(copies)]
                    turn[0] += 1
                    cuda_ext().gemm_bf16(yo, x, wi, res, epi, bn, None, 0, max(1, a.splits), ws)
            else:
                def fn():
                    wi = copies[turn[0] % len(copies)]
                    turn[0] += 1
                    ops.linear_swiglu(x, wi) if a.swiglu else ops.linear(x, wi, residual=res)
            nbytes = a.N * a.K * 2 + a.M * a.K * 2
            flops = 2.0 * a.M * a.N * a.K
        elif a.kind == "decode_bf16":
            Hq, Hk, D, bs = 32, 8, 128, 16
            nblk = (a.ctx + bs - 1) // bs
            NB = a.B * nblk
            cache = torch.randn(NB, 2, Hk, bs, D, device=dev).bfloat16()
            bt = torch.randperm(NB, device=dev).int().view(a.B, nblk)
            sl = torch.full((a.B,), a.ctx, dtype=torch.int32, device=dev)
            q = torch.randn(a.B, Hq, D, device=dev).bfloat16()
            sp = ops.decode_splits(a.B, Hk, a.ctx)

            def fn():
                ops.paged_decode_attention(q, cache, bt, sl, 1 / math.sqrt(D), sp)
            nbytes = cache.numel() * 2
            flops = None
        elif a.kind == "decode_fp8":
            Hq, Hk, D, bs = 32, 8, 128, 16
            nblk = (a.ctx + bs - 1) // bs
            NB = a.B * nblk
            cache = torch.randint(0, 120, (NB, 2, Hk, bs, D), dtype=torch.uint8, device=dev)  # finite e4m3
            scl = torch.rand(NB, 2, Hk, bs, device=dev) * 0.01
            bt = torch.randperm(NB, device=dev).int().view(a.B, nblk)
            sl = torch.full((a.B,), a.ctx, dtype=torch.int32, device=dev)
            q = torch.randn(a.B, Hq, D, device=dev).bfloat16()
            sp = ops.decode_splits(a.B, Hk, a.ctx)

            def fn():
                ops.paged_decode_attention(q, cache, bt, sl, 1 / math.sqrt(D), sp, kv_scales=scl)
            nbytes = cache.numel() + scl.numel() * 4
            flops = None
        elif a.kind in ("q4k", "int4"):
            # Q4_K super-blocks (144 B / 256 weights, random nibbles and 6-bit scales, fp16 d = dmin =
            # 2^-10) or GPTQ-style int4 (g128 scales); M tokens: GEMV for M <= 4, else the chunked
            # dequant + tcgen05 GEMM
            if a.kind == "q4k":
                from gollek_b200.loaders import gguf as G
                from gollek_b200.quant.gguf_weights import QWeight
                raw = torch.randint(0, 255, (a.N * a.K // 256 * 144,), dtype=torch.uint8)
                raw.view(-1, 144)[:, 0:4] = torch.tensor([0x00, 0x14, 0x00, 0x14], dtype=torch.uint8)
                copies = [QWeight(raw.to(dev), a.N, a.K, G.GGML_Q4_K) for _ in range(_n_copies(raw.numel()))]
                nbytes = raw.numel()
            else:
                from gollek_b200.quant.int4 import quantize_rtn
                w4 = quantize_rtn((torch.randn(a.N, a.K, device=dev) * 0.02).bfloat16())
                wb = a.N * a.K // 2 + a.N * (a.K // 128) * 4
                copies = [w4] + [quantize_rtn((torch.randn(a.N, a.K, device=dev) * 0.02).bfloat16())
                                 for _ in range(_n_copies(wb) - 1)]
                nbytes = wb
            x = torch.randn(a.M, a.K, device=dev).bfloat16()
            turn = [0]

            def fn():
                ops.linear(x, copies[turn[0] % len(copies)])
                turn[0] += 1
            flops = 2.0 * a.M * a.N * a.K
        elif a.kind == "q6k":
            from gollek_b200.loaders import gguf as G
            from gollek_b200.quant.gguf_weights import QWeight
            raw = torch.randint(0, 255, (a.N * a.K // 256 * 210,), dtype=torch.uint8)
            raw.view(-1, 210)[:, 208:210] = torch.tensor([0x00, 0x20], dtype=torch.uint8)  # d = 2^-7 (fp16)
            copies = [QWeight(raw.to(dev), a.N, a.K, G.GGML_Q6_K) for _ in range(_n_copies(raw.numel()))]
            x = torch.randn(a.M, a.K, device=dev).bfloat16()
            turn = [0]

            def fn():
                ops.linear(x, copies[turn[0] % len(copies)])
                turn[0] += 1
            nbytes = raw.numel()
            flops = None
        else:
            from gollek_b200.quant.fp8 import quantize_weight
            w = (torch.randn(a.N, a.K, device=dev) * 0.02).bfloat16()
            copies = [quantize_weight(w) for _ in range(_n_copies(a.N * a.K))]
            x = torch.randn(a.M, a.K, device=dev).bfloat16()
            turn = [0]

            def fn():
                ops.linear(x, copies[turn[0] % len(copies)])
                turn[0] += 1
            nbytes = a.N * a.K + a.M * a.K * 2
            flops = 2.0 * a.M * a.N * a.K
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        # the repetitions replay as one CUDA graph (serving runs decode steps as graphs): the time is
        # the kernels', not the host's launch rate
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(a.reps):
                fn()
        g.replay()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        g.replay()
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / a.reps
        res = {"kind": a.kind, "ms": round(ms, 4), "GBps": round(nbytes / ms / 1e6, 1),
               "hbm_frac_of_measured": round(nbytes / ms / 1e6 / HBM_GBS, 3)}
        if flops:
            res["TFLOPs"] = round(flops / ms / 1e9, 1)
            if a.kind == "fp8gemm":
                res["frac_of_2x_measured_bf16"] = round(flops / ms / 1e9 / (2 * BF16_TFLOPS), 3)
            elif a.kind in ("q4k", "int4"):
                pass
            else:
                res["frac_of_measured_bf16_sustained"] = round(flops / ms / 1e9 / BF16_TFLOPS, 3)
                res["frac_of_measured_bf16_burst"] = round(flops / ms / 1e9 / BF16_BURST, 3)
        print(json.dumps(res))
    elif a.kind == "decode":
        Hq, Hk, D, bs = 32, 8, 128, 16
        nblk = (a.ctx + bs - 1) // bs
        cache = torch.randn(a.B * nblk, 2, Hk, bs, D, device=dev).bfloat16()
        bt = torch.randperm(a.B * nblk, device=dev).int().view(a.B, nblk)
        sl = torch.full((a.B,), a.ctx, dtype=torch.int32, device=dev)
        q = torch.randn(a.B, Hq, D, device=dev).bfloat16()
        for _ in range(a.reps):
            ops.paged_decode_attention(q, cache, bt, sl, 1 / math.sqrt(D), ops.decode_splits(a.B, Hk, a.ctx))
    else:
        Hq, Hk, D, bs = 32, 8, 128, 16
        T = a.nseq * a.L
        nblk = a.L // bs
        cache = torch.randn(a.nseq * nblk, 2, Hk, bs, D, device=dev).bfloat16()
        bt = torch.arange(a.nseq * nblk, device=dev).int().view(a.nseq, nblk)
        sl = torch.full((a.nseq,), a.L, dtype=torch.int32, device=dev)
        qs = torch.arange(0, T + 1, a.L, dtype=torch.int32, device=dev)
        q = torch.randn(T, Hq, D, device=dev).bfloat16()
        for _ in range(a.reps):
            ops.paged_prefill_attention(q, cache, bt, sl, qs, 1 / math.sqrt(D), emu=a.emu)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
