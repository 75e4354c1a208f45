"""Per-kernel timing at Llama-3-8B serving shapes against the measured B200 roofline.

Every number: median of CUDA-event timings on the launching stream after warm-up, with a
256 MB buffer written between iterations to flush the 126 MB L2. Fractions are of the measured
peaks in MEASURED_PEAKS.json (HBM copy GB/s, cuBLAS bf16 TFLOP/s burst). cuBLAS (torch.matmul)
timings are printed beside our GEMMs as a reference point only.

    python benchmarks/kernel_bench.py [--only gemm,attn,prefill,norm,gdn] [--json out.jsonl]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

from gollek_b200 import ops  # noqa: E402
from gollek_b200.utils.timing import time_cuda  # noqa: E402


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "of measured"
    return 6650.0, 1590.0, "of fallback"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,attn,norm,sample")
    ap.add_argument("--json", default=None)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    only = set(args.only.split(","))
    hbm, tflops, tag = peaks()
    dev = "cuda"
    torch.manual_seed(0)
    rows = []
    flush = 256 << 20

    def rec(name, ms, flops=0.0, nbytes=0.0, extra=None):
        r = {"kernel": name, "ms": round(ms, 4)}
        if flops:
            r["tflops"] = round(flops / ms / 1e9, 1)
            r["frac_compute"] = round(flops / ms / 1e9 / tflops, 3)
        if nbytes:
            r["gbs"] = round(nbytes / ms / 1e6, 1)
            r["frac_hbm"] = round(nbytes / ms / 1e6 / hbm, 3)
        if flops or nbytes:
            t_roof = max(flops / (tflops * 1e12), nbytes / (hbm * 1e9)) * 1e3
            r["frac_roofline"] = round(t_roof / ms, 3)
        if extra:
            r.update(extra)
        rows.append(r)
        print(json.dumps(r), flush=True)

    if "gemm" in only:
        shapes = [("qkv", 6144, 4096), ("o_proj", 4096, 4096), ("gate_up_swiglu", 28672, 4096),
                  ("down", 4096, 14336), ("lm_head", 128256, 4096)]
        for M in (64, 256, 1024, 8192):
            for name, N, K in shapes:
                if name == "lm_head" and M > 256:
                    continue
                a = torch.randn(M, K, device=dev).bfloat16()
                w = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
                sw = name.endswith("swiglu")
                out = torch.empty(M, N // 2 if sw else N, device=dev, dtype=torch.bfloat16)
                fn = (lambda: ops.linear_swiglu(a, w, out=out)) if sw else (lambda: ops.linear(a, w, out=out))
                ms = time_cuda(fn, iters=args.iters, flush_bytes=flush)
                flops = 2.0 * M * N * K
                nbytes = 2.0 * (M * K + N * K + M * (N // 2 if sw else N))
                cub = time_cuda(lambda: torch.matmul(a, w.t()), iters=args.iters, flush_bytes=flush)
                bn = ops.cuda_ext().gemm_pick_bn(M, N, 2 if sw else 0)
                rec(f"gemm_{name}_M{M}", ms, flops, nbytes, {"shape": [M, N, K], "bn": bn,
                                                              "cublas_ms": round(cub, 4)})
    if "attn" in only or "prefill" in only:
        Hq, Hk, D, bs = 32, 8, 128, 16
        for B, ctx in ((256, 1200), (64, 4096), (8, 2048), (1, 8192)) if "attn" in only else ():
            nblk = (ctx + bs - 1) // bs
            NB = B * nblk
            cache = torch.randn(NB, 2, Hk, bs, D, device=dev).bfloat16()
            bt = torch.randperm(NB, device=dev).int().view(B, nblk)
            sl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
            q = torch.randn(B, Hq, D, device=dev).bfloat16()
            splits = ops.decode_splits(B, Hk, ctx)
            ws = torch.empty(B * Hq * splits * (D + 2), device=dev)
            out = torch.empty_like(q)
            ms = time_cuda(lambda: ops.paged_decode_attention(q, cache, bt, sl, 1 / math.sqrt(D), splits, out=out,
                                                              workspace=ws), iters=args.iters, flush_bytes=flush)
            nbytes = B * ctx * Hk * D * 2 * 2
            flops = 4.0 * B * ctx * Hq * D
            rec(f"attn_decode_B{B}_ctx{ctx}", ms, flops, nbytes, {"splits": splits})
        for nseq, L in ((4, 2048), (8, 1024), (1, 8192), (1, 1088), (2, 1024)):
            T = nseq * L
            nblk = L // bs
            NB = nseq * nblk
            cache = torch.randn(NB, 2, Hk, bs, D, device=dev).bfloat16()
            bt = torch.arange(NB, device=dev).int().view(nseq, nblk)
            sl = torch.full((nseq,), L, dtype=torch.int32, device=dev)
            qs = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
            q = torch.randn(T, Hq, D, device=dev).bfloat16()
            out = torch.empty_like(q)
            flops = 4.0 * nseq * (L * L / 2) * Hq * D
            nbytes = 2.0 * (2 * T * Hq * D + 2 * T * Hk * D)
            work = ops.prefill_schedule(qs.tolist(), sl.tolist(), Hq, Hk, D).to(dev)
            variants = [(f"tcgen05_emu{e}", work, True, e) for e in (0, 1, 2)]
            for form in ("pairs", "rows"):  # both work-item forms, whichever the schedule picked
                wf = ops.prefill_schedule(qs.tolist(), sl.tolist(), Hq, Hk, D, form=form).to(dev)
                variants.append((f"tcgen05_{form}", wf, True, ops.PREFILL_EMU))
            variants += [("tcgen05_1tile", ops.prefill_tiles(qs.tolist(), 128).to(dev), True, 0),
                         ("mmasync", ops.prefill_tiles(qs.tolist(), 64).to(dev), False, 0)]
            for name, tiles, tc, emu in variants:
                ms = time_cuda(lambda: ops.paged_prefill_attention(q, cache, bt, sl, qs, 1 / math.sqrt(D), tiles=tiles,
                                                                   out=out, tensor_cores=tc, emu=emu),
                               iters=args.iters, flush_bytes=flush)
                rec(f"attn_prefill_{name}_{nseq}x{L}", ms, flops, nbytes)
    if "lora" in only:
        # K10 multi-LoRA shrink + expand on fused q/k/v (rank 16 x 3 modules), 64 adapters by Zipf(1.1)
        from gollek_b200.native import cuda_ext
        ext = cuda_ext()
        K, r, S, N1, N2, N = 4096, 16, 64, 4096, 5120, 6144
        A = (torch.randn(S, 3 * r, K, device=dev) * 0.02).bfloat16()
        Bw = (torch.randn(S, N, r, device=dev) * 0.02).bfloat16()
        scales = torch.ones(S, device=dev)
        zipf = torch.tensor([1.0 / (i + 1) ** 1.1 for i in range(S)])
        for T, per_seq in ((256, 1), (8192, 512)):
            n_seq = T // per_seq
            seq_ad = torch.multinomial(zipf, n_seq, replacement=True, generator=torch.Generator().manual_seed(3))
            groups = {}
            for i, a in enumerate(seq_ad.tolist()):
                groups.setdefault(a, []).extend(range(i * per_seq, (i + 1) * per_seq))
            seg_slot = sorted(groups)
            seg_ptr, tok, tiles = [0], [], []
            for i, sl in enumerate(seg_slot):
                tiles += [[i, q] for q in range(len(tok), len(tok) + len(groups[sl]), 64)]
                tok += groups[sl]
                seg_ptr.append(len(tok))
            d = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731
            sp, tk, ss, tl = d(seg_ptr), d(tok), d(seg_slot), d(tiles)
            mx = max(len(v) for v in groups.values())
            x = torch.randn(T, K, device=dev).bfloat16()
            y = torch.randn(T, N, device=dev).bfloat16()
            V = torch.zeros(T, 3 * r, device=dev)

            def run():
                V.zero_()
                ext.lora_shrink(V, x, A, sp, tk, ss, tl, mx)
                ext.lora_expand(y, V, Bw, N1, N2, scales, sp, tk, ss, tl)
            ms = time_cuda(run, iters=args.iters, flush_bytes=flush)
            nbytes = 2.0 * (T * K + len(seg_slot) * 3 * r * K + 2 * T * N + len(seg_slot) * N * r)
            rec(f"lora_qkv_T{T}_segs{len(seg_slot)}", ms, 2.0 * T * 3 * r * (K + N // 3), nbytes)
    if "gdn" in only:
        # K14 gated delta rule: decode (one token per sequence, state-bandwidth bound: the fp32 state of
        # every head is read and written) and one long prefill sequence (CUDA-core FMAs)
        Hg, D = 32, 128
        for nseq, L in ((256, 1), (1, 4096), (8, 1024)):
            T = nseq * L
            proj = torch.randn(T, 4 * Hg * D + 2 * Hg, device=dev).bfloat16()
            state = torch.zeros(nseq, Hg, D, D, device=dev)
            slots = torch.arange(nseq, dtype=torch.int32, device=dev)
            reset = torch.zeros(nseq, dtype=torch.int32, device=dev)
            qs = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
            a_log, dt = torch.zeros(Hg, device=dev), torch.zeros(Hg, device=dev)
            out = torch.empty(T, Hg, D, device=dev).bfloat16()
            ms = time_cuda(lambda: ops.gdn_scan(proj, state, slots, reset, qs, a_log, dt, Hg, out=out),
                           iters=args.iters, flush_bytes=flush)
            rec(f"gdn_scan_{nseq}x{L}", ms, 6.0 * T * Hg * D * D, 2.0 * nseq * Hg * D * D * 4 + proj.numel() * 2)
    if "kvnorm" in only:
        # K15 KV eviction scoring: mean key norm of 512 blocks of a Llama-3-8B cache (every layer)
        cache = torch.randn(32, 4096, 2, 8, 16, 128, device=dev).bfloat16()
        ids = torch.randperm(4096, device=dev)[:512].int()
        ms = time_cuda(lambda: ops.kv_key_norms(cache, ids), iters=args.iters, flush_bytes=flush)
        rec("kv_key_norms_512blocks", ms, 0, 2.0 * 32 * 512 * 8 * 16 * 128)
    if "norm" in only:
        d = 4096
        for T in (256, 8192):
            x = torch.randn(T, d, device=dev).bfloat16()
            r = torch.randn(T, d, device=dev).bfloat16()
            w = torch.ones(d, device=dev).bfloat16()
            out = torch.empty_like(x)
            ms = time_cuda(lambda: ops.fused_add_rms_norm(x, r, w, 1e-5, out=out), iters=args.iters, flush_bytes=flush)
            rec(f"fused_add_rms_norm_T{T}", ms, 0, 2.0 * 4 * T * d)
            from gollek_b200.config import preset
            from gollek_b200.models.reference import rope_cos_sin
            cs = rope_cos_sin(preset("llama-3-8b"), 8192, device=dev)
            qkv = torch.randn(T, 6144, device=dev).bfloat16()
            pos = torch.arange(T, device=dev).int() % 8000
            cache = torch.zeros(T // 16 + 1, 2, 8, 16, 128, device=dev).bfloat16()
            slots = torch.arange(T, device=dev).int()
            qo = torch.empty(T, 32, 128, device=dev).bfloat16()
            ms = time_cuda(lambda: ops.rope_kv_write(qkv, pos, cs, cache, slots, 32, 8, 128, q_out=qo),
                           iters=args.iters, flush_bytes=flush)
            rec(f"rope_kv_write_T{T}", ms, 0, 2.0 * (T * 6144 + T * 4096 + T * 2048))
    if "sample" in only:
        for B in (256,):
            V = 128256
            logits = torch.randn(B, V, device=dev).bfloat16()
            out = torch.empty(B, dtype=torch.int64, device=dev)
            ms = time_cuda(lambda: ops.argmax(logits, out=out), iters=args.iters, flush_bytes=flush)
            rec(f"argmax_B{B}_V{V}", ms, 0, 2.0 * B * V)
            lf = logits.float()
            t = torch.full((B,), 0.8, device=dev)
            k = torch.full((B,), 50, dtype=torch.int32, device=dev)
            p = torch.full((B,), 0.9, device=dev)
            mp = torch.zeros(B, device=dev)
            sd = torch.arange(B, device=dev)
            off = torch.zeros(B, dtype=torch.int64, device=dev)
            ms = time_cuda(lambda: ops.sample(lf, t, k, p, mp, sd, off, out=out), iters=args.iters, flush_bytes=flush)
            rec(f"sample_topk_topp_B{B}_V{V}", ms, 0, 4.0 * B * V)
    if "gguf" in only:
        from gollek_b200.native import host_ext
        from gollek_b200.quant.gguf_weights import QWeight
        h = host_ext()
        for name, N, K in (("qkv", 6144, 4096), ("gate_up", 28672, 4096), ("down", 4096, 14336)):
            w = torch.randn(N * K) * 0.02
            for qtype, q in ((12, h.quantize_q4_k), (8, h.quantize_q8_0)):
                qw = QWeight(q(w).to(dev), N, K, qtype)
                for M in (1, 4, 16, 64, 256):
                    x = torch.randn(M, K, device=dev).bfloat16()
                    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                    ms = time_cuda(lambda: ops.linear(x, qw, out=out), iters=args.iters, flush_bytes=flush)
                    rec(f"gguf_{'q4k' if qtype == 12 else 'q8_0'}_{name}_M{M}", ms, 2.0 * M * N * K,
                        qw.nbytes() + 2.0 * M * (K + N))
    if "int4" in only:
        from gollek_b200.quant import int4 as I4
        for name, N, K in (("qkv", 6144, 4096), ("gate_up", 28672, 4096), ("down", 4096, 14336)):
            w = (torch.randn(N, K, device=dev) * 0.02)
            for fmt, qw in (("int4g128", I4.quantize_rtn(w, 128)), ("nf4", I4.quantize_nf4(w, 64))):
                qw = qw.to(dev)
                for M in (1, 8, 256):
                    x = torch.randn(M, K, device=dev).bfloat16()
                    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                    ms = time_cuda(lambda: ops.linear(x, qw, out=out), iters=args.iters, flush_bytes=flush)
                    rec(f"{fmt}_{name}_M{M}", ms, 2.0 * M * N * K, qw.nbytes() + 2.0 * M * (K + N))
    if "fp8" in only:
        from gollek_b200.quant import fp8 as F8
        # Llama-3-70B per-rank shapes at TP=8 (hidden 8192, 64/8 heads, ffn 28672)
        for name, N, K in (("qkv", 1280, 8192), ("o_proj", 8192, 1024), ("gate_up", 7168, 8192), ("down", 8192, 3584)):
            w = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
            fw = F8.quantize_weight(w)
            for M in (64, 1024, 8192):
                x = torch.randn(M, K, device=dev).bfloat16()
                out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                ms = time_cuda(lambda: ops.linear(x, fw, out=out), iters=args.iters, flush_bytes=flush)
                rec(f"fp8_{name}_tp8_M{M}", ms, 2.0 * M * N * K, N * K + 2.0 * M * (K + N),
                    {"splits": ops.cuda_ext().gemm_fp8_splits(M, N, K, 0)})
    if "gemm_sweep" in only:
        # tile width x split-K at the token counts of a saturated serving step (~255 decodes + one prompt)
        shapes = [("qkv", 6144, 4096, 0), ("o_proj", 4096, 4096, 1), ("gate_up_swiglu", 28672, 4096, 2),
                  ("down", 4096, 14336, 1)]
        for M in (1344, 2048, 4352):
            for name, N, K, epi in shapes:
                a = torch.randn(M, K, device=dev).bfloat16()
                w = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
                res = torch.randn(M, N, device=dev).bfloat16() if epi == 1 else None
                out = torch.empty(M, N // 2 if epi == 2 else N, device=dev, dtype=torch.bfloat16)
                ws = torch.empty(4 * M * N, device=dev)
                auto = ops.cuda_ext().gemm_plan(M, N, K, epi)
                for bn in ((128, 256) if epi == 2 else (128, 256)):
                    for sp in (1, 2, 3):
                        fn = lambda: ops.cuda_ext().gemm_bf16(out, a, w, res, epi, bn, None, 0, sp, ws)
                        ms = time_cuda(fn, iters=args.iters, flush_bytes=flush)
                        rec(f"gemm_{name}_M{M}_bn{bn}_s{sp}", ms, 2.0 * M * N * K,
                            2.0 * (M * K + N * K + M * N), {"auto": auto})
    if "moe" in only:
        # Mixtral-8x7B MoE layer (H 4096, F 14336, 8 experts, top-2): all experts on one GPU, and the
        # one-expert shard a rank holds under EP=8 (its partial sum; the all-reduce is not included)
        H, F, E, k = 4096, 14336, 8, 2
        router = (torch.randn(E, H, device=dev) * 0.02).bfloat16()
        for e_loc in (8, 1):
            gu = (torch.randn(e_loc * 2 * F, H, device=dev) * 0.02).bfloat16()
            dn = (torch.randn(e_loc * H, F, device=dev) * 0.02).bfloat16()
            for T in (64, 256, 2048, 8192):
                x = torch.randn(T, H, device=dev).bfloat16()
                out = torch.empty_like(x)
                ms = time_cuda(lambda: ops.fused_moe(x, router, gu, dn, k, e0=0, e_loc=e_loc, out=out),
                               iters=args.iters, flush_bytes=flush)
                with torch.no_grad():
                    ids, _ = ops.moe_route_ref(x[:min(T, 4096)].float(), router.float(), k)
                nrows = T * k * e_loc / E  # expected routed rows on these experts (uniform router)
                active = min(e_loc, len(set(ids.flatten().tolist()) & set(range(e_loc))) or e_loc)
                flops = 2.0 * nrows * 3 * H * F
                nbytes = active * 3.0 * H * F * 2 + 2.0 * 2 * T * H + 2.0 * nrows * (2 * H + F)
                rec(f"moe_mixtral_{'all8' if e_loc == 8 else 'ep8_shard'}_T{T}", ms, flops, nbytes)
    if args.json:
        with open(args.json, "w") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")
    print(f"# peaks: HBM {hbm} GB/s, bf16 {tflops} TFLOP/s ({tag})")


if __name__ == "__main__":
    main()
