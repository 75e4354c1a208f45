"""One Mixtral-8x7B MoE layer under expert parallelism (EP = number of GPUs), one process per GPU.

    torchrun --nproc-per-node N benchmarks/ep_a2a_bench.py [--T 128 2048 8192] [--iters 20]

Variants, all producing the next layer's normalised input rows on every rank from the MoE input:
  a2a         token-sharded: route the owned rows, NVLink dispatch (P2P stores), grouped tcgen05
              expert GEMMs, scatter-epilogue combine, weighted sum + residual + RMSNorm gathered with
              multimem.st (parallel/ep_a2a.py, csrc/comm/ep_a2a.cu)
  replicated  every rank holds every row: the local experts' grouped GEMMs over all T rows, then
              the NVLS all-reduce + residual + RMSNorm
  nccl_a2a    the token-sharded protocol with NCCL all_to_all as the transport and the same expert
              kernels per local expert (the NCCL baseline)
Times are CUDA-event medians, max over ranks. Roofline of a2a: the slower of the expert FLOPs of
one rank at the measured sustained bf16 rate and the rows that must cross NVLink (each owned
row's k copies out and back, minus the share that stays local) at 770 GB/s per direction.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

LINK_GBS = 770.0
BF16_TFLOPS = 1400.9  # sustained, measured on this system


def _time(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts.sort()
    t = torch.tensor([ts[len(ts) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t) * 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, nargs="+", default=[128, 2048, 8192])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    ap.add_argument("--experts", type=int, default=8)
    ap.add_argument("--topk", type=int, default=2)
    a = ap.parse_args()
    from gollek_b200 import ops
    from gollek_b200.parallel.dist import cpu_group, init_distributed
    from gollek_b200.parallel.ep_a2a import EPAllToAll, moe_all_to_all_reference, owned_rows
    from gollek_b200.parallel.symm import FusedTPComm
    di = init_distributed(timeout_s=120)
    W, r = di.world_size, di.rank
    H, F, E, k = a.hidden, a.ffn, a.experts, a.topk
    e_loc = E // W
    dev = torch.device("cuda", di.local_rank)
    g = torch.Generator(device=dev).manual_seed(0)
    router = (torch.randn(E, H, device=dev, generator=g) * 0.02).bfloat16()
    gu_all = [(torch.randn(2 * F, H, device=dev, generator=g) * 0.02).bfloat16() for _ in range(E)]
    dn_all = [(torch.randn(H, F, device=dev, generator=g) * 0.02).bfloat16() for _ in range(E)]
    gu = torch.cat(gu_all[r * e_loc:(r + 1) * e_loc]).contiguous()
    dn = torch.cat(dn_all[r * e_loc:(r + 1) * e_loc]).contiguous()
    del gu_all, dn_all
    wn = torch.ones(H, device=dev).bfloat16()
    Tmax = max(a.T)
    ep = EPAllToAll(r, W, max_tokens=Tmax, hidden=H, ffn=F, num_experts=E, top_k=k, cpu_group=cpu_group())
    comm = FusedTPComm(r, W, max_tokens=Tmax, hidden=H, cpu_group=cpu_group(), nvls=True)
    comm.nvls_one_shot_max = 0
    rows = []
    for T in a.T:
        g2 = torch.Generator(device=dev).manual_seed(10 + T)  # same rows on every rank
        x = torch.randn(T, H, device=dev, generator=g2).bfloat16()
        res = torch.randn(T, H, device=dev, generator=g2).bfloat16()
        r0, Tn = owned_rows(T, r, W)
        xo = x[r0:r0 + Tn].contiguous()

        def v_a2a():
            ep.moe(xo, res, router, gu, dn, wn, 1e-5, T)

        def v_replicated():
            part = comm.partial_buffer(T)
            ops.fused_moe(x, router, gu, dn, k, r * e_loc, e_loc, out=part)
            comm.allreduce_add_rmsnorm(part, res, wn, 1e-5)

        def v_nccl():
            ids, wts = ops.moe_route_ref(xo, router, k)
            ids, wts = ids.to(dev), wts.to(dev)

            def expert(xe, e):
                return ops.linear(ops.linear_swiglu(xe, gu[e * 2 * F:(e + 1) * 2 * F]), dn[e * H:(e + 1) * H])

            y = moe_all_to_all_reference(xo, ids, wts, gu, dn, e_loc, expert_fn=expert)
            ops.fused_add_rms_norm(y.bfloat16(), res[r0:r0 + Tn], wn, 1e-5)

        t_a2a = _time(v_a2a, a.iters)
        ep.check()
        t_rep = _time(v_replicated, a.iters)
        t_nccl = _time(v_nccl, a.iters)
        flops = 2.0 * T * k * 3 * H * F / W
        link_bytes = 2.0 * (T / W) * k * H * 2 * (W - 1) / W
        roof = max(flops / (BF16_TFLOPS * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e6
        rows.append({"T": T, "world": W, "a2a_us": round(t_a2a, 1), "replicated_us": round(t_rep, 1),
                     "nccl_a2a_us": round(t_nccl, 1), "a2a_roofline_us": round(roof, 1),
                     "a2a_frac": round(roof / t_a2a, 3)})
    if r == 0:
        for row in rows:
            print(json.dumps(row))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
