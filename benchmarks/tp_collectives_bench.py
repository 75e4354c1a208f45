"""Row-parallel GEMM + all-reduce/residual/RMSNorm variants at Llama-3-8B shapes, one process per GPU.

    torchrun --nproc-per-node N benchmarks/tp_collectives_bench.py [--T 256 1344 8192] [--iters 50]

Every variant is first checked against an fp32 oracle: the partials of all ranks are gathered
(NCCL, fp32) and summed in rank order, the residual added and the RMSNorm applied in fp32; the
variant's normalised rows and updated residual rows must match within bf16 rounding.

Times (CUDA events around CUDA-graph replays of 8 calls, per call, median of iterations, max over
ranks):
  gemm        the row-parallel GEMM alone (o_proj / down_proj shard)
  nvls        GEMM into the symmetric partial buffer + the NVLS multimem all-reduce/residual/RMSNorm
  pull        GEMM into the symmetric partial buffer + the P2P pull all-reduce/residual/RMSNorm
  nccl        GEMM + NCCL all-reduce + fused residual/RMSNorm kernel
and the collective alone (`*_ar`: partial already written). The NVLink roofline of the collective
is the bytes one rank must receive at least, T·d·2 (the reduced rows), over the measured peer
bandwidth (770 GB/s per direction); `frac` = roofline time / measured time.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

LINK_GBS = 770.0  # measured peer copy bandwidth per direction on this B200 system


def _time(fn, iters: int, reps: int = 8) -> float:
    """Median over ``iters`` replays of a CUDA graph holding ``reps`` calls of ``fn`` (so host
    launch overhead is not measured), per call, max over ranks, in us."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) / reps)
    ts.sort()
    t = torch.tensor([ts[len(ts) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return float(t) * 1e3  # us


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, nargs="+", default=[64, 256, 1344, 8192])
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    a = ap.parse_args()
    from gollek_b200 import ops
    from gollek_b200.parallel.dist import cpu_group, init_distributed
    from gollek_b200.parallel.symm import FusedTPComm
    di = init_distributed(timeout_s=60)
    W, r = di.world_size, di.rank
    d = a.hidden
    comms = {"nvls": FusedTPComm(r, W, max_tokens=max(a.T), hidden=d, cpu_group=cpu_group(), nvls=True),
             "pull": FusedTPComm(r, W, max_tokens=max(a.T), hidden=d, cpu_group=cpu_group(), nvls=False)}
    if not comms["nvls"].nvls:
        if r == 0:
            print(json.dumps({"nvls": "unavailable", "why": comms["nvls"].heap.multicast_error}))
        comms.pop("nvls")
    rows, checks = [], []
    for T in a.T:
        for name, K in (("o_proj", d // W), ("down", a.ffn // W)):
            g = torch.Generator(device="cuda").manual_seed(1000 * r + T)
            x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
            w = (torch.randn(d, K, device="cuda", generator=g) * 0.02).bfloat16()
            g0 = torch.Generator(device="cuda").manual_seed(7 + T)  # identical on every rank
            res0 = torch.randn(T, d, device="cuda", generator=g0).bfloat16()
            nw = (1.0 + 0.1 * torch.randn(d, device="cuda", generator=g0)).bfloat16()
            # fp32 oracle
            part = (x.float() @ w.float().t())
            parts = [torch.empty_like(part) for _ in range(W)]
            dist.all_gather(parts, part)
            tot = torch.zeros_like(part)
            for p in parts:
                tot += p
            ref_res = res0.float() + tot
            ref_x = ref_res * torch.rsqrt(ref_res.pow(2).mean(-1, keepdim=True) + 1e-5) * nw.float()
            chunk = (T + W - 1) // W
            for vname, comm in comms.items():
                res = res0.clone()
                h = ops.linear(x, w, out=comm.partial_buffer(T))
                xo = comm.allreduce_add_rmsnorm(h, res, nw, 1e-5).float()
                comm.check()
                two_shot = comm.nvls and T > comm.nvls_one_shot_max
                own = slice(r * chunk, min(T, (r + 1) * chunk)) if two_shot else slice(0, T)
                ex = (xo - ref_x).abs().max().item()
                er = (res[own].float() - ref_res[own]).abs().max().item()
                # bf16 partials (one rounding each) + bf16 residual: a few ulps of the row scale
                ok = ex < 0.06 and er < 0.06 * max(1.0, ref_res.abs().max().item() / 8)
                checks.append({"T": T, "gemm": name, "variant": vname, "max_abs_err_x": round(ex, 5),
                               "max_abs_err_residual": round(er, 5), "ok": bool(ok)})
            res = res0.clone()
            for vname, comm in comms.items():
                def v_full(comm=comm):
                    h = ops.linear(x, w, out=comm.partial_buffer(T))
                    comm.allreduce_add_rmsnorm(h, res, nw, 1e-5)

                def v_ar(comm=comm):
                    comm.allreduce_add_rmsnorm(comm.partial_buffer(T), res, nw, 1e-5)

                rows.append({"T": T, "gemm": name, "variant": vname, "us": round(_time(v_full, a.iters), 1),
                             "world": W})
                t_ar = _time(v_ar, a.iters)
                roof_us = T * d * 2 / (LINK_GBS * 1e9) * 1e6
                rows.append({"T": T, "gemm": name, "variant": vname + "_ar", "us": round(t_ar, 1), "world": W,
                             "roofline_us": round(roof_us, 1), "frac": round(roof_us / t_ar, 3)})
                comm.check()
            pc = comms.get("pull")

            def v_gemm():
                ops.linear(x, w, out=pc.partial_buffer(T))

            def v_nccl():
                h = ops.linear(x, w)
                dist.all_reduce(h)
                ops.fused_add_rms_norm(h, res, nw, 1e-5)

            hbuf = torch.randn(T, d, device="cuda").bfloat16()

            def v_nccl_ar():
                dist.all_reduce(hbuf)
                ops.fused_add_rms_norm(hbuf, res, nw, 1e-5)

            rows.append({"T": T, "gemm": name, "variant": "gemm", "us": round(_time(v_gemm, a.iters), 1), "world": W})
            rows.append({"T": T, "gemm": name, "variant": "nccl", "us": round(_time(v_nccl, a.iters), 1), "world": W})
            t_ar = _time(v_nccl_ar, a.iters)
            roof_us = T * d * 2 / (LINK_GBS * 1e9) * 1e6
            rows.append({"T": T, "gemm": name, "variant": "nccl_ar", "us": round(t_ar, 1), "world": W,
                         "roofline_us": round(roof_us, 1), "frac": round(roof_us / t_ar, 3)})
    for c in comms.values():
        c.check()
    oks = torch.tensor([all(c["ok"] for c in checks)], dtype=torch.int32, device="cuda")
    dist.all_reduce(oks, op=dist.ReduceOp.MIN)
    if r == 0:
        for c in checks:
            print(json.dumps({"check": c, "world": W}))
        for row in rows:
            print(json.dumps(row))
        print(json.dumps({"all_checks_ok": bool(oks.item()), "world": W,
                          "backend": {k: c.heap.backend for k, c in comms.items()}}))
    dist.barrier()
    dist.destroy_process_group()
    if not oks.item():
        sys.exit(1)


if __name__ == "__main__":
    main()
