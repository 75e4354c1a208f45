"""Row-parallel GEMM + all-reduce variants at Llama-3-8B shapes, one process per GPU.

    torchrun --nproc-per-node 2 benchmarks/tp_collectives_bench.py [--T 256] [--iters 50]

Times (CUDA events on the launching stream, max over ranks, median of iterations):
  gemm        the row-parallel GEMM alone (o_proj / down_proj shard)
  pull        GEMM into the symmetric partial buffer + the fused all-reduce/residual/RMSNorm kernel
  push        GEMM with the push epilogue + the local-reduce/residual/RMSNorm consumer
  nccl        GEMM + NCCL all-reduce + fused residual/RMSNorm kernel
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, nargs="+", default=[64, 256, 1344])
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args()
    from gollek_b200 import ops
    from gollek_b200.parallel.dist import cpu_group, init_distributed
    from gollek_b200.parallel.symm import FusedTPComm
    di = init_distributed(timeout_s=60)
    W, r = di.world_size, di.rank
    d = 4096
    comm = FusedTPComm(r, W, max_tokens=max(a.T), hidden=d, cpu_group=cpu_group(), push_max_tokens=max(a.T))
    rows = []
    for T in a.T:
        for name, K in (("o_proj", 4096 // W), ("down", 14336 // W)):
            g = torch.Generator(device="cuda").manual_seed(r)
            x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
            w = (torch.randn(d, K, device="cuda", generator=g) * 0.02).bfloat16()
            res = torch.randn(T, d, device="cuda").bfloat16()
            nw = torch.ones(d, device="cuda").bfloat16()

            def v_gemm():
                ops.linear(x, w, out=comm.partial_buffer(T))

            def v_pull():
                h = ops.linear(x, w, out=comm.partial_buffer(T))
                comm.allreduce_add_rmsnorm(h, res, nw, 1e-5)

            def v_push():
                h = comm.push_linear(x, w)
                comm.allreduce_add_rmsnorm(h, res, nw, 1e-5)

            def v_nccl():
                h = ops.linear(x, w)
                dist.all_reduce(h)
                ops.fused_add_rms_norm(h, res, nw, 1e-5)

            for vname, fn in (("gemm", v_gemm), ("pull", v_pull), ("push", v_push), ("nccl", v_nccl)):
                for _ in range(5):
                    fn()
                torch.cuda.synchronize()
                dist.barrier()
                ts = []
                for _ in range(a.iters):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    fn()
                    e1.record()
                    e1.synchronize()
                    ts.append(e0.elapsed_time(e1))
                ts.sort()
                t = torch.tensor([ts[len(ts) // 2]], device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                rows.append({"T": T, "gemm": name, "variant": vname, "us": round(float(t) * 1e3, 1), "world": W})
    comm.check()
    if r == 0:
        for row in rows:
            print(json.dumps(row))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
