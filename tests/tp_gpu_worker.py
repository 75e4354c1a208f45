"""Per-rank body of the 2-GPU collective tests (spawned processes, NCCL + symmetric heap)."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run_collectives(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from gollek_b200 import ops
        from gollek_b200.parallel.dist import cpu_group, init_distributed
        from gollek_b200.parallel.symm import FusedTPComm
        init_distributed(backend="nccl", timeout_s=60)
        d = 4096
        # the P2P pull / push kernels (full residual rows on every rank); NVLS is covered by run_selfcheck
        comm = FusedTPComm(rank, world, max_tokens=1024, hidden=d, cpu_group=cpu_group(), one_shot_max_tokens=16,
                           push_max_tokens=256, nvls=False)
        errs = []
        for T in (1, 7, 16, 300, 1024):
            for rep in range(3):  # consecutive calls exercise the buffer parity and epochs
                g = torch.Generator(device="cuda").manual_seed(1000 * T + 10 * rep + rank)
                h = (torch.randn(T, d, device="cuda", generator=g) * 0.5).bfloat16()
                gs = torch.Generator(device="cuda").manual_seed(7 * T + rep)
                res = torch.randn(T, d, device="cuda", generator=gs).bfloat16()
                w = (torch.rand(d, device="cuda", generator=gs) + 0.5).bfloat16()
                # NCCL oracle
                h_ref = h.clone()
                dist.all_reduce(h_ref)
                res_ref = res.clone()
                x_ref = ops.fused_add_rms_norm(h_ref, res_ref, w, 1e-5)
                x = comm.allreduce_add_rmsnorm(h, res, w, 1e-5)
                torch.cuda.synchronize()
                # relative to magnitude: the fused kernel rounds the fp32 sum once, NCCL + norm twice
                errs.append((T, rep, float(((x.float() - x_ref.float()).abs() / (1 + x_ref.float().abs())).max()),
                             float(((res.float() - res_ref.float()).abs() / (1 + res_ref.float().abs())).max())))
            # plain all-reduce
            t = (torch.randn(T, d, device="cuda", generator=g)).bfloat16()
            t_ref = t.clone()
            dist.all_reduce(t_ref)
            comm.all_reduce(t)
            torch.cuda.synchronize()
            errs.append((T, "ar", float(((t.float() - t_ref.float()).abs() / (1 + t_ref.float().abs())).max()), 0.0))
        # GEMM -> all-reduce push path against (a) the pull kernels on the same GEMM output (bitwise)
        # and (b) NCCL; push and pull calls interleave to exercise buffer parity and epochs
        K = 1024
        for T in (1, 7, 64, 200, 256):
            for rep in range(2):
                g = torch.Generator(device="cuda").manual_seed(5000 * T + rep * 10 + rank)
                a = torch.randn(T, K, device="cuda", generator=g).bfloat16()
                wt = (torch.randn(d, K, device="cuda", generator=g) * 0.03).bfloat16()
                gs = torch.Generator(device="cuda").manual_seed(11 * T + rep)
                res = torch.randn(T, d, device="cuda", generator=gs).bfloat16()
                w = (torch.rand(d, device="cuda", generator=gs) + 0.5).bfloat16()
                res_pull = res.clone()
                h = comm.push_linear(a, wt)
                assert h is not None
                x = comm.allreduce_add_rmsnorm(h, res, w, 1e-5)
                hp = ops.linear(a, wt, out=comm.partial_buffer(T))
                x_pull = comm.allreduce_add_rmsnorm(hp, res_pull, w, 1e-5)
                h_ref = ops.linear(a, wt)
                dist.all_reduce(h_ref)
                res_ref = torch.randn(T, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(
                    11 * T + rep)).bfloat16()
                x_ref = ops.fused_add_rms_norm(h_ref, res_ref, w, 1e-5)
                torch.cuda.synchronize()
                errs.append((T, f"push{rep}", float(((x.float() - x_ref.float()).abs() / (1 + x_ref.float().abs())).max()),
                             float((x.float() - x_pull.float()).abs().max() + (res.float() - res_pull.float()).abs().max())))
        # C5 distributed argmax vs the argmax of the all-gathered logits (incl. a cross-rank tie)
        V = 32000
        for B in (1, 37, 256):
            g = torch.Generator(device="cuda").manual_seed(77 * B + rank)
            shard = torch.randn(B, V // world, device="cuda", generator=g).bfloat16()
            if B > 1:
                shard[1, 5] = 50.0  # same maximum on every rank: the lowest global id must win
            ids = comm.argmax_last(shard, rank * (V // world))
            full = comm.all_gather_last(shard)
            ref = full.float().argmax(-1)
            torch.cuda.synchronize()
            errs.append((B, "argmax", float((ids != ref).sum()), 0.0))
        comm.check()
        result_q.put((rank, errs, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        result_q.put((rank, None, traceback.format_exc()))


def run_selfcheck(rank, world, port, kind, result_q):
    """Collectives and a two-layer TP engine against fp32 oracles (gollek_b200.parallel.selfcheck).
    ``kind``: "nvls" (multimem kernels), "p2p" (pull kernels) or "nccl" (engine with the NCCL
    baseline comm)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from gollek_b200.parallel import selfcheck as sc
        from gollek_b200.parallel.dist import NcclComm, cpu_group, init_distributed
        from gollek_b200.parallel.symm import FusedTPComm
        init_distributed(backend="nccl", timeout_s=120)
        out = {}
        if kind == "nccl":
            out["engine"] = sc.engine_check(lambda mt, hid: NcclComm(rank, world))
        else:
            def make(mt, hid):
                return FusedTPComm(rank, world, max_tokens=mt, hidden=hid, cpu_group=cpu_group(),
                                   nvls=(kind == "nvls"))
            comm = make(8192 + 64, 4096)
            out["nvls_active"] = comm.nvls
            out["collectives"] = sc.collectives_check(comm, sizes=(1, 7, 64, 129, 300, 1344, 8192))
            out["engine"] = sc.engine_check(make)
            # Mixtral-shaped slice with the experts partitioned over the ranks (the NVLink
            # all-to-all under NVLS, replicated activations with the P2P kernels)
            out["moe_engine"] = sc.engine_check(make, model="mixtral-8x7b", expert_parallel=True,
                                                overrides={"intermediate_size": 2048})
        result_q.put((rank, out, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        result_q.put((rank, None, traceback.format_exc()))
