"""Per-rank bodies of the expert-parallel all-to-all tests (spawned processes)."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def moe_case(E=8, H=256, F=128, T=37, seed=0, dtype=torch.float32):
    """Random MoE layer (every rank builds the same one) and T token rows."""
    g = torch.Generator().manual_seed(seed)
    router = torch.randn(E, H, generator=g) * 0.05
    experts = [(torch.randn(F, H, generator=g) * 0.05, torch.randn(F, H, generator=g) * 0.05,
                torch.randn(H, F, generator=g) * 0.05) for _ in range(E)]
    x = torch.randn(T, H, generator=g)
    return router.to(dtype), [tuple(w.to(dtype) for w in e) for e in experts], x.to(dtype)


def fused_local(experts, e0, e_loc):
    """The rank's experts in the fused layouts: gate/up interleaved in groups of 64, down stacked."""
    from gollek_b200.ops import reference as ref
    gu = torch.cat([ref.interleave_gate_up(experts[e][0], experts[e][1]) for e in range(e0, e0 + e_loc)])
    dn = torch.cat([experts[e][2] for e in range(e0, e0 + e_loc)])
    return gu, dn


def run_restatement(rank, world, port, T, k, result_q):
    """gloo ranks: the torch.distributed restatement of the dispatch / combine protocol against the
    dense fp32 MoE on this rank's owned rows."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import torch.distributed as dist
        from gollek_b200.models.reference import moe_ref
        from gollek_b200.ops import reference as ref
        from gollek_b200.parallel.ep_a2a import moe_all_to_all_reference, owned_rows
        dist.init_process_group("gloo", rank=rank, world_size=world)
        E = 8
        router, experts, x = moe_case(E=E, T=T)
        e_loc = E // world
        gu, dn = fused_local(experts, rank * e_loc, e_loc)
        r0, Tn = owned_rows(T, rank, world)
        xo = x[r0:r0 + Tn]
        ids, wts = ref.moe_route(xo.float() @ router.float().t(), k)
        got = moe_all_to_all_reference(xo, ids, wts, gu, dn, e_loc)
        want = moe_ref(xo, router, experts, k).float()
        err = float((got - want).abs().max()) if Tn else 0.0
        result_q.put((rank, err, None))
        dist.destroy_process_group()
    except Exception:
        import traceback
        result_q.put((rank, None, traceback.format_exc()))


def run_ep_gpu(rank, world, port, result_q):
    """NVLink kernels (EPAllToAll) on `world` GPUs: every rank's gathered output rows and its owned
    residual rows against the dense fp32 MoE + residual + RMSNorm, over several token counts
    (consecutive calls advance the epochs; some counts leave ranks without tokens)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from gollek_b200.models.reference import moe_ref
        from gollek_b200.parallel.dist import cpu_group, init_distributed
        from gollek_b200.parallel.ep_a2a import EPAllToAll, owned_rows
        init_distributed(backend="nccl", timeout_s=120)
        E, H, F, k = 8, 1024, 512, 2
        router, experts, _ = moe_case(E=E, H=H, F=F, T=1)
        e_loc = E // world
        gu, dn = fused_local(experts, rank * e_loc, e_loc)
        dev = torch.device("cuda", rank)
        ep = EPAllToAll(rank, world, max_tokens=2048, hidden=H, ffn=F, num_experts=E, top_k=k,
                        cpu_group=cpu_group())
        r_b, gu_b, dn_b = router.bfloat16().to(dev), gu.bfloat16().to(dev), dn.bfloat16().to(dev)
        wn = (1.0 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(9))).bfloat16()
        experts_b = [tuple(w.bfloat16().float() for w in e) for e in experts]  # the weights as served
        worst_x = worst_r = 0.0
        for T in (1, 7, 300, 2048, 64):
            g = torch.Generator().manual_seed(100 + T)
            x = torch.randn(T, H, generator=g).bfloat16()
            res = torch.randn(T, H, generator=g).bfloat16()
            r0, Tn = owned_rows(T, rank, world)
            resd = res.to(dev)
            out = ep.moe(x[r0:r0 + Tn].to(dev), resd, r_b, gu_b, dn_b, wn.to(dev), 1e-5, T).float().cpu()
            torch.cuda.synchronize()
            ep.check()
            y = moe_ref(x.float(), router.bfloat16().float(), experts_b, k).float()
            ref_res = res.float() + y
            ref_x = ref_res * torch.rsqrt(ref_res.pow(2).mean(-1, keepdim=True) + 1e-5) * wn.float()
            worst_x = max(worst_x, float(((out - ref_x).abs() / (1 + ref_x.abs())).max()))
            if Tn:
                got_r = resd[r0:r0 + Tn].float().cpu()
                worst_r = max(worst_r, float(((got_r - ref_res[r0:r0 + Tn]).abs()
                                              / (1 + ref_res[r0:r0 + Tn].abs())).max()))
        result_q.put((rank, (worst_x, worst_r), None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        result_q.put((rank, None, traceback.format_exc()))
