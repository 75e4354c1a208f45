"""Per-rank body of the context-parallel attention test (gloo ranks on the CPU)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run_ring(rank, world, port, S, H, Hk, D, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        import torch
        import torch.distributed as dist
        from gollek_b200.parallel.context_parallel import full_causal_attention, ring_attention, split_sequence
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(11)
        qa, ka, va = (torch.randn(S, n, D, generator=g) for n in (H, Hk, Hk))
        ref = full_causal_attention(qa, ka, va, D ** -0.5)
        ql, pos = split_sequence(qa, world, rank)
        kl, _ = split_sequence(ka, world, rank)
        vl, _ = split_sequence(va, world, rank)
        out = ring_attention(ql, kl, vl, pos, D ** -0.5)
        err = float((out - ref[pos]).abs().max())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, err, None))
    except Exception:
        import traceback
        q.put((rank, None, traceback.format_exc()))
