"""Worker body shared by the multi-process tensor-parallel tests (spawned per rank)."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run_tp(rank, world, port, backend, comm_kind, prompts, max_tokens, result_q, num_layers=None,
           model="tiny-llama", expert_parallel=False):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                       LOCAL_RANK=str(rank))
    try:
        from gollek_b200.config import EngineConfig, preset
        from gollek_b200.engine.engine import LLMEngine
        from gollek_b200.engine.sequence import SamplingParams
        from gollek_b200.models.reference import init_random_weights
        from gollek_b200.parallel.dist import NcclComm, init_distributed, cpu_group
        init_distributed(backend=backend, timeout_s=60)
        cfg = preset(model)
        if num_layers:
            cfg.num_hidden_layers = num_layers
        w = init_random_weights(cfg, seed=0)
        dev = "cuda" if backend == "nccl" else "cpu"
        if comm_kind == "fused":
            from gollek_b200.parallel.symm import FusedTPComm
            comm = FusedTPComm(rank, world, max_tokens=512, hidden=cfg.hidden_size, cpu_group=cpu_group(),
                               one_shot_max_tokens=8)
        else:
            comm = NcclComm(rank, world)
        ec = EngineConfig(device=dev, dtype="bfloat16" if dev == "cuda" else "float32", block_size=16,
                          max_num_seqs=8, max_num_batched_tokens=256, max_model_len=512,
                          use_cuda_graphs=False, tensor_parallel_size=world,
                          enable_expert_parallel=expert_parallel)
        eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, comm=comm, num_blocks=128)
        outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True))
        if comm_kind == "fused":
            comm.check()
        result_q.put((rank, [o.output_token_ids for o in outs], None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        import traceback
        result_q.put((rank, None, traceback.format_exc()))


def run_ep_rebalance(rank, world, port, prompts, max_tokens, result_q, model):
    """EP engine on gloo: generate, force a skewed re-placement (experts moved between ranks), generate
    again; then an engine that rebalances every step from its tracked loads."""
    import torch.distributed as dist
    import numpy as np
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        from gollek_b200.config import EngineConfig, preset
        from gollek_b200.engine.engine import LLMEngine
        from gollek_b200.engine.sequence import SamplingParams
        from gollek_b200.models.reference import init_random_weights
        from gollek_b200.parallel.dist import NcclComm, init_distributed
        init_distributed(backend="gloo", timeout_s=60)
        cfg = preset(model)
        w = init_random_weights(cfg, seed=0)
        sp = SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)

        def engine(interval=0):
            ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=8,
                              max_num_batched_tokens=256, max_model_len=512, use_cuda_graphs=False,
                              tensor_parallel_size=world, enable_expert_parallel=True,
                              ep_rebalance_interval=interval)
            return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, comm=NcclComm(rank, world), num_blocks=128)

        eng = engine()
        first = [o.output_token_ids for o in eng.generate(prompts, sp)]
        E = cfg.num_local_experts
        skew = {li: np.linspace(100.0, 1.0, E) for li, L in enumerate(eng.model.layers) if "moe_gu" in L}
        rep = eng.model.rebalance_experts(loads=skew)
        moved = sum(r["moved"] for r in rep.values())
        second = [o.output_token_ids for o in eng.generate(prompts, sp)]
        eng2 = engine(interval=1)
        third = [o.output_token_ids for o in eng2.generate(prompts, sp)]
        result_q.put((rank, (first, second, third, moved, len(eng2.ep_reports)), None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        result_q.put((rank, None, traceback.format_exc()))
