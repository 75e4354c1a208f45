"""Self-check of the tensor-parallel path on the GPUs it runs on, against fp32 oracles.

Run by every rank (one process per GPU) before a multi-GPU benchmark, and by the multi-GPU tests:

* ``collectives_check`` — the fused all-reduce + residual + RMSNorm (one-shot and two-shot sizes,
  consecutive calls so buffer parities and epochs advance), the plain all-reduce, the
  vocab-parallel argmax and the vocab-parallel logits gather, each against the fp32 result computed from every rank's inputs
  (gathered in fp32 over the process group and summed in rank order).
* ``engine_check`` — a two-layer slice of the Llama-3-8B shape (or of Mixtral with its experts
  partitioned over the ranks) served by the TP engine (chunked prefill with a two-shot-sized
  step, then batched decode) whose greedy tokens are checked against the dense fp32 oracle: every
  chosen token's oracle logit, given the same history, must be within ``tol`` of the maximum;
  seeded top-k / top-p requests must draw the same tokens on every rank.

Both return plain dicts (JSON-ready) with the worst errors and an ``ok`` verdict that is the
same on every rank.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def _gather_sum_fp32(t: torch.Tensor, world: int, group=None) -> torch.Tensor:
    parts = [torch.empty_like(t, dtype=torch.float32) for _ in range(world)]
    dist.all_gather(parts, t.float().contiguous(), group=group)
    tot = torch.zeros_like(parts[0])
    for p in parts:
        tot += p
    return tot


def _agree(ok: bool, device) -> bool:
    f = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(f, op=dist.ReduceOp.MIN)
    return bool(f.item())


def collectives_check(comm, sizes=(1, 7, 64, 129, 300, 1024), vocab: int = 32000, seed: int = 0) -> dict:
    """Check ``comm`` (a ``FusedTPComm``) against fp32 oracles; sizes above its capacity are skipped."""
    from .. import ops
    rank, world, d = comm.rank, comm.size, comm.hidden
    dev = torch.device("cuda", torch.cuda.current_device())
    worst_x = worst_r = worst_ar = 0.0
    bad_argmax = 0
    for T in [t for t in sizes if t <= comm.max_tokens]:
        for rep in range(2):
            g = torch.Generator(device=dev).manual_seed(seed + 1000 * T + 10 * rep + rank)
            h = (torch.randn(T, d, device=dev, generator=g) * 0.5).bfloat16()
            gs = torch.Generator(device=dev).manual_seed(seed + 7 * T + rep)  # same on every rank
            res = torch.randn(T, d, device=dev, generator=gs).bfloat16()
            w = (torch.rand(d, device=dev, generator=gs) + 0.5).bfloat16()
            ref_res = res.float() + _gather_sum_fp32(h, world)
            ref_x = ref_res * torch.rsqrt(ref_res.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
            x = comm.allreduce_add_rmsnorm(h, res, w, 1e-5).float()
            rows = comm.residual_rows(T)
            # errors relative to magnitude (bf16 partials, one bf16 rounding of the sum)
            worst_x = max(worst_x, float(((x - ref_x).abs() / (1 + ref_x.abs())).max()))
            worst_r = max(worst_r, float(((res[rows].float() - ref_res[rows]).abs()
                                          / (1 + ref_res[rows].abs())).max()))
        t = torch.randn(T, d, device=dev, generator=g).bfloat16()
        ref = _gather_sum_fp32(t, world)
        out = comm.all_reduce(t).float()
        worst_ar = max(worst_ar, float(((out - ref).abs() / (1 + ref.abs())).max()))
    # sizes that are not whole hidden-width rows, and one past the partial buffer (chunked)
    for n in (8 * 1001, comm.max_tokens * d + 8 * 999):
        g = torch.Generator(device=dev).manual_seed(seed + n + rank)
        t = torch.randn(n, device=dev, generator=g).bfloat16()
        ref = _gather_sum_fp32(t, world)
        out = comm.all_reduce(t).float()
        worst_ar = max(worst_ar, float(((out - ref).abs() / (1 + ref.abs())).max()))
    for B in (1, 37, min(256, comm.max_tokens)):
        g = torch.Generator(device=dev).manual_seed(seed + 77 * B + rank)
        shard = torch.randn(B, vocab // world, device=dev, generator=g).bfloat16()
        if B > 1:
            shard[1, 5] = 50.0  # the same maximum on every rank: the lowest global id must win
        ids = comm.argmax_last(shard, rank * (vocab // world))
        full = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(full, shard)
        ref_ids = torch.cat(full, dim=1).float().argmax(-1)
        bad_argmax += int((ids != ref_ids).sum())
    # vocab-parallel logits gather: bit-exact against the process group's all-gather; row counts past
    # one buffer (chunked), fp32 shards (moved as bf16 units) and a shard width that is not a whole
    # number of 16-byte vectors (2-byte stores)
    bad_gather = 0
    comm.reserve_logits(vocab // world)
    per = getattr(comm, "lg_cap", 0) // (vocab // world * world * 2)
    cases = [(1, vocab // world, torch.bfloat16), (37, vocab // world, torch.bfloat16),
             (min(256, comm.max_tokens), vocab // world, torch.bfloat16), (5, vocab // world, torch.float32),
             (3, 1001, torch.bfloat16)]
    if per:
        cases.append((per + 3, vocab // world, torch.bfloat16))
    for B, v, dt in cases:
        g = torch.Generator(device=dev).manual_seed(seed + 131 * B + v + rank)
        shard = torch.randn(B, v, device=dev, generator=g).to(dt)
        got = comm.all_gather_last(shard).clone()
        full = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(full, shard)
        bad_gather += int((got != torch.cat(full, dim=1)).sum())
    comm.check()
    torch.cuda.synchronize()
    ok = worst_x < 0.02 and worst_r < 0.02 and worst_ar < 0.02 and bad_argmax == 0 and bad_gather == 0
    return {"max_rel_err_x": round(worst_x, 6), "max_rel_err_residual": round(worst_r, 6),
            "max_rel_err_allreduce": round(worst_ar, 6), "argmax_mismatches": bad_argmax,
            "logits_gather_mismatches": bad_gather,
            "nvls": bool(getattr(comm, "nvls", False)), "ok": _agree(ok, dev)}


def engine_check(comm_factory, layers: int = 2, vocab: int = 32000, new_tokens: int = 4,
                 prompt_lens=(150, 23, 5), tol_frac: float = 0.1, seed: int = 3,
                 group: Optional[object] = None, model: str = "llama-3-8b", expert_parallel: bool = False,
                 overrides: Optional[dict] = None) -> dict:
    """Serve a ``layers``-layer slice of ``model`` (vocabulary ``vocab``) at TP = world size with
    ``comm_factory(max_tokens, hidden)`` as the collectives (and, for MoE models with
    ``expert_parallel``, the experts partitioned over the ranks: the NVLink all-to-all when the comm
    has NVLS); compare the greedy tokens with the fp32 oracle (computed on rank 0's CPU).
    ``tol_frac`` scales the allowed logit gap by the oracle logits' standard deviation there."""
    from ..config import EngineConfig, preset
    from ..engine.engine import LLMEngine
    from ..engine.sequence import SamplingParams
    from ..models.reference import ReferenceDecoder, init_random_weights
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = preset(model, num_hidden_layers=layers, vocab_size=vocab, **(overrides or {}))
    w = init_random_weights(cfg, seed=seed)
    g = torch.Generator().manual_seed(seed)
    prompts = [torch.randint(0, vocab, (n,), generator=g).tolist() for n in prompt_lens]
    max_tokens = 512
    comm = comm_factory(max_tokens + 16, cfg.hidden_size)
    ec = EngineConfig(device="cuda", dtype="bfloat16", block_size=16, max_num_seqs=8,
                      max_num_batched_tokens=max_tokens, max_model_len=512, use_cuda_graphs=False,
                      tensor_parallel_size=world, enable_prefix_caching=False,
                      enable_expert_parallel=expert_parallel)
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, comm=comm, num_blocks=128)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=new_tokens, ignore_eos=True))
    if hasattr(comm, "check"):
        comm.check()
    ep_a2a = getattr(eng.model, "ep_a2a", None) is not None
    if ep_a2a:
        eng.model.ep_a2a.check()
    toks = [o.output_token_ids for o in outs]
    # sampled requests (the vocab shards gathered, then the same seeded draw on every rank)
    souts = eng.generate(prompts, SamplingParams(temperature=0.8, top_k=40, top_p=0.9, seed=11,
                                                 max_tokens=new_tokens, ignore_eos=True))
    if hasattr(comm, "check"):
        comm.check()
    stoks = [t for o in souts for t in o.output_token_ids]
    sflat = torch.tensor(stoks, dtype=torch.int64, device=dev)
    sall = [torch.empty_like(sflat) for _ in range(world)]
    dist.all_gather(sall, sflat)
    sampled_same = all(bool((a == sflat).all()) for a in sall) and len(stoks) == new_tokens * len(prompts)
    # every rank must hold the same tokens
    flat = torch.tensor([t for ts in toks for t in ts], dtype=torch.int64, device=dev)
    allt = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(allt, flat)
    same = all(bool((a == flat).all()) for a in allt)
    worst_gap_frac, near = 0.0, True
    if rank == 0:
        ref = ReferenceDecoder(cfg, w)
        for p, ts in zip(prompts, toks):
            logits = ref.forward(torch.tensor(p + ts))[len(p) - 1: len(p) - 1 + len(ts)]
            chosen = logits[torch.arange(len(ts)), torch.tensor(ts)]
            gap = (logits.max(-1).values - chosen) / logits.std(-1)
            worst_gap_frac = max(worst_gap_frac, float(gap.max()))
        near = worst_gap_frac <= tol_frac
    res = torch.tensor([worst_gap_frac], device=dev)
    dist.broadcast(res, 0)
    ok = _agree(same and sampled_same and (near if rank == 0 else True), dev)
    del eng
    torch.cuda.empty_cache()
    return {"model": model, "layers": layers, "prompt_lens": list(prompt_lens), "new_tokens": new_tokens,
            "expert_parallel": expert_parallel, "ep_all_to_all": ep_a2a,
            "ranks_agree": same, "sampled_ranks_agree": sampled_same, "max_logit_gap_over_std": round(float(res.item()), 5), "ok": ok}
