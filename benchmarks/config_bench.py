"""End-to-end benchmarks of the named serving workloads besides the headline one (``bench.py``).

    llama70b-fp8   Llama-3-70B, block-scaled fp8 (128x128 weight / 1x128 activation scales), TP=N:
                   decode batch 64 at context 4096 (4096-token prompts + 512 generated tokens), and
                   a prefill sweep of 1k / 4k / 8k-token prompts at batch 8
    mixtral-ep     Mixtral-8x7B bf16, expert parallel over the TP ranks: prefill of 16 x 2048 tokens,
                   then 256 decode steps at batch 128
    gguf-lora      Llama-3-8B with Q4_K linear weights and Q8_0 embedding / output, 64 rank-16 LoRA
                   adapters on q/k/v/o picked per request by Zipf(1.1); 512 requests, prompts
                   U[64, 1024], 128 output tokens

    python benchmarks/config_bench.py --workload gguf-lora
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/config_bench.py --workload llama70b-fp8

Weights are random (no checkpoints offline); token ids are uniform random; sampling is greedy with
EOS ignored. Every number is device time (CUDA events around the timed engine steps), max over
ranks; one JSON line per measurement on rank 0. For gguf-lora, one random layer is quantized to
Q4_K on the host and its blocks are copied into every layer (each layer still reads its own copy,
so the memory traffic per step is that of distinct layers; host quantization of all 8B weights
would take minutes).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--workload", required=True, choices=["llama70b-fp8", "mixtral-ep", "deepseek-ep", "gguf-lora"])
    p.add_argument("--model", default=None, help="preset override (small runs)")
    p.add_argument("--layers", type=int, default=0, help="override the layer count (small runs)")
    p.add_argument("--ffn", type=int, default=0, help="override the FFN width (small runs)")
    p.add_argument("--device", default="cuda")
    p.add_argument("--decode-steps", type=int, default=64)
    p.add_argument("--skip-prefill", action="store_true", help="llama70b-fp8: decode only, no prefill sweep")
    p.add_argument("--scale", type=float, default=1.0, help="shrink batch / lengths (small runs)")
    p.add_argument("--kv-cache-dtype", default="auto", choices=["auto", "fp8"],
                   help="llama70b-fp8: KV cache in the model dtype, or fp8 e4m3 with a scale per token and head")
    p.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                   help="TP collectives: fused P2P kernels over the IPC heap, or NCCL")
    return p.parse_args(argv)


class DeviceTimer:
    """Device time of a region (CUDA events; host clock on CPU), max over ranks."""

    def __init__(self, cuda: bool):
        self.cuda = cuda

    def __enter__(self):
        if self.cuda:
            torch.cuda.synchronize()
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e1 = torch.cuda.Event(enable_timing=True)
            self.e0.record()
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self.cuda:
            self.e1.record()
            torch.cuda.synchronize()
            ms = self.e0.elapsed_time(self.e1)
        else:
            ms = (time.perf_counter() - self.t0) * 1e3
        if torch.distributed.is_initialized():
            t = torch.tensor([ms], dtype=torch.float64, device="cuda" if self.cuda else "cpu")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t)
        self.ms = ms


def _emit(rank: int, rec: dict) -> None:
    if rank == 0:
        print(json.dumps(rec), flush=True)


def _engine(mcfg, ec_kw, weights=None, comm=None):
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine
    ec = EngineConfig(**ec_kw)
    return LLMEngine(ec, model_cfg=mcfg, weights=weights, comm=comm)


def _run_until_done(eng, ids):
    done = {}
    while len(done) < len(ids):
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o
    return done


def llama70b_fp8(args, di, comm):
    from gollek_b200.config import preset
    from gollek_b200.engine.sequence import SamplingParams
    cuda = args.device == "cuda"
    mcfg = preset(args.model or "llama-3-70b")
    if args.layers:
        mcfg.num_hidden_layers = args.layers
    if args.ffn:
        mcfg.intermediate_size = args.ffn
    B, ctx, gen = max(1, int(64 * args.scale)), max(16, int(4096 * args.scale)), max(16, int(512 * args.scale))
    kw = dict(model="llama-3-70b", device=args.device, dtype="bfloat16", quantization="fp8",
              tensor_parallel_size=di.world_size, max_num_seqs=max(B, 8), max_num_batched_tokens=8192,
              max_model_len=max(ctx + gen, int(8192 * args.scale) + 16) + 16, enable_prefix_caching=False,
              use_cuda_graphs=cuda, gpu_memory_utilization=0.9, kv_cache_dtype=args.kv_cache_dtype)
    eng = _engine(mcfg, kw, comm=comm)
    rng = np.random.default_rng(0)
    V = mcfg.vocab_size
    # decode batch B at context ctx: prefill untimed, then K timed decode steps
    sp = SamplingParams(temperature=0.0, max_tokens=gen, ignore_eos=True)
    for i in range(B):
        eng.add_request(f"d{i}", rng.integers(0, V, ctx).tolist(), SamplingParams(**vars(sp)))
    while any(s.num_computed_tokens < s.num_prompt_tokens for s in eng.scheduler.running) or eng.scheduler.waiting:
        eng.step()
    for _ in range(3):
        eng.step()
    K = max(1, min(args.decode_steps, gen - 8))
    with DeviceTimer(cuda) as t:
        n = sum(len(eng.step()) for _ in range(K))
    _emit(di.rank, {"workload": "llama70b-fp8-decode", "n_gpus": di.world_size, "batch": B, "context": ctx,
                    "steps": K, "tokens": n, "ms": round(t.ms, 2), "tok_s": round(n / t.ms * 1e3, 1),
                    "tpot_ms": round(t.ms / K, 3), "dtype": "fp8 (block-scaled weights and activations)",
                    "kv_cache_dtype": args.kv_cache_dtype,
                    "data": "synthetic, random-init"})
    for i in range(B):
        eng.abort_request(f"d{i}")
    while eng.has_unfinished():
        eng.step()
    # prefill sweep: batch 8 of L-token prompts, time until every first token is out
    for L in (() if args.skip_prefill else (1024, 4096, 8192)):
        L = max(16, int(L * args.scale))
        ids = [f"p{L}-{i}" for i in range(8)]
        for r in ids:
            eng.add_request(r, rng.integers(0, V, L).tolist(), SamplingParams(temperature=0.0, max_tokens=1,
                                                                             ignore_eos=True))
        with DeviceTimer(cuda) as t:
            _run_until_done(eng, ids)
        _emit(di.rank, {"workload": "llama70b-fp8-prefill", "n_gpus": di.world_size, "batch": 8, "prompt": L,
                        "ms": round(t.ms, 2), "prefill_tok_s": round(8 * L / t.ms * 1e3, 1),
                        "dtype": "fp8 (block-scaled)", "data": "synthetic, random-init"})


def mixtral_ep(args, di, comm):
    from gollek_b200.config import preset
    from gollek_b200.engine.sequence import SamplingParams
    cuda = args.device == "cuda"
    ds = args.workload == "deepseek-ep"
    mcfg = preset(args.model or ("deepseek-v3" if ds else "mixtral-8x7b"))
    name = "deepseek-v3-ep" if ds else "mixtral-ep"
    if args.layers:
        mcfg.num_hidden_layers = args.layers
    if args.ffn:
        mcfg.intermediate_size = args.ffn
    n_pf, L, B = max(1, int(16 * args.scale)), max(16, int(2048 * args.scale)), max(1, int(128 * args.scale))
    steps = max(4, min(int(256 * args.scale), args.decode_steps))  # timed decode steps (TPOT is per step)
    kw = dict(model="mixtral-8x7b", device=args.device, dtype="bfloat16", tensor_parallel_size=di.world_size,
              enable_expert_parallel=di.world_size > 1, max_num_seqs=max(B, n_pf), max_num_batched_tokens=8192,
              max_model_len=L + steps + 32, enable_prefix_caching=False, use_cuda_graphs=cuda,
              gpu_memory_utilization=0.9)
    eng = _engine(mcfg, kw, comm=comm)
    rng = np.random.default_rng(1)
    V = mcfg.vocab_size
    ids = [f"pf{i}" for i in range(n_pf)]
    for r in ids:
        eng.add_request(r, rng.integers(0, V, L).tolist(), SamplingParams(temperature=0.0, max_tokens=1,
                                                                         ignore_eos=True))
    with DeviceTimer(cuda) as t:
        _run_until_done(eng, ids)
    _emit(di.rank, {"workload": f"{name}-prefill", "layers": mcfg.num_hidden_layers, "n_gpus": di.world_size, "sequences": n_pf, "prompt": L,
                    "ms": round(t.ms, 2), "prefill_tok_s": round(n_pf * L / t.ms * 1e3, 1), "dtype": "bf16",
                    "parallelism": f"ep{di.world_size}+tp{di.world_size}", "data": "synthetic, random-init"})
    sp = SamplingParams(temperature=0.0, max_tokens=steps + 16, ignore_eos=True)
    for i in range(B):
        eng.add_request(f"dec{i}", rng.integers(0, V, 64).tolist(), SamplingParams(**vars(sp)))
    while eng.scheduler.waiting or any(s.num_computed_tokens < s.num_prompt_tokens for s in eng.scheduler.running):
        eng.step()
    with DeviceTimer(cuda) as t:
        n = sum(len(eng.step()) for _ in range(steps))
    _emit(di.rank, {"workload": f"{name}-decode", "layers": mcfg.num_hidden_layers, "n_gpus": di.world_size, "batch": B, "steps": steps,
                    "tokens": n, "ms": round(t.ms, 2), "tok_s": round(n / t.ms * 1e3, 1),
                    "tpot_ms": round(t.ms / steps, 3), "dtype": "bf16",
                    "parallelism": f"ep{di.world_size}+tp{di.world_size}", "data": "synthetic, random-init"})


def _gguf_weights(mcfg, seed=0):
    """Weights getter: Q4_K q/k/v/o/gate/up/down (one random layer's blocks in every layer), Q8_0
    embedding and output, bf16 norms."""
    from gollek_b200.loaders.gguf import GGML_Q4_K, GGML_Q8_0, QuantizedWeight
    from gollek_b200.native import host_ext
    h = host_ext()
    g = torch.Generator().manual_seed(seed)
    hs, q, kv, f, V = mcfg.hidden_size, mcfg.q_size, mcfg.kv_size, mcfg.intermediate_size, mcfg.vocab_size

    def quant(shape, qtype):
        x = torch.randn(*shape, generator=g) * 0.02
        raw = h.quantize_q4_k(x.reshape(-1)) if qtype == GGML_Q4_K else h.quantize_q8_0(x.reshape(-1))
        return QuantizedWeight(raw, tuple(shape), qtype)

    layer = {"self_attn.q_proj.weight": quant((q, hs), GGML_Q4_K), "self_attn.k_proj.weight": quant((kv, hs), GGML_Q4_K),
             "self_attn.v_proj.weight": quant((kv, hs), GGML_Q4_K), "self_attn.o_proj.weight": quant((hs, q), GGML_Q4_K),
             "mlp.gate_proj.weight": quant((f, hs), GGML_Q4_K), "mlp.up_proj.weight": quant((f, hs), GGML_Q4_K),
             "mlp.down_proj.weight": quant((hs, f), GGML_Q4_K)}
    top = {"model.embed_tokens.weight": quant((V, hs), GGML_Q8_0), "lm_head.weight": quant((V, hs), GGML_Q8_0),
           "model.norm.weight": torch.ones(hs)}

    def get(name):
        if name in top:
            return top[name]
        rest = name.split(".", 3)[3]  # model.layers.{i}.<rest>
        if rest.endswith("layernorm.weight"):
            return torch.ones(hs)
        w = layer[rest]
        return QuantizedWeight(w.raw.clone(), w.shape, w.ggml_type)  # each layer its own copy

    return get


def gguf_lora(args, di, comm):
    from gollek_b200.config import preset
    from gollek_b200.engine.sequence import SamplingParams
    cuda = args.device == "cuda"
    mcfg = preset(args.model or "llama-3-8b")
    if args.layers:
        mcfg.num_hidden_layers = args.layers
    if args.ffn:
        mcfg.intermediate_size = args.ffn
    n_req, pmin, pmax, out = max(4, int(512 * args.scale)), max(8, int(64 * args.scale)), \
        max(16, int(1024 * args.scale)), max(4, int(128 * args.scale))
    n_ad = max(2, int(64 * min(1.0, args.scale * 8)))
    kw = dict(model="llama-3-8b", device=args.device, dtype="bfloat16", quantization="gguf",
              tensor_parallel_size=di.world_size, enable_lora=True, max_loras=n_ad, max_lora_rank=16,
              max_num_seqs=256, max_num_batched_tokens=8192, max_model_len=pmax + out + 16,
              enable_prefix_caching=False, use_cuda_graphs=False, gpu_memory_utilization=0.9)
    eng = _engine(mcfg, kw, weights=_gguf_weights(mcfg), comm=comm)
    adapters = [eng.add_lora(f"ad{i}", seed=i, rank=16) for i in range(n_ad)]
    rng = np.random.default_rng(2)
    zipf = 1.0 / np.arange(1, n_ad + 1) ** 1.1
    zipf /= zipf.sum()
    V = mcfg.vocab_size
    ids = []
    for i in range(n_req):
        L = int(rng.integers(pmin, pmax + 1))
        a = adapters[int(rng.choice(n_ad, p=zipf))]
        eng.add_request(f"g{i}", rng.integers(0, V, L).tolist(),
                        SamplingParams(temperature=0.0, max_tokens=out, ignore_eos=True), lora_id=a)
        ids.append(f"g{i}")
    eng.metrics.ttft.clear()
    with DeviceTimer(cuda) as t:
        done = _run_until_done(eng, ids)
    n = sum(len(o.output_token_ids) for o in done.values())
    ttft = [1e3 * v for v in eng.metrics.ttft]  # host clock, all requests queued at t0
    _emit(di.rank, {"workload": "gguf-q4k-multilora", "n_gpus": di.world_size, "requests": n_req, "adapters": n_ad,
                    "tokens": n, "ms": round(t.ms, 2), "tok_s": round(n / t.ms * 1e3, 1),
                    "ttft_p50_ms": round(float(np.median(ttft)), 1) if ttft else None,
                    "dtype": "Q4_K linear / Q8_0 embedding+output, bf16 activations",
                    "data": "synthetic, random-init (one Q4_K layer copied into every layer)"})


def main(argv=None):
    args = parse(argv)
    from gollek_b200.parallel.dist import NcclComm, init_distributed
    cuda = args.device == "cuda"
    di = init_distributed(timeout_s=600)
    comm = None
    if cuda:
        torch.cuda.set_device(di.local_rank)
    if di.world_size > 1:
        if args.comm == "fused" and cuda:
            from gollek_b200.config import preset
            from gollek_b200.parallel.dist import cpu_group
            from gollek_b200.parallel.symm import FusedTPComm
            default = {"llama70b-fp8": "llama-3-70b", "mixtral-ep": "mixtral-8x7b", "deepseek-ep": "deepseek-v3",
                       "gguf-lora": "llama-3-8b"}
            hidden = preset(args.model or default[args.workload]).hidden_size
            comm = FusedTPComm(di.rank, di.world_size, max_tokens=8192 + 256, hidden=hidden, cpu_group=cpu_group())
        else:
            comm = NcclComm(di.rank, di.world_size)
    {"llama70b-fp8": llama70b_fp8, "mixtral-ep": mixtral_ep, "deepseek-ep": mixtral_ep,
     "gguf-lora": gguf_lora}[args.workload](args, di, comm)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
