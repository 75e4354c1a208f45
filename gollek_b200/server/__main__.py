"""Start the HTTP server: ``python -m gollek_b200.server --model llama-3-8b --port 8000``.

With ``--tensor-parallel-size N`` launch under ``torchrun --nproc-per-node N``: every rank runs
the engine in lock-step (identical scheduling from identical inputs; rank 0 broadcasts each
step's new requests), and only rank 0 serves HTTP.
"""
from __future__ import annotations

import argparse
import os
import sys


def main(argv=None):
    ap = argparse.ArgumentParser(prog="gollek_b200.server")
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--config", default=None)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--served-model-name", default=None)
    ap.add_argument("--api-key", action="append", default=None)
    ap.add_argument("--device", default=None)
    ap.add_argument("--max-model-len", type=int, default=None)
    ap.add_argument("--max-num-seqs", type=int, default=None)
    ap.add_argument("--rate-limit", type=float, default=0.0, help="requests/s per API key (0 = off)")
    ap.add_argument("--tensor-parallel-size", type=int, default=None)
    ap.add_argument("--comm", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--speculative-method", choices=["none", "ngram", "draft"], default=None)
    ap.add_argument("--draft-model", default=None)
    ap.add_argument("--enable-expert-parallel", action="store_true")
    ap.add_argument("--asr-model", default=None, help="Whisper checkpoint directory for /v1/audio/*")
    ap.add_argument("--tts-model", default=None, help="SpeechT5 text-to-speech directory for /v1/audio/speech")
    ap.add_argument("--tts-vocoder", default=None, help="HiFi-GAN vocoder directory for /v1/audio/speech")
    ap.add_argument("--provider", action="append", default=[], metavar="ID=URL[,KEY]",
                    help="OpenAI-compatible upstream serving models this server does not (repeatable)")
    args = ap.parse_args(argv)
    import uvicorn
    from ..config import EngineConfig
    from ..engine.engine import LLMEngine
    from .app import create_app
    from .async_engine import AsyncEngine
    over = {"model": args.model}
    for k in ("device", "max_model_len", "max_num_seqs"):
        if getattr(args, k) is not None:
            over[k] = getattr(args, k)
    if args.device == "cpu":
        over.update(dtype="float32", use_cuda_graphs=False)
    for k in ("speculative_method", "draft_model"):
        if getattr(args, k) is not None:
            over[k] = getattr(args, k)
    if args.enable_expert_parallel:
        over["enable_expert_parallel"] = True
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.tensor_parallel_size is not None and args.tensor_parallel_size != world:
        raise SystemExit(f"--tensor-parallel-size {args.tensor_parallel_size} needs torchrun with "
                         f"--nproc-per-node {args.tensor_parallel_size} (WORLD_SIZE={world})")
    over["tensor_parallel_size"] = world
    cfg = EngineConfig.load(args.config, **over)
    keys = args.api_key or [k for k in os.environ.get("GOLLEK_API_KEYS", "").split(",") if k]
    if world > 1:
        return _serve_tp(args, cfg, keys)
    ae = AsyncEngine(LLMEngine(cfg)).start()
    app = create_app(ae, model_name=args.served_model_name or os.path.basename(args.model.rstrip("/")),
                     api_keys=keys, rate=args.rate_limit, asr=_asr(args, cfg), tts=_tts(args, cfg),
                     providers=parse_providers(args.provider))
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="info")
    finally:
        ae.shutdown(drain=True)


def _asr(args, cfg):
    """The speech model behind /v1/audio/* (on rank 0's device), or None."""
    if not args.asr_model:
        return None
    import torch
    from ..models.whisper import WhisperASR
    dev = str(cfg.device)
    return WhisperASR(args.asr_model, device=dev, dtype=torch.float32 if dev == "cpu" else torch.bfloat16)


def parse_providers(specs):
    """``ID=URL[,KEY]`` strings -> a registry of OpenAI-compatible upstreams."""
    from .providers import OpenAIHTTPProvider, ProviderRegistry
    reg = ProviderRegistry()
    for spec in specs or []:
        pid, eq, rest = spec.partition("=")
        if not eq or not pid or not rest:
            raise SystemExit(f"--provider {spec!r}: expected ID=URL[,KEY]")
        url, _, key = rest.partition(",")
        reg.register(OpenAIHTTPProvider(pid, url, key))
    return reg


def _tts(args, cfg):
    """The text-to-speech model behind /v1/audio/speech (on rank 0's device), or None."""
    if not args.tts_model:
        return None
    if not args.tts_vocoder:
        raise SystemExit("--tts-model needs --tts-vocoder (a HiFi-GAN checkpoint directory)")
    import torch
    from ..models.speecht5 import SpeechSynth
    dev = str(cfg.device)
    return SpeechSynth(args.tts_model, args.tts_vocoder, device=dev,
                       dtype=torch.float32 if dev == "cpu" else torch.bfloat16)


def _serve_tp(args, cfg, keys):
    """One process per GPU: rank 0 serves HTTP through a DriverEngine that publishes every step's
    request events; the other ranks follow those events in lock-step."""
    import torch.distributed as dist
    import uvicorn
    from ..engine.engine import LLMEngine
    from ..parallel.control import ControlPlane, DriverEngine, follow
    from ..parallel.dist import NcclComm, cpu_group, init_distributed
    from .app import create_app
    from .async_engine import AsyncEngine
    from ..engine.engine import load_model_source
    di = init_distributed(timeout_s=120)
    mc, weights, tok = load_model_source(str(cfg.model), keep_quantized=cfg.quantization == "gguf")
    if args.comm == "fused" and cfg.device != "cpu":
        from ..parallel.symm import FusedTPComm
        comm = FusedTPComm(di.rank, di.world_size, max_tokens=cfg.max_num_batched_tokens + cfg.max_num_seqs,
                           hidden=mc.hidden_size, cpu_group=cpu_group())
    else:
        comm = NcclComm(di.rank, di.world_size)
    engine = LLMEngine(cfg, model_cfg=mc, weights=weights, comm=comm, tokenizer=tok)
    store = dist.distributed_c10d._get_default_store()
    cp = ControlPlane(di.rank, di.world_size, store, timeout_s=3600.0).start_heartbeat()
    try:
        if di.rank != 0:
            follow(engine, cp)
            return
        drv = DriverEngine(engine, cp)
        ae = AsyncEngine(drv).start()
        app = create_app(ae, model_name=args.served_model_name or os.path.basename(str(args.model).rstrip("/")),
                         api_keys=keys, rate=args.rate_limit, asr=_asr(args, cfg), tts=_tts(args, cfg),
                         providers=parse_providers(args.provider))
        try:
            uvicorn.run(app, host=args.host, port=args.port, log_level="info")
        finally:
            ae.shutdown(drain=True)
            drv.shutdown_workers()
    finally:
        cp.stop()
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1:])
