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
    cfg = EngineConfig.load(args.config, **over)
    keys = args.api_key or [k for k in os.environ.get("GOLLEK_API_KEYS", "").split(",") if k]
    ae = AsyncEngine(LLMEngine(cfg)).start()
    app = create_app(ae, model_name=args.served_model_name or os.path.basename(args.model.rstrip("/")),
                     api_keys=keys, rate=args.rate_limit)
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="info")
    finally:
        ae.shutdown(drain=True)


if __name__ == "__main__":
    main(sys.argv[1:])
