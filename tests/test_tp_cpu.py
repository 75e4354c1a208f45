"""Tensor parallelism on CPU ranks (gloo, world size 2): sharded model == single-process oracle."""
import multiprocessing as mp
import socket

import torch

from gollek_b200.models.reference import ReferenceDecoder


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tp2_gloo_matches_oracle(tiny_cfg, tiny_weights):
    from tests.tp_worker import run_tp
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 33)]
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    expect = [ref.greedy(p, 6)[0] for p in prompts]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_tp, args=(r, 2, port, "gloo", "nccl", prompts, 6, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, toks, err in res:
        assert err is None, err
        assert toks == expect, (rank, toks, expect)
