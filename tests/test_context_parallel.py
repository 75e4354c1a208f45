"""Context-parallel (ring) attention over gloo ranks on the CPU equals full causal attention."""
import multiprocessing as mp
import socket

import pytest
import torch


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_zigzag_layout_balances_causal_work():
    from gollek_b200.parallel.context_parallel import zigzag_indices
    S, W = 64, 4
    parts = [zigzag_indices(S, W, r) for r in range(W)]
    assert sorted(torch.cat(parts).tolist()) == list(range(S))
    work = [int((p + 1).sum()) for p in parts]  # keys visible to each rank's queries
    assert max(work) == min(work)


@pytest.mark.parametrize("world,H,Hk", [(2, 4, 2), (3, 2, 2)])
def test_ring_attention_matches_full_attention(world, H, Hk):
    from tests.cp_worker import run_ring
    S, D = 12 * world, 16
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_ring, args=(r, world, port, S, H, Hk, D, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err, tb in res:
        assert tb is None, tb
        assert err < 1e-5, (rank, err)
